"""The comparator recipe (oracle/build_ref_kernels.py) without a GPU: the module
names, where the built extensions go, and that each built module imports and
exposes the reference's entry point (kernels/decode.cu:216-217,
kernels/rmsnorm.cu:295-297, kernels/fused_proj_conv_silu.cu:357-358,
kernels/prefill_chunked.cu:509-526).  Skipped per module when it was not built."""
import os

import pytest

from oracle import build_ref_kernels as R

ENTRY = {"gdn_ref_decode": "forward", "gdn_ref_rmsnorm": "forward", "gdn_ref_proj": "forward",
         "gdn_ref_prefill": "prefill"}


def test_recipe_covers_the_reference_kernels():
    assert set(R.KERNELS) == set(ENTRY)
    assert {src for src, _ in R.KERNELS.values()} == {"decode.cu", "rmsnorm.cu", "fused_proj_conv_silu.cu",
                                                      "prefill_chunked.cu"}
    assert os.path.basename(R.OUT) == "_ref" and os.path.dirname(R.OUT) == R.HERE


@pytest.mark.parametrize("name", sorted(ENTRY))
def test_built_module_imports(name):
    if R.so_path(name) is None:
        pytest.skip(f"{name} not built")
    assert os.path.dirname(os.path.dirname(R.so_path(name))) == R.OUT
    mod = R.load(name)
    assert callable(getattr(mod, ENTRY[name]))
    if name == "gdn_ref_prefill":                  # the head shape it is compiled for
        assert (mod.H_DIM, mod.K_DIM, mod.V_DIM, mod.C_DIM) == (16, 128, 256, 64)
