"""RMSNorm / gated RMSNorm parity vs the reference goldens and the oracle."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import load_golden, to_dev, to_np

pytestmark = pytest.mark.gpu


def _ulp_ok(got, want, max_frac_diff=0.01):
    g, w = O.bf16_to_f32(got), O.bf16_to_f32(want)
    assert np.all(np.abs(g - w) <= np.abs(w) * 2.0 ** -7 + 1e-6), "more than 1 bf16 ulp apart"
    assert np.mean(g != w) <= max_frac_diff


@pytest.mark.parametrize("name", ["rmsnorm_2048", "rmsnorm_512"])
def test_rmsnorm_golden(cuda_device, name):
    import torch
    from gdn_18646_b200 import ops
    g = load_golden(name)
    y = ops.rmsnorm(to_dev(g["x"]), to_dev(g["gamma"]), float(g["eps"]))
    torch.cuda.synchronize()
    _ulp_ok(to_np(y), g["y"])


@pytest.mark.parametrize("R,D", [(1, 2048), (37, 2048), (1000, 128), (17, 4096), (3, 8192), (5, 8), (64, 1024)])
def test_rmsnorm_vs_oracle(cuda_device, R, D):
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(R * 7 + D)
    x = O.f32_to_bf16(rng.standard_normal((R, D), dtype=np.float32))
    gamma = O.f32_to_bf16(1 + 0.1 * rng.standard_normal(D, dtype=np.float32))
    y = ops.rmsnorm(to_dev(x), to_dev(gamma), 1e-6)
    torch.cuda.synchronize()
    _ulp_ok(to_np(y), O.rmsnorm(x, gamma, 1e-6))


def test_rmsnorm_reference_test_sizes_vs_fp32_torch(cuda_device):
    """tests/test_rmsnorm.py:25-52: fp32 nn.RMSNorm ground truth, max-abs < 5e-2, rel < 0.02."""
    import torch
    import gdn_18646_b200 as G
    ext = G.exts()["rmsnorm"]
    for B, T in ((1, 1), (8, 2048), (32, 4096)):
        x = torch.randn(B * T, 2048, device="cuda", dtype=torch.bfloat16)
        gamma = torch.ones(2048, device="cuda", dtype=torch.bfloat16)
        y = ext.forward(x, gamma, 1e-6, 256, 2)
        ref = torch.nn.functional.rms_norm(x.float(), (2048,), torch.ones(2048, device="cuda"), 1e-6)
        diff = (y.float() - ref).abs()
        assert diff.max().item() < 5e-2
        assert (diff / (ref.abs() + 1e-8)).max().item() < 0.02


@pytest.mark.parametrize("xdt", ["bf16", "f32"])
@pytest.mark.parametrize("R,D", [(64, 128), (9, 256), (3, 2048)])
def test_gated_rmsnorm_vs_oracle(cuda_device, xdt, R, D):
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(R + D)
    xf = rng.standard_normal((R, D), dtype=np.float32)
    x = O.f32_to_bf16(xf) if xdt == "bf16" else xf
    z = O.f32_to_bf16(rng.standard_normal((R, D), dtype=np.float32))
    gamma = O.f32_to_bf16(1 + 0.1 * rng.standard_normal(D, dtype=np.float32))
    y = ops.gated_rmsnorm(to_dev(x), to_dev(z), to_dev(gamma), 1e-6)
    torch.cuda.synchronize()
    _ulp_ok(to_np(y), O.gated_rmsnorm(x, z, gamma, 1e-6), max_frac_diff=0.02)
