"""Prefill over host buffers (gdn_prefill_host): the token axis cut into
segments whose copies in and out overlap the prefill of their neighbours.

Each segment is a prefill call whose state comes from the previous segment in
fp32 and whose boundaries are chunk boundaries, so the result must equal
gdn_prefill_fwd on the whole sequence bit for bit, whatever the segment length;
and the oracle's within the prefill bar (bf16 o max-abs <= 2e-2, fp32 state
relative Frobenius <= 1e-3)."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import max_abs, to_dev, to_np

pytestmark = pytest.mark.gpu


def _host(x, pin=True):
    """numpy -> torch CPU tensor (bf16 for uint16 bit patterns), pinned by default."""
    import torch
    t = to_dev(x, "cpu")
    return t.pin_memory() if pin else t


def _device_prefill(inp, layout, mask, dt_bias):
    import torch
    from gdn_18646_b200 import ops
    o, s = ops.prefill(to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]),
                       to_dev(inp["a"]), to_dev(inp["b"]), dt_bias=dt_bias,
                       mask=None if mask is None else to_dev(mask),
                       state_in=None if inp["state_in"] is None else to_dev(inp["state_in"]),
                       scale=inp["scale"], layout=layout)
    torch.cuda.synchronize()
    return to_np(o), to_np(s)


def _host_prefill(inp, layout, mask, dt_bias, seg, pin=True):
    from gdn_18646_b200 import ops
    o, s = ops.prefill_host(_host(inp["q"], pin), _host(inp["k"], pin), _host(inp["v"], pin),
                            _host(inp["A_log"], pin), _host(inp["a"], pin), _host(inp["b"], pin),
                            dt_bias=dt_bias, mask=None if mask is None else _host(mask, pin),
                            state_in=None if inp["state_in"] is None else _host(inp["state_in"], pin),
                            scale=inp["scale"], layout=layout, seg_tokens=seg)
    assert not o.is_cuda and not s.is_cuda
    return to_np(o), to_np(s)


@pytest.mark.parametrize("seg", [0, 64, 256, 4096])
def test_host_equals_device_prefill(cuda_device, seg):
    inp = O.make_prefill_inputs(11, 2, 1000, 4, 128, 128, gate_dtype="f32", state_std=0.02)
    want_o, want_s = _device_prefill(inp, "bhtd", None, 0.0)
    got_o, got_s = _host_prefill(inp, "bhtd", None, 0.0, seg)
    assert np.array_equal(got_o, want_o)
    assert np.array_equal(got_s, want_s)


def test_host_bthd_grouped_mask_bf16_gates(cuda_device):
    import torch
    inp = O.make_prefill_inputs(12, 2, 700, 8, 128, 128, gate_dtype="bf16", state_std=0.02, layout="bthd", Hqk=4)
    rng = np.random.default_rng(3)
    mask = (rng.random((2, 700)) > 0.2).astype(np.float32)
    dtb = rng.standard_normal(8).astype(np.float32) * 0.5
    want_o, want_s = _device_prefill(inp, "bthd", mask, to_dev(dtb))
    from gdn_18646_b200 import ops
    o, s = ops.prefill_host(_host(inp["q"]), _host(inp["k"]), _host(inp["v"]), _host(inp["A_log"]),
                            _host(inp["a"]), _host(inp["b"]), dt_bias=_host(dtb), mask=_host(mask),
                            state_in=_host(inp["state_in"]), scale=inp["scale"], layout="bthd", seg_tokens=128)
    assert np.array_equal(to_np(o), want_o)
    assert np.array_equal(to_np(s), want_s)


def test_host_matches_oracle_without_state(cuda_device):
    inp = O.make_prefill_inputs(13, 1, 300, 2, 64, 128, gate_dtype="f32", state_std=0.0)
    got_o, got_s = _host_prefill(inp, "bhtd", None, 0.0, 128)
    want_o, want_s = O.prefill(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], 0.0, inp["b"], inp["mask"],
                               state_in=None, scale=inp["scale"])
    assert max_abs(got_o, want_o) <= 2e-2
    assert np.linalg.norm(got_s - want_s) <= 1e-3 * np.linalg.norm(want_s)


def test_host_accepts_pageable_and_device_tensors(cuda_device):
    import torch
    from gdn_18646_b200 import ops
    inp = O.make_prefill_inputs(14, 1, 200, 2, 128, 128, gate_dtype="f32", state_std=0.02)
    want_o, want_s = _device_prefill(inp, "bhtd", None, 0.0)
    got_o, got_s = _host_prefill(inp, "bhtd", None, 0.0, 64, pin=False)
    assert np.array_equal(got_o, want_o) and np.array_equal(got_s, want_s)
    # device inputs and device outputs go through the same copies (device to device)
    o_d = torch.empty(to_dev(inp["v"]).shape, dtype=torch.bfloat16, device="cuda")
    s_d = torch.empty(1, 2, 128, 128, dtype=torch.float32, device="cuda")
    ops.prefill_host(to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]),
                     to_dev(inp["a"]), to_dev(inp["b"]), state_in=to_dev(inp["state_in"]), scale=inp["scale"],
                     out=o_d, state_out=s_d, seg_tokens=64)
    assert np.array_equal(to_np(o_d), want_o) and np.array_equal(to_np(s_d), want_s)


def test_host_back_to_back_calls_keep_order(cuda_device):
    """Two calls without a synchronisation between them reuse the library's copy
    streams and events; each must still see only its own inputs."""
    import torch
    from gdn_18646_b200 import ops
    i1 = O.make_prefill_inputs(15, 2, 512, 4, 128, 128, gate_dtype="f32", state_std=0.02)
    i2 = O.make_prefill_inputs(16, 2, 512, 4, 128, 128, gate_dtype="f32", state_std=0.02)
    w1, w2 = _device_prefill(i1, "bhtd", None, 0.0), _device_prefill(i2, "bhtd", None, 0.0)
    outs, keep = [], []                      # host inputs stay alive until the stream completes
    for inp in (i1, i2):
        hin = [_host(inp[n]) for n in ("q", "k", "v", "A_log", "a", "b", "state_in")]
        keep.append(hin)
        outs.append(ops.prefill_host(*hin[:6], state_in=hin[6], scale=inp["scale"], seg_tokens=64,
                                     synchronize=False))
    torch.cuda.synchronize()
    for (o, s), (wo, ws) in zip(outs, (w1, w2)):
        assert np.array_equal(to_np(o), wo) and np.array_equal(to_np(s), ws)


def test_host_rejects_bad_segment(cuda_device):
    from gdn_18646_b200 import ops
    inp = O.make_prefill_inputs(17, 1, 128, 2, 128, 128, gate_dtype="f32")
    with pytest.raises(RuntimeError, match="seg_tokens"):
        ops.prefill_host(_host(inp["q"]), _host(inp["k"]), _host(inp["v"]), _host(inp["A_log"]),
                         _host(inp["a"]), _host(inp["b"]), scale=inp["scale"], seg_tokens=100)
