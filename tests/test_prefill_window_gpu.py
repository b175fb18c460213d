"""The windowed prefill (gdn_prefill_window_ws): a call over the tokens
[t0, t0 + Tw) of whole tensors, reading q, k, v, gates and mask in place and
writing o into the same tokens of the output.  Windows chained through their
fp32 states, every start on a 64-token chunk boundary, must equal one call over
the whole sequence bit for bit; tokens outside the window must stay untouched."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import to_dev, to_np

pytestmark = pytest.mark.gpu


def _whole(inp, layout, mask, dt_bias):
    import torch
    from gdn_18646_b200 import ops
    o, s = ops.prefill(to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]),
                       to_dev(inp["a"]), to_dev(inp["b"]), dt_bias=dt_bias, mask=mask,
                       state_in=None if inp["state_in"] is None else to_dev(inp["state_in"]),
                       scale=inp["scale"], layout=layout)
    torch.cuda.synchronize()
    return to_np(o), to_np(s)


def _windowed(inp, layout, mask, dt_bias, plan, fill=None):
    import torch
    from gdn_18646_b200 import ops
    q, k, v = to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"])
    out = torch.empty_like(v) if fill is None else torch.full_like(v, fill)
    s = None if inp["state_in"] is None else to_dev(inp["state_in"])
    B = v.shape[0]
    Hv, dv = (v.shape[1], v.shape[3]) if layout == "bhtd" else (v.shape[2], v.shape[3])
    for t0, tw in plan:
        s_out = torch.empty(B, Hv, q.shape[-1], dv, dtype=torch.float32, device="cuda")
        ops.prefill_window(q, k, v, to_dev(inp["A_log"]), to_dev(inp["a"]), to_dev(inp["b"]), t0, tw, out=out,
                           dt_bias=dt_bias, mask=mask, state_in=s, state_out=s_out, scale=inp["scale"],
                           layout=layout)
        s = s_out
    torch.cuda.synchronize()
    return to_np(out), to_np(s)


@pytest.mark.parametrize("plan", [[(0, 1000)], [(0, 512), (512, 488)], [(0, 64), (64, 640), (704, 296)],
                                  [(i, min(128, 1000 - i)) for i in range(0, 1000, 128)]])
def test_windows_equal_whole_call(cuda_device, plan):
    inp = O.make_prefill_inputs(21, 2, 1000, 4, 128, 128, gate_dtype="f32", state_std=0.02)
    want_o, want_s = _whole(inp, "bhtd", None, 0.0)
    got_o, got_s = _windowed(inp, "bhtd", None, 0.0, plan)
    assert np.array_equal(got_o, want_o)
    assert np.array_equal(got_s, want_s)


def test_windows_bthd_grouped_mask_bf16_gates(cuda_device):
    inp = O.make_prefill_inputs(22, 2, 700, 8, 128, 128, gate_dtype="bf16", state_std=0.02, layout="bthd", Hqk=4)
    rng = np.random.default_rng(5)
    mask = to_dev((rng.random((2, 700)) > 0.2).astype(np.float32))
    dtb = to_dev(rng.standard_normal(8).astype(np.float32) * 0.5)
    want_o, want_s = _whole(inp, "bthd", mask, dtb)
    got_o, got_s = _windowed(inp, "bthd", mask, dtb, [(0, 192), (192, 128), (320, 380)])
    assert np.array_equal(got_o, want_o)
    assert np.array_equal(got_s, want_s)


def test_window_touches_only_its_tokens(cuda_device):
    """One window in the middle: o outside [t0, t0 + Tw) keeps the fill value, o
    inside equals a whole call on the sliced tensors with the same start state."""
    import torch
    from gdn_18646_b200 import ops
    inp = O.make_prefill_inputs(23, 1, 640, 2, 64, 128, gate_dtype="f32", state_std=0.02)
    t0, tw = 256, 200
    got_o, got_s = _windowed(inp, "bhtd", None, 0.0, [(t0, tw)], fill=3.0)
    fill = 0x4040                                         # bf16 bits of 3.0
    assert np.all(got_o[:, :, :t0] == fill) and np.all(got_o[:, :, t0 + tw:] == fill)
    sl = {n: np.ascontiguousarray(inp[n][..., t0:t0 + tw, :]) for n in ("q", "k", "v")}
    sl.update({n: np.ascontiguousarray(inp[n][..., t0:t0 + tw]) for n in ("a", "b")})
    o, s = ops.prefill(to_dev(sl["q"]), to_dev(sl["k"]), to_dev(sl["v"]), to_dev(inp["A_log"]), to_dev(sl["a"]),
                       to_dev(sl["b"]), state_in=to_dev(inp["state_in"]), scale=inp["scale"])
    torch.cuda.synchronize()
    assert np.array_equal(got_o[:, :, t0:t0 + tw], to_np(o))
    assert np.array_equal(got_s, to_np(s))


def test_window_rejects_outside(cuda_device):
    import torch
    from gdn_18646_b200 import ops
    inp = O.make_prefill_inputs(24, 1, 128, 2, 128, 128, gate_dtype="f32")
    v = to_dev(inp["v"])
    with pytest.raises(RuntimeError, match="window"):
        ops.prefill_window(to_dev(inp["q"]), to_dev(inp["k"]), v, to_dev(inp["A_log"]), to_dev(inp["a"]),
                           to_dev(inp["b"]), 64, 128, out=torch.empty_like(v))
