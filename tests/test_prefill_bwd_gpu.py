"""Prefill backward (gdn_prefill_bwd) against the oracle's hand-written
derivative (oracle prefill_backward, itself pinned to finite differences),
in float64 on the same bf16-quantised inputs, for both algorithms: the
chunked one (tcgen05 products on bf16 hi/lo operands, fp32 accumulation) and
the token-recurrent one (fp32 on CUDA cores).  Every gradient must match to a
relative max error of 1e-3 of its own magnitude."""
import math

import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import to_dev, to_np

pytestmark = pytest.mark.gpu


def _rel(got, want):
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-12))


@pytest.mark.parametrize("algorithm,window", [("token", None), ("token", 32), ("chunked", None)])
@pytest.mark.parametrize("B,H,T,dk,dv,do_bf16", [(2, 2, 100, 64, 64, False), (1, 3, 130, 128, 128, True),
                                                  (1, 2, 70, 128, 64, False), (2, 1, 65, 64, 128, True)])
def test_prefill_bwd_vs_oracle(cuda_device, B, H, T, dk, dv, do_bf16, algorithm, window):
    """window=32 runs the token-recurrent backward in several token windows (the last one
    ragged) from checkpoints of the state at every window start; "chunked" runs the
    64-token chunk form (every T here ends in a ragged chunk).  The mask zeroes tokens
    inside a chunk as well as at the end."""
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(B * 100 + T + dk + dv)
    inp = O.make_prefill_inputs(7 + T, B, T, H, dk, dv, gate_dtype="f32", state_std=0.05)
    mask = np.ones((B, T), np.float32)
    mask[:, T - 3:] = 0.0
    mask[0, 20:23] = 0.0
    dtb = (rng.standard_normal(H) * 0.2).astype(np.float32)
    dO = rng.standard_normal((B, H, T, dv)).astype(np.float32)
    if do_bf16:
        dO = O.bf16_to_f32(O.f32_to_bf16(dO))
    dSf = (rng.standard_normal((B, H, dk, dv)) * 0.1).astype(np.float32)
    ref = O.prefill_backward(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], dtb, inp["b"], mask, dO,
                             state_in=inp["state_in"], dS_final=dSf, scale=inp["scale"])
    dO_t = to_dev(dO)
    if do_bf16:
        dO_t = dO_t.bfloat16()
    got = ops.prefill_backward(to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]),
                               to_dev(inp["a"]), to_dev(inp["b"]), dO_t, dt_bias=to_dev(dtb), mask=to_dev(mask),
                               state_in=to_dev(inp["state_in"]), dS_final=to_dev(dSf), scale=inp["scale"],
                               window=window, algorithm=algorithm)
    torch.cuda.synchronize()
    for name in ("dq", "dk", "dv", "da", "db", "dA_log", "ddt_bias", "dstate_in"):
        err = _rel(to_np(got[name]).astype(np.float64), ref[name])
        assert err < 1e-3, f"{name}: relative max error {err:.2e}"


@pytest.mark.parametrize("algorithm", ["token", "chunked"])
def test_prefill_bwd_scalar_dt_bias_and_no_state(cuda_device, algorithm):
    """Scalar dt_bias (its gradient summed over heads), no initial state, no mask,
    no final-state gradient, T a multiple of the chunk."""
    import torch
    from gdn_18646_b200 import ops
    B, H, T, dk, dv = 1, 2, 128, 64, 64
    inp = O.make_prefill_inputs(3, B, T, H, dk, dv, gate_dtype="f32")
    rng = np.random.default_rng(4)
    dO = rng.standard_normal((B, H, T, dv)).astype(np.float32)
    ref = O.prefill_backward(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], 0.3, inp["b"], np.ones((B, T)),
                             dO, scale=inp["scale"])
    got = ops.prefill_backward(to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]),
                               to_dev(inp["a"]), to_dev(inp["b"]), to_dev(dO), dt_bias=0.3, scale=inp["scale"],
                               algorithm=algorithm)
    torch.cuda.synchronize()
    assert _rel(float(got["ddt_bias"]), np.array(ref["ddt_bias"].sum())) < 1e-3
    for name in ("dq", "dk", "dv", "da", "db", "dstate_in"):
        assert _rel(to_np(got[name]).astype(np.float64), ref[name]) < 1e-3, name


def test_prefill_autograd_function(cuda_device):
    """PrefillFunction: torch autograd through the forward kernel and the backward
    kernels gives prefill_backward's gradients (cast to the inputs' dtypes)."""
    import torch
    from gdn_18646_b200 import ops
    B, H, T, dk, dv = 1, 2, 96, 64, 64
    inp = O.make_prefill_inputs(21, B, T, H, dk, dv, gate_dtype="f32", state_std=0.05)
    t = {n: to_dev(inp[n]) for n in ("q", "k", "v", "A_log", "a", "b", "state_in")}
    dtb = torch.tensor([0.1, -0.2], device="cuda")
    leaves = {n: x.clone().requires_grad_(True) for n, x in t.items()}
    dtb_l = dtb.clone().requires_grad_(True)
    o, S = ops.prefill_autograd(leaves["q"], leaves["k"], leaves["v"], leaves["A_log"], leaves["a"], leaves["b"],
                                dtb_l, leaves["state_in"], inp["scale"])
    rng = np.random.default_rng(5)
    dO = to_dev(rng.standard_normal((B, H, T, dv)).astype(np.float32))
    (o.float() * dO).sum().backward()
    # o is bf16, so the gradient reaching the backward is dO rounded to bf16
    g = ops.prefill_backward(t["q"], t["k"], t["v"], t["A_log"], t["a"], t["b"], dO.bfloat16(), dt_bias=dtb,
                             state_in=t["state_in"], scale=inp["scale"])
    torch.cuda.synchronize()
    assert torch.allclose(leaves["v"].grad.float(), g["dv"].bfloat16().float())
    assert torch.allclose(leaves["a"].grad, g["da"]) and torch.allclose(leaves["state_in"].grad, g["dstate_in"])
    assert torch.allclose(dtb_l.grad, g["ddt_bias"]) and torch.allclose(leaves["A_log"].grad, g["dA_log"])


def test_prefill_bwd_windows_bit_identical(cuda_device):
    """The windowed backward recomputes each window's states from checkpoints with the
    same fp32 recurrence and carries dS through memory exactly: every gradient equals
    the one-window run bit for bit, for windows that divide T and ragged ones."""
    import torch
    from gdn_18646_b200 import ops
    B, H, T, dk, dv = 2, 2, 200, 128, 128
    inp = O.make_prefill_inputs(17, B, T, H, dk, dv, gate_dtype="f32", state_std=0.05)
    rng = np.random.default_rng(5)
    mask = np.ones((B, T), np.float32)
    mask[1, 150:] = 0.0
    dO = to_dev(rng.standard_normal((B, H, T, dv)).astype(np.float32))
    dSf = to_dev((rng.standard_normal((B, H, dk, dv)) * 0.1).astype(np.float32))
    args = (to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]), to_dev(inp["a"]),
            to_dev(inp["b"]), dO)
    kw = dict(dt_bias=0.1, mask=to_dev(mask), state_in=to_dev(inp["state_in"]), dS_final=dSf, scale=inp["scale"])
    whole = ops.prefill_backward(*args, **kw, window=T, algorithm="token")
    for w in (32, 40, 64, 199):
        got = ops.prefill_backward(*args, **kw, window=w, algorithm="token")
        torch.cuda.synchronize()
        for name in whole:
            assert torch.equal(got[name], whole[name]), f"{name} differs with {w}-token windows"


@pytest.mark.parametrize("B,H,T,dk,dv", [(1, 4, 4096, 128, 128), (2, 2, 1000, 64, 128)])
def test_prefill_bwd_chunked_vs_token_long(cuda_device, B, H, T, dk, dv):
    """At sequence lengths the float64 oracle is too slow for, the chunked backward
    agrees with the token-recurrent one (both fp32, different summation orders) to a
    relative max error of 1e-3 per gradient, bf16 inputs, a bf16 dO and a masked tail."""
    import torch
    from gdn_18646_b200 import ops
    inp = O.make_prefill_inputs(31 + T, B, T, H, dk, dv, gate_dtype="bf16", state_std=0.05)
    rng = np.random.default_rng(T)
    mask = np.ones((B, T), np.float32)
    mask[-1, T - 77:] = 0.0
    dO = to_dev(rng.standard_normal((B, H, T, dv)).astype(np.float32)).bfloat16()
    dSf = to_dev((rng.standard_normal((B, H, dk, dv)) * 0.1).astype(np.float32))
    a = to_dev(inp["a"])
    b = to_dev(inp["b"])
    args = (to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]), a, b, dO)
    kw = dict(dt_bias=to_dev((rng.standard_normal(H) * 0.2).astype(np.float32)), mask=to_dev(mask),
              state_in=to_dev(inp["state_in"]), dS_final=dSf, scale=inp["scale"])
    want = ops.prefill_backward(*args, **kw, algorithm="token")
    got = ops.prefill_backward(*args, **kw, algorithm="chunked")
    torch.cuda.synchronize()
    for name in want:
        w = want[name].double().cpu().numpy()
        g = got[name].double().cpu().numpy()
        assert np.isfinite(g).all(), name
        err = _rel(g, w)
        assert err < 1e-3, f"{name}: relative max error {err:.2e}"


@pytest.mark.parametrize("T", [1, 5, 64])
@pytest.mark.parametrize("algorithm", ["chunked", "token"])
def test_prefill_bwd_short_sequences(cuda_device, T, algorithm):
    """A sequence shorter than one chunk, or exactly one: a single (ragged) chunk, no
    chunk recurrence steps, against the oracle at the same 1e-3 bar."""
    import torch
    from gdn_18646_b200 import ops
    B, H, dk, dv = 2, 3, 128, 64
    inp = O.make_prefill_inputs(100 + T, B, T, H, dk, dv, gate_dtype="f32", state_std=0.05)
    rng = np.random.default_rng(T)
    dtb = (rng.standard_normal(H) * 0.2).astype(np.float32)
    dO = rng.standard_normal((B, H, T, dv)).astype(np.float32)
    dSf = (rng.standard_normal((B, H, dk, dv)) * 0.1).astype(np.float32)
    ref = O.prefill_backward(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], dtb, inp["b"], np.ones((B, T)), dO,
                             state_in=inp["state_in"], dS_final=dSf, scale=inp["scale"])
    got = ops.prefill_backward(to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"]), to_dev(inp["A_log"]),
                               to_dev(inp["a"]), to_dev(inp["b"]), to_dev(dO), dt_bias=to_dev(dtb),
                               state_in=to_dev(inp["state_in"]), dS_final=to_dev(dSf), scale=inp["scale"],
                               algorithm=algorithm)
    torch.cuda.synchronize()
    for name in ("dq", "dk", "dv", "da", "db", "dA_log", "ddt_bias", "dstate_in"):
        err = _rel(to_np(got[name]).astype(np.float64), ref[name])
        assert err < 1e-3, f"{name}: relative max error {err:.2e}"
