"""Decode step parity: libgdn_b200 (through the C ABI) vs the CPU oracle and
the reference's golden vectors.  Tolerances: fp32 everywhere, so tight."""
import math

import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import load_golden, to_dev, to_np

pytestmark = pytest.mark.gpu


def _run(q, k, v, a, b, A_log, dtb, S, *, inplace=True, scale=0.0):
    import torch
    from gdn_18646_b200 import ops
    St = to_dev(S).clone()
    S_out = St if inplace else torch.empty_like(St)
    o = ops.decode_step(to_dev(q), to_dev(k), to_dev(v), to_dev(a), to_dev(b), to_dev(A_log), to_dev(dtb), St,
                        scale=scale, state_out=S_out)
    torch.cuda.synchronize()
    return to_np(o), to_np(S_out)


def test_decode_golden_chained(cuda_device):
    g = load_golden("decode_config2_small")
    S = g["state_in"]
    for st in range(g["q"].shape[0]):
        o, S = _run(g["q"][st], g["k"][st], g["v"][st], g["a"][st], g["b"][st], g["A_log"], g["dt_bias"], S,
                    scale=1.0 / math.sqrt(128))
        np.testing.assert_allclose(o, g["o"][st], rtol=1e-4, atol=1e-6)
        np.testing.assert_allclose(S, g["state_out"][st], rtol=1e-4, atol=1e-6)


def test_decode_golden_refshape_dv256(cuda_device):
    g = load_golden("decode_refshape")
    o, S = _run(g["q"], g["k"], g["v"], g["a"], g["b"], g["A_log"], g["dt_bias"], g["state_in"],
                scale=1.0 / math.sqrt(128))
    np.testing.assert_allclose(o, g["o"], rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(S, g["state_out"], rtol=1e-4, atol=1e-7)
    # the reference test's own gate (tests/test_decode.py:56-65)
    assert np.abs(o - g["o"]).max() < 1e-2 and np.abs(S - g["state_out"]).max() < 1e-2


@pytest.mark.parametrize("dk,dv", [(64, 64), (64, 128), (128, 64), (128, 128), (128, 256), (256, 128), (256, 256)])
def test_decode_dims_vs_oracle(cuda_device, dk, dv):
    steps, S, A_log, dtb = O.make_decode_inputs(11 + dk + dv, 3, 4, dk, dv)
    st = steps[0]
    o, S1 = _run(st["q"], st["k"], st["v"], st["a"], st["b"], A_log, dtb, S)
    o_r, S_r = O.decode(st["q"], st["k"], st["v"], S, A_log, st["a"], dtb, st["b"], dt=np.float64)
    np.testing.assert_allclose(o, o_r, rtol=1e-4, atol=1e-6)
    assert O.rel_fro(S1, S_r) < 1e-6


def test_decode_gva_and_f32_gates(cuda_device):
    rng = np.random.default_rng(3)
    B, Hqk, Hv, dk, dv = 2, 2, 8, 128, 128
    q = O.normalized_bf16(rng, (B, Hqk, dk))
    k = O.normalized_bf16(rng, (B, Hqk, dk))
    v = O.f32_to_bf16(rng.standard_normal((B, Hv, dv), dtype=np.float32))
    a = rng.standard_normal((B, Hv), dtype=np.float32)
    b = rng.standard_normal((B, Hv), dtype=np.float32)
    S = rng.standard_normal((B, Hv, dk, dv), dtype=np.float32) * np.float32(0.02)
    A_log = np.full((Hv,), math.log(0.1), np.float32)
    dtb = rng.standard_normal(Hv).astype(np.float32) * np.float32(0.1)
    o, S1 = _run(q, k, v, a, b, A_log, dtb, S)
    o_r, S_r = O.decode(np.repeat(q, Hv // Hqk, 1), np.repeat(k, Hv // Hqk, 1), v, S, A_log, a, dtb, b,
                        dt=np.float64)
    np.testing.assert_allclose(o, o_r, rtol=1e-4, atol=1e-6)
    assert O.rel_fro(S1, S_r) < 1e-6


@pytest.mark.parametrize("dk,dv,Hqk", [(128, 128, 4), (64, 256, 2), (256, 64, 1)])
def test_decode_l2norm_qk_flag(cuda_device, dk, dv, Hqk):
    """GDN_DECODE_L2NORM_QK: unnormalised q, k in; the kernel normalises per head and
    rounds to bf16 before the step.  Against the oracle on the oracle-normalised
    inputs (O.l2norm_heads, the projection epilogue's restatement): both round the
    same fp32 values to bf16, so a q/k element may differ by one bf16 ulp where the
    sums of squares round differently."""
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(dk + dv)
    B, Hv = 2, 4
    q = O.f32_to_bf16(rng.standard_normal((B, Hqk, dk), dtype=np.float32) * np.float32(0.3))
    k = O.f32_to_bf16(rng.standard_normal((B, Hqk, dk), dtype=np.float32) * np.float32(0.3))
    v = O.f32_to_bf16(rng.standard_normal((B, Hv, dv), dtype=np.float32))
    a = O.f32_to_bf16(rng.standard_normal((B, Hv), dtype=np.float32))
    b = O.f32_to_bf16(rng.standard_normal((B, Hv), dtype=np.float32))
    S = rng.standard_normal((B, Hv, dk, dv), dtype=np.float32) * np.float32(0.02)
    A_log = np.full((Hv,), math.log(0.1), np.float32)
    dtb = np.zeros(Hv, np.float32)
    St = to_dev(S)
    o = ops.decode_step(to_dev(q), to_dev(k), to_dev(v), to_dev(a), to_dev(b), to_dev(A_log), to_dev(dtb), St,
                        l2norm_qk=True)
    torch.cuda.synchronize()
    qn = O.l2norm_heads(q.reshape(B, Hqk * dk), dk).reshape(B, Hqk, dk)
    kn = O.l2norm_heads(k.reshape(B, Hqk * dk), dk).reshape(B, Hqk, dk)
    o_r, S_r = O.decode(np.repeat(qn, Hv // Hqk, 1), np.repeat(kn, Hv // Hqk, 1), v, S, A_log, a, dtb, b,
                        dt=np.float64)
    np.testing.assert_allclose(to_np(o), o_r, rtol=1e-2, atol=2e-3)
    assert O.rel_fro(to_np(St), S_r) < 1e-3


def test_decode_inplace_equals_out_of_place(cuda_device):
    steps, S, A_log, dtb = O.make_decode_inputs(5, 4, 8, 128, 128)
    st = steps[0]
    o1, S1 = _run(st["q"], st["k"], st["v"], st["a"], st["b"], A_log, dtb, S, inplace=True)
    o2, S2 = _run(st["q"], st["k"], st["v"], st["a"], st["b"], A_log, dtb, S, inplace=False)
    assert np.array_equal(o1, o2) and np.array_equal(S1, S2)


def test_decode_config2_full_size_sampled(cuda_device):
    """Config 2 at full size (B=256, H=32, 128x128, ~537 MB state), 4 chained
    in-place steps; a sample of (b, h) heads is checked against the oracle and
    the whole state against a checksum identity of the update."""
    import torch
    from gdn_18646_b200 import ops
    B, H, dk, dv = 256, 32, 128, 128
    steps, S0, A_log, dtb = O.make_decode_inputs(2024, B, H, dk, dv, steps=4)
    St = to_dev(S0)
    outs = []
    for st in steps:
        outs.append(ops.decode_step(to_dev(st["q"]), to_dev(st["k"]), to_dev(st["v"]), to_dev(st["a"]),
                                    to_dev(st["b"]), to_dev(A_log), to_dev(dtb), St))
    torch.cuda.synchronize()
    S_end = to_np(St)
    rng = np.random.default_rng(0)
    for bi, hi in zip(rng.integers(0, B, 6), rng.integers(0, H, 6)):
        S = S0[bi:bi + 1, hi:hi + 1].astype(np.float64)
        for n, st in enumerate(steps):
            o_r, S = O.decode(st["q"][bi:bi + 1, hi:hi + 1], st["k"][bi:bi + 1, hi:hi + 1],
                              st["v"][bi:bi + 1, hi:hi + 1], S, A_log[hi:hi + 1], st["a"][bi:bi + 1, hi:hi + 1],
                              dtb[hi:hi + 1], st["b"][bi:bi + 1, hi:hi + 1], dt=np.float64)
            np.testing.assert_allclose(to_np(outs[n][bi, hi]), o_r[0, 0], rtol=1e-4, atol=1e-6)
        assert O.rel_fro(S_end[bi, hi], S[0, 0]) < 1e-6
    assert np.isfinite(S_end).all()


def test_decode_reference_module_surface(cuda_device):
    """The reference's decode call signature (kernels/decode.cu:172-214) via exts()."""
    import torch
    import gdn_18646_b200 as G
    ext = G.exts()["decode"]
    g = load_golden("decode_refshape")
    o = torch.zeros(1, 4, 256, device="cuda")
    S_in = to_dev(g["state_in"])
    S_out = torch.zeros_like(S_in)
    ext.forward(to_dev(g["q"]), to_dev(g["k"]), to_dev(g["v"]), to_dev(g["a"]), to_dev(g["b"]), to_dev(g["A_log"]),
                to_dev(g["dt_bias"]), S_in, 1.0 / math.sqrt(128), o, S_out)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(o), g["o"], rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(to_np(S_out), g["state_out"], rtol=1e-4, atol=1e-7)


@pytest.mark.parametrize("dk,dv,l2", [(128, 128, True), (64, 256, False), (256, 64, True), (128, 64, False)])
def test_decode_gated_norm_fused(cuda_device, dk, dv, l2):
    """gdn_decode_step_gated: the step plus the gated output norm of each head's o row
    in one kernel.  The state and the fp32 o are the plain step's, bit for bit; y is
    gdn_gated_rmsnorm_fwd's on the same o up to the order of the fp32 sum of squares
    (one bf16 ulp at most)."""
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(dk * 3 + dv)
    B, Hqk, Hv = 3, 2, 4
    q = O.f32_to_bf16(rng.standard_normal((B, Hqk, dk), dtype=np.float32) * np.float32(0.3))
    k = O.f32_to_bf16(rng.standard_normal((B, Hqk, dk), dtype=np.float32) * np.float32(0.3))
    v = O.f32_to_bf16(rng.standard_normal((B, Hv, dv), dtype=np.float32))
    a = O.f32_to_bf16(rng.standard_normal((B, Hv), dtype=np.float32))
    b = O.f32_to_bf16(rng.standard_normal((B, Hv), dtype=np.float32))
    z = O.f32_to_bf16(rng.standard_normal((B, Hv, dv), dtype=np.float32))
    gamma = O.f32_to_bf16(1.0 + 0.3 * rng.standard_normal(dv, dtype=np.float32))
    S = rng.standard_normal((B, Hv, dk, dv), dtype=np.float32) * np.float32(0.02)
    A_log = np.full((Hv,), math.log(0.1), np.float32)
    dtb = (0.1 * rng.standard_normal(Hv)).astype(np.float32)
    args = [to_dev(x) for x in (q, k, v, a, b, A_log, dtb)]
    S1, S2 = to_dev(S), to_dev(S)
    o1 = ops.decode_step(*args, S1, l2norm_qk=l2)
    y1 = ops.gated_rmsnorm(o1.view(B * Hv, dv), to_dev(z).view(B * Hv, dv), to_dev(gamma), 1e-6)
    o2 = torch.empty_like(o1)
    y2 = ops.decode_step_gated(*args, S2, to_dev(z), to_dev(gamma), 1e-6, out=o2, l2norm_qk=l2)
    torch.cuda.synchronize()
    assert torch.equal(S1, S2) and torch.equal(o1, o2)
    y1f, y2f = y1.float().view(-1), y2.float().view(-1)
    ulp = torch.clamp(y1f.abs(), min=1e-30) * 2.0 ** -7
    assert bool(((y1f - y2f).abs() <= ulp + 1e-30).all())
    # without the fp32 o: same y
    S3 = to_dev(S)
    y3 = ops.decode_step_gated(*args, S3, to_dev(z), to_dev(gamma), 1e-6, l2norm_qk=l2)
    torch.cuda.synchronize()
    assert torch.equal(y3, y2) and torch.equal(S3, S2)
