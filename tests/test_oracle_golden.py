"""Pin the CPU oracle to golden vectors produced by the reference's own
PyTorch functions (tests/golden/make_golden.py).  CPU only."""
import math
import os

import numpy as np
import pytest

from oracle import gdn_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


PREFILL_CASES = ["prefill_config0", "prefill_config1_small", "prefill_mask", "prefill_ragged",
                 "prefill_scale0", "prefill_gva", "prefill_refshape"]


@pytest.mark.parametrize("name", PREFILL_CASES)
def test_prefill_oracle_matches_reference(name):
    g = load(name)
    H = g["v"].shape[1]
    q, k = g["q"], g["k"]
    if q.shape[1] != H:
        q, k = O.expand_qk_heads(q, H), O.expand_qk_heads(k, H)
    o, S = O.prefill(q, k, g["v"], g["A_log"], g["a"], float(g["dt_bias"]), g["b"], g["mask"],
                     state_in=g.get("state_in"), scale=float(g["scale"]), chunk_size=int(g["chunk"]))
    assert o.shape == g["o"].shape and S.shape == g["state_out"].shape
    np.testing.assert_allclose(o, g["o"], rtol=2e-4, atol=2e-5)
    assert O.rel_fro(S, g["state_out"]) < 1e-5


@pytest.mark.parametrize("name", ["prefill_config0", "prefill_mask", "prefill_ragged"])
def test_chunked_oracle_matches_token_recurrence(name):
    """The chunked WY restatement equals the per-token recurrence of the
    reference docstring (prefill_ref.py:18-23) -- an independent check."""
    g = load(name)
    o_c, S_c = O.prefill(g["q"], g["k"], g["v"], g["A_log"], g["a"], float(g["dt_bias"]), g["b"],
                         g["mask"], state_in=g.get("state_in"), scale=float(g["scale"]),
                         chunk_size=int(g["chunk"]), dt=np.float64)
    o_r, S_r = O.prefill_recurrent(g["q"], g["k"], g["v"], g["A_log"], g["a"], float(g["dt_bias"]),
                                   g["b"], g["mask"], state_in=g.get("state_in"),
                                   scale=float(g["scale"]))
    np.testing.assert_allclose(o_c, o_r, rtol=1e-9, atol=1e-10)
    assert O.rel_fro(S_c, S_r) < 1e-10


def test_chunk_size_invariance():
    g = load("prefill_config0")
    outs = [O.prefill(g["q"], g["k"], g["v"], g["A_log"], g["a"], 0.0, g["b"], g["mask"],
                      scale=float(g["scale"]), chunk_size=c, dt=np.float64) for c in (16, 64, 128)]
    for o, S in outs[1:]:
        np.testing.assert_allclose(o, outs[0][0], rtol=1e-9, atol=1e-11)
        assert O.rel_fro(S, outs[0][1]) < 1e-10


def test_decode_oracle_matches_reference_chained():
    g = load("decode_config2_small")
    S = g["state_in"]
    for step in range(g["q"].shape[0]):
        o, S = O.decode(g["q"][step], g["k"][step], g["v"][step], S, g["A_log"], g["a"][step],
                        g["dt_bias"], g["b"][step], 1.0 / math.sqrt(128))
        np.testing.assert_allclose(o, g["o"][step], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(S, g["state_out"][step], rtol=1e-5, atol=1e-6)


def test_decode_oracle_matches_reference_refshape():
    g = load("decode_refshape")
    o, S = O.decode(g["q"], g["k"], g["v"], g["state_in"], g["A_log"], g["a"], g["dt_bias"],
                    g["b"], 1.0 / math.sqrt(128))
    np.testing.assert_allclose(o, g["o"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(S, g["state_out"], rtol=1e-5, atol=1e-7)


def test_decode_loop_equals_prefill():
    """bench_gdn.py:200-219 check, restated: T decode steps == one prefill."""
    inp = O.make_prefill_inputs(5, 1, 64, 2, 64, 64, state_std=0.02)
    o_p, S_p = O.prefill(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], 0.0, inp["b"],
                         inp["mask"], state_in=inp["state_in"], scale=inp["scale"], chunk_size=64,
                         dt=np.float64)
    S = inp["state_in"].astype(np.float64)
    dtb = np.zeros(2)
    for t in range(64):
        o, S = O.decode(inp["q"][:, :, t], inp["k"][:, :, t], inp["v"][:, :, t], S, inp["A_log"],
                        inp["a"][:, :, t], dtb, inp["b"][:, :, t], inp["scale"], dt=np.float64)
        np.testing.assert_allclose(o, o_p[:, :, t], rtol=1e-9, atol=1e-11)
    assert O.rel_fro(S, S_p) < 1e-10


@pytest.mark.parametrize("name", ["proj_small", "proj_t1"])
def test_proj_conv_silu_oracle_matches_reference(name):
    g = load(name)
    y, _ = O.proj_conv_silu(g["x"], g["W"], g["conv_w"])
    got, want = O.bf16_to_f32(y), O.bf16_to_f32(g["y"])
    # bf16 rounding points match the reference; summation order may flip 1 ulp
    ulp = np.abs(want) * 2.0 ** -7 + 1e-6
    assert np.mean(got != want) < 0.02
    assert np.all(np.abs(got - want) <= 2 * ulp)


@pytest.mark.parametrize("name", ["rmsnorm_2048", "rmsnorm_512"])
def test_rmsnorm_oracle_matches_reference(name):
    g = load(name)
    y = O.rmsnorm(g["x"], g["gamma"], float(g["eps"]))
    got, want = O.bf16_to_f32(y), O.bf16_to_f32(g["y"])
    assert np.mean(got != want) < 0.01
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -7 + 1e-6)


def test_bf16_roundtrip_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0, 1e-40, np.inf], np.float32)
    import torch
    want = torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16(x), want)
