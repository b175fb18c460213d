"""The oracle's backward (prefill_backward) pinned against central finite
differences of its token-recurrent forward (prefill_recurrent), in float64,
for every input: q, k, v, the gate inputs a and b, A_log, dt_bias and the
initial state, with a mask and a gradient on the final state."""
import numpy as np

from oracle import gdn_oracle as O


def _loss(q, k, v, A_log, a, dtb, b, mask, S0, dO, dSf, scale):
    o, S = O.prefill_recurrent(q, k, v, A_log, a, dtb, b, mask, state_in=S0, scale=scale, dt=np.float64)
    return float((o * dO).sum() + (S * dSf).sum())


def test_prefill_backward_matches_finite_differences():
    rng = np.random.default_rng(0)
    B, H, T, K, V = 1, 2, 6, 4, 3
    q = rng.standard_normal((B, H, T, K)) * 0.5
    k = rng.standard_normal((B, H, T, K)) * 0.5
    v = rng.standard_normal((B, H, T, V))
    a = rng.standard_normal((B, H, T))
    b = rng.standard_normal((B, H, T))
    A_log = np.log(np.array([0.3, 0.1]))
    dtb = np.array([0.2, -0.1])
    mask = np.ones((B, T))
    mask[0, 4] = 0.0
    S0 = rng.standard_normal((B, H, K, V)) * 0.3
    dO = rng.standard_normal((B, H, T, V))
    dSf = rng.standard_normal((B, H, K, V))
    scale = 0.7
    gr = O.prefill_backward(q, k, v, A_log, a, dtb, b, mask, dO, state_in=S0, dS_final=dSf, scale=scale)
    args = dict(q=q, k=k, v=v, A_log=A_log, a=a, dtb=dtb, b=b, S0=S0)
    names = dict(q="dq", k="dk", v="dv", A_log="dA_log", a="da", dtb="ddt_bias", b="db", S0="dstate_in")
    eps = 1e-6
    for arg, gname in names.items():
        x = args[arg]
        num = np.zeros_like(x)
        for idx in np.ndindex(x.shape):
            xp, xm = x.copy(), x.copy()
            xp[idx] += eps
            xm[idx] -= eps
            lp = _loss(**{**args, arg: xp}, mask=mask, dO=dO, dSf=dSf, scale=scale)
            lm = _loss(**{**args, arg: xm}, mask=mask, dO=dO, dSf=dSf, scale=scale)
            num[idx] = (lp - lm) / (2 * eps)
        np.testing.assert_allclose(gr[gname], num, rtol=1e-5, atol=1e-7, err_msg=arg)


def test_chunked_backward_matches_token_recurrent():
    """prefill_backward_chunked (per-chunk checkpoints only, the form of a chunked
    GPU backward) equals prefill_backward on the same inputs: ragged last chunks,
    a mask, a per-head dt_bias, an initial state and a final-state gradient."""
    for (B, H, T, K, V, C, seed) in [(1, 2, 70, 16, 8, 16, 1), (2, 2, 130, 32, 16, 32, 2), (1, 1, 128, 64, 64, 64, 3)]:
        inp = O.make_prefill_inputs(seed, B, T, H, K, V, state_std=0.1)
        mask = np.ones((B, T), np.float32)
        mask[:, 5:9] = 0.0
        mask[-1, -3:] = 0.0
        rng = np.random.default_rng(seed)
        dtb = rng.standard_normal(H) * 0.3 if H > 1 else 0.1
        dO = rng.standard_normal((B, H, T, V))
        dSf = rng.standard_normal((B, H, K, V)) * 0.1
        args = (inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], dtb, inp["b"], mask, dO)
        ref = O.prefill_backward(*args, state_in=inp["state_in"], dS_final=dSf, scale=inp["scale"])
        got = O.prefill_backward_chunked(*args, state_in=inp["state_in"], dS_final=dSf, scale=inp["scale"],
                                         chunk_size=C)
        for name in ref:
            np.testing.assert_allclose(got[name], ref[name], rtol=1e-9, atol=1e-11 * np.abs(ref[name]).max(),
                                       err_msg=f"{name} at {(B, H, T, K, V, C)}")
