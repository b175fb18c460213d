"""The config-3 layer (gdn_18646_b200.layer) against the oracle composition,
prefill -> decode continuation, and CUDA-graph decode.  Tolerance follows the
reference harness's layer check (bench_gdn.py:152-169: atol 5e-2, rtol 0.1)."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import to_dev, to_np

pytestmark = pytest.mark.gpu


def _layer(seed=0):
    from gdn_18646_b200.layer import GDNConfig, GDNLayer, make_weights
    cfg = GDNConfig()
    return GDNLayer(make_weights(cfg, seed=seed), cfg)


def _close(got, want, atol=5e-2, rtol=0.1):
    g = O.bf16_to_f32(to_np(got)) if not isinstance(got, np.ndarray) else O.bf16_to_f32(got)
    w = O.bf16_to_f32(want)
    assert np.all(np.abs(g - w) <= atol + rtol * np.abs(w)), f"max diff {np.abs(g - w).max():.3e}"


def test_layer_prefill_vs_oracle(cuda_device):
    import torch
    layer = _layer()
    B, T = 1, 192
    x = torch.randn(B, T, 2048, device="cuda").bfloat16()
    y, st = layer.prefill(x)
    torch.cuda.synchronize()
    wn = {k: to_np(v) for k, v in layer.w.items()}
    y_ref, S_ref = O.layer_prefill(to_np(x), wn)
    _close(y, y_ref)
    assert O.rel_fro(to_np(st["recurrent"]), S_ref) < 1e-2


def test_layer_prefill_then_decode_matches_full_prefill(cuda_device):
    """gdn_layer.py has no prefill->decode carry; the layer here does: prefill
    T1 tokens, then decode the rest one at a time == one prefill over T."""
    import torch
    layer = _layer(1)
    B, T, T1 = 2, 72, 64
    x = torch.randn(B, T, 2048, device="cuda").bfloat16()
    y_full, st_full = layer.prefill(x)
    y1, st = layer.prefill(x[:, :T1].contiguous())
    ys = [y1]
    for t in range(T1, T):
        yt, st = layer.decode(x[:, t:t + 1].contiguous(), st)
        ys.append(yt)
    y_cat = torch.cat(ys, 1)
    torch.cuda.synchronize()
    _close(y_cat, to_np(y_full))
    assert O.rel_fro(to_np(st["recurrent"]), to_np(st_full["recurrent"])) < 1e-3
    for key in ("conv_q", "conv_k", "conv_v"):
        # the decode projection is a GEMV, the prefill's a tensor-core GEMM: the
        # fp32 summation orders differ, so a cached bf16 value may differ by an ulp
        g, w = O.bf16_to_f32(to_np(st[key])), O.bf16_to_f32(to_np(st_full[key]))
        assert np.all(np.abs(g - w) <= np.abs(w) * 2.0 ** -6 + 1e-2)
        assert np.mean(g != w) <= 0.05


@pytest.mark.parametrize("overlap", [True, False])
def test_layer_decode_cuda_graph_matches_eager(cuda_device, overlap):
    """The CUDA-graph decode step, with and without programmatic dependent launch
    between its kernels, gives the eager step's bits."""
    import torch
    from gdn_18646_b200.layer import DecodeGraph
    layer = _layer(2)
    B, T0, steps = 2, 64, 6
    x = torch.randn(B, T0 + steps, 2048, device="cuda").bfloat16()
    _, st_e = layer.prefill(x[:, :T0].contiguous())
    st_g = {k: v.clone() for k, v in st_e.items()}
    graph = DecodeGraph(layer, st_g, B, overlap=overlap)
    for t in range(T0, T0 + steps):
        ye, st_e = layer.decode(x[:, t:t + 1].contiguous(), st_e)
        yg = graph.step(x[:, t:t + 1])
        torch.cuda.synchronize()
        assert torch.equal(ye, yg)
    assert torch.equal(st_e["recurrent"], st_g["recurrent"])


def test_layer_decode_stacked_graph_matches_eager(cuda_device):
    """Three layers in one CUDA graph (each layer's output feeding the next, with
    programmatic dependent launch across the stack) give the eager chain's bits."""
    import torch
    from gdn_18646_b200.layer import DecodeStackGraph
    layers = [_layer(3 + i) for i in range(3)]
    B, T0, steps = 2, 64, 4
    x = torch.randn(B, T0 + steps, 2048, device="cuda").bfloat16()
    st_e = [layer.prefill(x[:, :T0].contiguous())[1] for layer in layers]
    st_g = [{k: v.clone() for k, v in s.items()} for s in st_e]
    stack = DecodeStackGraph(layers, st_g, B)
    for t in range(T0, T0 + steps):
        y = x[:, t:t + 1].contiguous()
        for i, layer in enumerate(layers):
            y, st_e[i] = layer.decode(y, st_e[i])
        yg = stack.step(x[:, t:t + 1])
        torch.cuda.synchronize()
        assert torch.equal(y, yg)
    for se, sg in zip(st_e, st_g):
        assert torch.equal(se["recurrent"], sg["recurrent"])
        assert torch.equal(se["conv_v"], sg["conv_v"])


def _stage(report, name, got_bits, want_bits, atol=0.0, ulps=1, max_frac=0.01, gemm=False):
    """Record one stage's agreement: every element within ``atol`` plus ``ulps``
    bf16 ulps of the oracle's value, and at most ``max_frac`` of them different.

    bf16 results of the same op with a different fp32 summation order differ by
    an ulp where the exact value sits near a rounding boundary.  A GEMM output
    (``gemm``: 2048- or 4096-term dot products) carries an fp32 summation error
    proportional to the sum of |terms|, not to the result, so small results
    differ by more ulps: those stages get two ulps plus an absolute 2^-8 of the
    output's RMS.  Where a stage sums neighbouring values (the conv over four
    projected tokens) a one-ulp change of an input becomes several ulps of a
    small output, which ``atol`` absorbs."""
    g, w = O.bf16_to_f32(got_bits).astype(np.float64), O.bf16_to_f32(want_bits).astype(np.float64)
    d = np.abs(g - w)
    if gemm:
        ulps, atol = 2, max(atol, float(np.sqrt(np.mean(w * w))) * 2.0 ** -8)
    tol = atol + ulps * np.abs(w) * 2.0 ** -7
    worst = np.unravel_index(np.argmax(d - tol), d.shape)
    report[name] = (float(d.max()), float(np.mean(d > 0)), bool(np.all(d <= tol)) and float(np.mean(d > 0)) <= max_frac,
                    f"worst: got {g[worst]:.6g} want {w[worst]:.6g} tol {tol[worst]:.3g}")


def test_layer_prefill_config3_shape(cuda_device):
    """Config 3's layer prefill at its shape (B=2, T=8192, hidden 2048, 16 q/k
    and 32 value heads) against the oracle composition (gdn_layer.py:120-159
    plus the BASELINE additions).

    Stage by stage, each kernel on the GPU's own inputs: RMSNorm, the q|k|v
    projections (conv4 + SiLU, q/k L2 norm) and z/a/b on sampled token windows,
    the prefill on sampled heads at the north_star bar, the gated norm, and the
    output projection on sampled rows.  Then end to end: the layer's y and final
    state against the whole oracle layer run on x alone, at north_star's bar
    (y max-abs <= 2e-2, state rel-Frobenius <= 1e-3)."""
    import torch
    layer = _layer(11)
    B, T, D = 2, 8192, 2048
    g = torch.Generator(device="cuda").manual_seed(31)
    x = torch.randn(B, T, D, generator=g, device="cuda").bfloat16()
    tr = {}
    y, st = layer.prefill(x, trace=tr)
    torch.cuda.synchronize()
    wn = {k_: to_np(v_) for k_, v_ in layer.w.items()}
    xb = to_np(x)
    t = {k_: to_np(v_) for k_, v_ in tr.items()}
    rep = {}

    _stage(rep, "rmsnorm", t["xn"], O.rmsnorm(xb.reshape(B * T, D), wn["norm_gamma"]).reshape(B, T, D))
    # projections on token windows (3 tokens of conv history before each), GPU xn as input
    for t0 in (0, 4093, T - 64):
        lo = max(t0 - 3, 0)
        xw = t["xn"][:, lo:t0 + 64]
        for name, Wn, cw, l2 in (("q", "W_q", "conv_q", True), ("k", "W_k", "conv_k", True),
                                 ("v", "W_v", "conv_v", False)):
            ref = O.proj_conv_silu(xw, wn[Wn], wn[cw])[0][:, t0 - lo:]
            if l2:
                ref = O.l2norm_heads(ref, 128)
            _stage(rep, f"{name}@{t0}", t[name][:, t0:t0 + 64], ref, atol=4e-3 if l2 else 1e-2, ulps=2,
                   max_frac=0.02)
        _stage(rep, f"z@{t0}", t["z"][:, t0:t0 + 64], O._bf16_matmul(t["xn"][:, t0:t0 + 64], wn["W_z"]), gemm=True)
        ab = O._bf16_matmul(t["xn"][:, t0:t0 + 64], wn["W_ab"])
        _stage(rep, f"a@{t0}", np.swapaxes(t["a"][:, :, t0:t0 + 64], 1, 2), ab[..., :32], gemm=True)
        _stage(rep, f"b@{t0}", np.swapaxes(t["b"][:, :, t0:t0 + 64], 1, 2), ab[..., 32:], gemm=True)
    # prefill on sampled (b, value head) pairs of the GPU's q/k/v/a/b (head h reads q/k head h // 2)
    S_gpu = to_np(st["recurrent"])
    for bi, h in ((0, 0), (1, 13), (1, 31)):
        hq = h // 2
        qh = np.swapaxes(t["q"].reshape(B, T, 16, 128)[bi:bi + 1, :, hq:hq + 1], 1, 2)
        kh = np.swapaxes(t["k"].reshape(B, T, 16, 128)[bi:bi + 1, :, hq:hq + 1], 1, 2)
        vh = np.swapaxes(t["v"].reshape(B, T, 32, 128)[bi:bi + 1, :, h:h + 1], 1, 2)
        o_r, S_r = O.prefill(qh, kh, vh, wn["A_log"][h:h + 1], t["a"][bi:bi + 1, h:h + 1],
                             float(wn["dt_bias"][h]), t["b"][bi:bi + 1, h:h + 1], np.ones((1, T), np.float32),
                             scale=128 ** -0.5, chunk_size=64, dt=np.float64)
        o_g = O.bf16_to_f32(np.swapaxes(t["o"][bi:bi + 1, :, h:h + 1], 1, 2))
        e_o, e_s = float(np.abs(o_g - o_r).max()), O.rel_fro(S_gpu[bi:bi + 1, h:h + 1], S_r)
        rep[f"prefill({bi},{h})"] = (e_o, e_s, e_o <= 2e-2 and e_s <= 1e-3, "o max-abs, state rel-F")
    # gated norm over every head row, GPU o and z as input
    _stage(rep, "gated_norm", t["y_norm"].reshape(-1, 128),
           O.gated_rmsnorm(t["o"].reshape(-1, 128), t["z"].reshape(-1, 128), wn["onorm_gamma"]))
    # output projection on sampled rows
    yb = to_np(y)
    for r0 in (0, 5000, T - 32):
        _stage(rep, f"out@{r0}", yb[:, r0:r0 + 32], O._bf16_matmul(t["y_norm"][:, r0:r0 + 32], wn["W_o"]), gemm=True)

    # end to end: the whole oracle layer on x
    y_ref, S_ref = O.layer_prefill(xb, wn)
    err_y = float(np.abs(O.bf16_to_f32(yb) - O.bf16_to_f32(y_ref)).max())
    err_s = O.rel_fro(S_gpu, S_ref)
    rep["end_to_end"] = (err_y, err_s, err_y <= 2e-2 and err_s <= 1e-3, "y max-abs, state rel-F")
    for k_, v_ in rep.items():
        print(f"config-3 layer {k_}: {v_[0]:.3e} {v_[1]:.3e} {'ok' if v_[2] else 'FAIL'} ({v_[3]})")
    bad = [k_ for k_, v_ in rep.items() if not v_[2]]
    assert not bad, f"stages outside their bar: {bad}"
