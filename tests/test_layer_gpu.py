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
