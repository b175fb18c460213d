"""Fused projection + causal conv1d(k=4) + SiLU parity vs the reference's
golden vectors and the oracle (same bf16 rounding points as
reference/fused_proj_conv_silu_ref.py:54-66).  Bar: at most 5% of elements
differ from the oracle, each by a few bf16 ulps (the fp32 summation order of
the projection differs), and the reference harness gate max-abs < 5e-2
(tests/test_fused_proj_conv_silu.py:59)."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import load_golden, to_dev, to_np

pytestmark = pytest.mark.gpu


def _close(got, want, frac=0.05):
    """A 1-ulp flip of the bf16-rounded projection (different fp32 summation
    order) propagates through the conv and SiLU roundings, so allow a few
    output ulps per element, and require almost all elements to be identical."""
    g, w = O.bf16_to_f32(got), O.bf16_to_f32(want)
    diff = np.abs(g - w)
    assert np.all(diff <= np.abs(w) * 2.0 ** -6 + 1e-2), f"max diff {diff.max():.3e}"
    assert diff.max() < 5e-2                       # the reference harness gate
    assert np.mean(g != w) <= frac, f"{np.mean(g != w):.3f} of elements differ"


def _run(x, W, cw, **kw):
    import torch
    from gdn_18646_b200 import ops
    y = ops.proj_conv_silu(to_dev(x), to_dev(W), to_dev(cw), **kw)
    torch.cuda.synchronize()
    return to_np(y)


@pytest.mark.parametrize("name", ["proj_small", "proj_t1"])
def test_proj_golden(cuda_device, name):
    g = load_golden(name)
    y = _run(g["x"], g["W"], g["conv_w"])
    _close(y, g["y"])


@pytest.mark.parametrize("B,T,D,Dout", [(1, 1, 64, 128), (2, 253, 128, 256), (2, 254, 128, 128),
                                         (1, 600, 256, 384), (3, 77, 2048, 128), (1, 1000, 512, 1024)])
def test_proj_vs_oracle(cuda_device, B, T, D, Dout):
    rng = np.random.default_rng(B * 131 + T + D + Dout)
    x = O.f32_to_bf16(rng.standard_normal((B, T, D), dtype=np.float32))
    W = O.f32_to_bf16(rng.standard_normal((Dout, D), dtype=np.float32) * np.float32(D ** -0.5))
    cw = O.f32_to_bf16(rng.standard_normal((Dout, 4), dtype=np.float32) * np.float32(0.5))
    y = _run(x, W, cw)
    y_ref, _ = O.proj_conv_silu(x, W, cw)
    _close(y, y_ref)


def test_proj_conv_state_continuation(cuda_device):
    """Running [0, T1) then [T1, T) with the conv state carried equals one pass,
    and conv_state_out holds the last three projected tokens."""
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(9)
    B, T, D, Dout, T1 = 2, 300, 256, 256, 130
    x = O.f32_to_bf16(rng.standard_normal((B, T, D), dtype=np.float32))
    W = O.f32_to_bf16(rng.standard_normal((Dout, D), dtype=np.float32) * np.float32(D ** -0.5))
    cw = O.f32_to_bf16(rng.standard_normal((Dout, 4), dtype=np.float32) * np.float32(0.5))
    xd, Wd, cwd = to_dev(x), to_dev(W), to_dev(cw)
    st1 = torch.empty(B, Dout, 3, dtype=torch.bfloat16, device="cuda")
    st2 = torch.empty_like(st1)
    y_full = ops.proj_conv_silu(xd, Wd, cwd)
    y1 = ops.proj_conv_silu(xd[:, :T1].contiguous(), Wd, cwd, conv_state_out=st1)
    y2 = ops.proj_conv_silu(xd[:, T1:].contiguous(), Wd, cwd, conv_state_in=st1, conv_state_out=st2)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([y1, y2], 1), y_full)
    _, proj = O.proj_conv_silu(x, W, cw)
    assert np.array_equal(to_np(st2), np.swapaxes(proj[:, T - 3:], 1, 2))
    # short continuation (T2 < 3) mixes history and new tokens in the state
    st3 = torch.empty_like(st1)
    ops.proj_conv_silu(xd[:, :2].contiguous(), Wd, cwd, conv_state_in=st2, conv_state_out=st3)
    torch.cuda.synchronize()
    want = np.concatenate([to_np(st2)[:, :, 2:], np.swapaxes(O.proj_conv_silu(x[:, :2], W, cw)[1], 1, 2)], 2)
    assert np.array_equal(to_np(st3), want)


@pytest.mark.parametrize("group", [128, 64])
def test_proj_l2norm_epilogue(cuda_device, group):
    rng = np.random.default_rng(group)
    B, T, D, Dout = 2, 300, 256, 256
    x = O.f32_to_bf16(rng.standard_normal((B, T, D), dtype=np.float32))
    W = O.f32_to_bf16(rng.standard_normal((Dout, D), dtype=np.float32) * np.float32(D ** -0.5))
    cw = O.f32_to_bf16(rng.standard_normal((Dout, 4), dtype=np.float32) * np.float32(0.5))
    y = _run(x, W, cw, l2norm_group=group)
    y_ref = O.l2norm_heads(O.proj_conv_silu(x, W, cw)[0], group)
    _close(y, y_ref)
    norms = np.sqrt((O.bf16_to_f32(y).reshape(B, T, -1, group) ** 2).sum(-1))
    assert np.allclose(norms, 1.0, atol=2e-2)


def test_proj_reference_module_surface_and_tolerance(cuda_device):
    """tests/test_fused_proj_conv_silu.py:45-66 shapes through exts()['proj']
    against a torch bf16 restatement of ref_proj_conv_silu."""
    import torch
    import torch.nn.functional as F
    import gdn_18646_b200 as G
    ext = G.exts()["proj"]
    for B, T, Dout in ((1, 1, 2048), (4, 128, 2048), (2, 64, 4096)):
        x = torch.randn(B, T, 2048, device="cuda", dtype=torch.bfloat16)
        W = torch.randn(Dout, 2048, device="cuda", dtype=torch.bfloat16) * 2048 ** -0.5
        cw = torch.randn(Dout, 4, device="cuda", dtype=torch.bfloat16) * 0.5
        y = ext.forward(x, W, cw)
        proj = (x @ W.T).transpose(1, 2)
        ref = F.silu(F.conv1d(F.pad(proj, (3, 0)), cw.unsqueeze(1), groups=Dout)).transpose(1, 2)
        diff = (y.float() - ref.float()).abs()
        assert diff.max().item() < 5e-2
        assert (diff / (ref.float().abs() + 1e-8)).max().item() < 0.1 or diff.max().item() < 2e-2


def test_proj_multi_matches_single_launches(cuda_device):
    """gdn_proj_multi_fwd: q | k | v-like conv segments (two L2-normalised, with and
    without conv histories) and a plain segment in one launch give the bits of the
    separate single-segment launches (the plain one: bf16 of the fp32 product, the
    conv ones: gdn_proj_conv_silu_fwd)."""
    import torch
    from gdn_18646_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(21)
    B, T, D = 2, 700, 256
    x = torch.randn(B, T, D, generator=g, device="cuda").bfloat16()
    Ws = [(torch.randn(C, D, generator=g, device="cuda") * 0.05).bfloat16() for C in (256, 128, 384, 128)]
    cws = [(torch.randn(C, 4, generator=g, device="cuda") * 0.5).bfloat16() for C in (256, 128, 384)]
    hin = [(torch.randn(B, C, 3, generator=g, device="cuda")).bfloat16() for C in (256, 128, 384)]
    hout_m = [torch.empty(B, C, 3, dtype=torch.bfloat16, device="cuda") for C in (256, 128, 384)]
    hout_s = [torch.empty_like(h) for h in hout_m]
    l2s = (128, 64, 0)
    outs = ops.proj_multi(x, [dict(W=Ws[i], conv_w=cws[i], l2norm_group=l2s[i],
                                   conv_state_in=hin[i] if i != 1 else None, conv_state_out=hout_m[i])
                              for i in range(3)] + [dict(W=Ws[3])])
    for i in range(3):
        ref = ops.proj_conv_silu(x, Ws[i], cws[i], l2norm_group=l2s[i], conv_state_in=hin[i] if i != 1 else None,
                                 conv_state_out=hout_s[i])
        torch.cuda.synchronize()
        assert torch.equal(outs[i], ref), f"segment {i}"
        assert torch.equal(hout_m[i], hout_s[i]), f"segment {i} history"
    plain = (x.float() @ Ws[3].float().T).bfloat16()
    # tensor-core fp32 accumulation vs torch's: compare within one bf16 ulp
    diff = (outs[3].float() - plain.float()).abs()
    assert bool((diff <= plain.float().abs() * 2.0 ** -7 + 1e-3).all())
