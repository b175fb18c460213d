"""Decode-step projection (gdn_decode_proj_fwd) against the oracle: one token
per sequence, optional fused RMSNorm of x, conv4 + SiLU over the cached
history (reference/fused_proj_conv_silu_ref.py:33-67 at T=1 with the
gdn_layer.py:43-55 history), per-head L2 norm, and plain GEMV rows.  The bar
is the projection test's: the fp32 summation order of the GEMV differs from
the oracle's, so a bf16 value may flip by one ulp and propagate through the
conv and SiLU roundings; a few output ulps per element, almost all identical."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import to_dev, to_np

pytestmark = pytest.mark.gpu


def _close(got, want, frac=0.05):
    g, w = O.bf16_to_f32(got), O.bf16_to_f32(want)
    diff = np.abs(g - w)
    assert np.all(diff <= np.abs(w) * 2.0 ** -6 + 1e-2), f"max diff {diff.max():.3e}"
    assert np.mean(g != w) <= frac, f"{np.mean(g != w):.3f} of elements differ"


def _bf16(rng, shape, s=1.0):
    return O.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(s))


def _oracle_seg(xn, W, cw=None, hist=None, l2=0):
    """One segment on the oracle: returns (y [B, C], new history [B, C, 3] or None)."""
    if cw is None:
        return O.f32_to_bf16(np.einsum("bd,cd->bc", O.bf16_to_f32(xn), O.bf16_to_f32(W), dtype=np.float32)), None
    y, proj = O.proj_conv_silu(xn[:, None, :], W, cw, conv_state=hist)
    y = y[:, 0]
    if l2:
        y = O.l2norm_heads(y, l2)
    h = np.zeros((xn.shape[0], W.shape[0], 3), np.uint16) if hist is None else hist
    return y, np.concatenate([h[:, :, 1:], proj[:, 0][:, :, None]], axis=2)


@pytest.mark.parametrize("B,D,norm", [(2, 2048, True), (1, 1024, False), (8, 1024, True), (5, 4096, False),
                                      (3, 4352, True)])   # 4352: 256-column stages
def test_decode_proj_segments_vs_oracle(cuda_device, B, D, norm):
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(B * 7 + D)
    x = _bf16(rng, (B, D))
    gamma = O.f32_to_bf16(1.0 + 0.1 * rng.standard_normal(D, dtype=np.float32))
    xn = O.rmsnorm(x, gamma, 1e-6) if norm else x
    segs = [  # (C, conv, l2): q-like (groups wider than a tile: cluster), small groups, 64-wide groups whose
        # last cluster group is half empty, v-like, z-like, a-like
        (256, True, 128), (64, True, 16), (192, True, 64), (384, True, 0), (512, False, 0), (32, False, 0),
        (48, False, 0)]
    W = [_bf16(rng, (C, D), D ** -0.5) for C, _, _ in segs]
    cw = [_bf16(rng, (C, 4), 0.5) if conv else None for C, conv, _ in segs]
    hist = [_bf16(rng, (B, C, 3)) if conv else None for C, conv, _ in segs]
    args = []
    for i, (C, conv, l2) in enumerate(segs):
        d = dict(W=to_dev(W[i]), l2_group=l2)
        if conv:
            d.update(conv_w=to_dev(cw[i]), conv_state_in=to_dev(hist[i]),
                     conv_state_out=torch.empty(B, C, 3, dtype=torch.bfloat16, device="cuda"))
        args.append(d)
    outs = ops.decode_proj(to_dev(x), args, norm_gamma=to_dev(gamma) if norm else None, eps=1e-6)
    torch.cuda.synchronize()
    for i, (C, conv, l2) in enumerate(segs):
        y_ref, h_ref = _oracle_seg(xn, W[i], cw[i], hist[i], l2)
        _close(to_np(outs[i]), y_ref)
        if conv:
            h = to_np(args[i]["conv_state_out"])
            assert np.array_equal(h[:, :, :2], hist[i][:, :, 1:])        # shifted history is exact
            _close(h[:, :, 2], h_ref[:, :, 2])                            # this step's projected value


def test_decode_proj_matches_tiled_projection_at_t1(cuda_device):
    """The GEMV path and the prefill projection kernel (T = 1, same history)
    agree, including the conv history each leaves behind."""
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(3)
    B, D, C = 2, 2048, 2048
    x, W, cw, hist = _bf16(rng, (B, D)), _bf16(rng, (C, D), D ** -0.5), _bf16(rng, (C, 4), 0.5), _bf16(rng, (B, C, 3))
    h1 = torch.empty(B, C, 3, dtype=torch.bfloat16, device="cuda")
    y_tiled = ops.proj_conv_silu(to_dev(x)[:, None, :], to_dev(W), to_dev(cw), conv_state_in=to_dev(hist),
                                 conv_state_out=h1, l2norm_group=128)
    h2 = to_dev(hist)                                                     # in place
    (y_gemv,) = ops.decode_proj(to_dev(x), [dict(W=to_dev(W), conv_w=to_dev(cw), conv_state_in=h2,
                                                  conv_state_out=h2, l2_group=128)])
    torch.cuda.synchronize()
    _close(to_np(y_gemv), to_np(y_tiled[:, 0]))
    _close(to_np(h2), to_np(h1))


def test_decode_proj_output_projection_shape(cuda_device):
    """The layer's output projection: x [B, 4096] -> [B, 2048], plain rows."""
    import torch
    from gdn_18646_b200 import ops
    rng = np.random.default_rng(5)
    B, D, C = 2, 4096, 2048
    x, W = _bf16(rng, (B, D)), _bf16(rng, (C, D), D ** -0.5)
    (y,) = ops.decode_proj(to_dev(x), [dict(W=to_dev(W))])
    ref = (to_dev(x).float() @ to_dev(W).float().T).bfloat16()
    torch.cuda.synchronize()
    _close(to_np(y), to_np(ref), frac=0.02)
