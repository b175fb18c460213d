"""Head-sharded output projection fused with its reduce-scatter
(gdn_outproj_rs_fwd + gdn_outproj_reduce).  On one GPU the `world` ranks are
emulated in turn: every rank's launch writes into every owner's receive buffer
(local buffers here, peer-mapped ones across GPUs; the kernel only sees device
pointers), then each owner reduces its slots.  Against the oracle's
restatement (partials rounded to bf16, summed in rank order): the tensor-core
and numpy fp32 sums differ in order, so a partial may round one bf16 ulp apart;
the bar is a few ulps on a small fraction of elements."""
import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import to_dev, to_np

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, world, seed):
    rng = np.random.default_rng(seed)
    xs = [O.f32_to_bf16(rng.standard_normal((M, K), dtype=np.float32)) for _ in range(world)]
    Ws = [O.f32_to_bf16(rng.standard_normal((N, K), dtype=np.float32) * np.float32(K ** -0.5)) for _ in range(world)]
    return xs, Ws


def _close(got, want, mag):
    """A partial that rounds one bf16 ulp apart moves the sum by that ulp, which is
    relative to the partial, not to the (possibly much smaller) sum: the bound is
    one ulp of every partial plus one of the result.  `mag` = sum over ranks of
    |partial| (fp32)."""
    g, w = O.bf16_to_f32(got), O.bf16_to_f32(want)
    d = np.abs(g - w)
    assert np.all(d <= mag * 2.0 ** -7 + np.abs(w) * 2.0 ** -7 + 1e-6), f"max diff {d.max():.3e}"
    assert np.mean(g != w) <= 0.02, f"{np.mean(g != w):.4f} of elements differ"


@pytest.mark.parametrize("M,N,K,world", [(1024, 256, 128, 2), (2048, 384, 256, 4), (512, 128, 64, 1),
                                         (4096, 2048, 512, 8)])
def test_outproj_rs_emulated_ranks(cuda_device, M, N, K, world):
    import torch
    from gdn_18646_b200 import ops
    xs, Ws = _inputs(M, N, K, world, seed=M + N + K + world)
    rows = M // world
    bufs = [torch.full((world, rows, N), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    ptrs = [b.data_ptr() for b in bufs]
    for r in range(world):
        ops.outproj_rs(to_dev(xs[r]), to_dev(Ws[r]), ptrs, r, world)
    outs = [ops.outproj_reduce(bufs[d]) for d in range(world)]
    torch.cuda.synchronize()
    want = O.outproj_reduce_scatter(xs, Ws)
    mag = sum(np.abs(np.matmul(O.bf16_to_f32(x), O.bf16_to_f32(W).T)) for x, W in zip(xs, Ws))
    got = np.concatenate([to_np(o) for o in outs])
    _close(got, want, mag)


def test_outproj_rs_matches_full_projection(cuda_device):
    """Sum of head-sharded partials == the unsharded projection of the
    concatenated heads (torch fp32 reference), within bf16 rounding."""
    import torch
    from gdn_18646_b200 import ops
    M, N, K, world = 1024, 2048, 1024, 4
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(M, K, generator=g, device="cuda").bfloat16()
    W = (torch.randn(N, K, generator=g, device="cuda") * K ** -0.5).bfloat16()
    kr = K // world
    rows = M // world
    bufs = [torch.empty(world, rows, N, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    for r in range(world):
        ops.outproj_rs(x[:, r * kr:(r + 1) * kr].contiguous(), W[:, r * kr:(r + 1) * kr].contiguous(),
                       [b.data_ptr() for b in bufs], r, world)
    y = torch.cat([ops.outproj_reduce(b) for b in bufs])
    ref = x.float() @ W.float().T
    torch.cuda.synchronize()
    err = (y.float() - ref).abs().max().item()
    assert err <= 0.02 * ref.abs().max().item(), err
