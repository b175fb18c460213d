"""The reference repository's own CUDA kernels, compiled for sm_100a by
oracle/build_ref_kernels.py, run beside this library's kernels on the same B200:
the same inputs go through both ``exts``-style modules (the reference's
``forward`` signatures, kernels/decode.cu:172-214, kernels/rmsnorm.cu:280-293,
kernels/fused_proj_conv_silu.cu:298-355), the outputs are compared, and both are
timed with CUDA events, the L2 flushed before every timed call.

The ops and their calls are the reference bench's per-op list
(bench_gdn.py:275-300); the shapes are the benchmark configurations': decode at
config 2 (B=256, H=32, dk=dv=128), and at config 3 (x [2, 8192, 2048]) the
RMSNorm of 16384 rows of 2048 and the fused q/k/v projection W [8192, 2048]
(2048 + 2048 + 4096 output channels) with the k=4 causal conv and SiLU.  The
reference's prefill kernel only runs H=16, dk=128, dv=256
(kernels/prefill_chunked.cu:15-18): it is compared at config 1's batch, length
and distributions with that head shape, both outputs also against the fp64
oracle on a sampled head.

Skipped when the comparator modules were not built (no reference checkout on the
machine that built the repository)."""
import json
import os

import numpy as np
import pytest

from oracle import build_ref_kernels as R

pytestmark = pytest.mark.gpu

L2_FLUSH_BYTES = 256 << 20


def _ref(name):
    mod = R.load(name)
    if mod is None:
        pytest.skip(f"{name} not built (python oracle/build_ref_kernels.py <reference checkout>)")
    return mod


def _time_ms(fn, iters=20, warmup=3):
    """Median CUDA-event time of fn() on the current stream, with a 256 MB write
    flushing L2 before each call."""
    import torch
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for i in range(warmup + iters):
        flush.zero_()
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        if i >= warmup:
            ts.append(e0.elapsed_time(e1))
    return float(np.median(ts))


def _report(kernel, shape, ours_ms, ref_ms, alg_bytes=None, flops=None):
    rec = {"kernel": kernel, "shape": shape, "ours_ms": round(ours_ms, 4), "reference_ms": round(ref_ms, 4),
           "speedup": round(ref_ms / ours_ms, 2)}
    if alg_bytes:
        rec["ours_GBs"] = round(alg_bytes / ours_ms / 1e6, 1)
        rec["reference_GBs"] = round(alg_bytes / ref_ms / 1e6, 1)
    if flops:
        rec["ours_TFs"] = round(flops / ours_ms / 1e9, 1)
        rec["reference_TFs"] = round(flops / ref_ms / 1e9, 1)
    line = json.dumps(rec)
    print("REFCMP " + line)
    out = os.environ.get("GDN_REFCMP_OUT")
    if out:
        with open(out, "a") as f:
            f.write(line + "\n")


def test_decode_vs_reference_kernel(cuda_device):
    import torch
    from gdn_18646_b200 import ops
    ref = _ref("gdn_ref_decode")
    ours = ops.exts()["decode"]
    B, H, dk, dv = 256, 32, 128, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    bf = torch.bfloat16
    q = torch.nn.functional.normalize(torch.randn(B, H, dk, device="cuda", generator=g), dim=-1).to(bf)
    k = torch.nn.functional.normalize(torch.randn(B, H, dk, device="cuda", generator=g), dim=-1).to(bf)
    v = torch.randn(B, H, dv, device="cuda", generator=g).to(bf)
    a = torch.randn(B, H, device="cuda", generator=g).to(bf)
    b = torch.randn(B, H, device="cuda", generator=g).to(bf)
    A_log = torch.full((H,), float(np.log(0.1)), device="cuda")
    dtb = torch.randn(H, device="cuda", generator=g) * 0.1
    S_in = torch.randn(B, H, dk, dv, device="cuda", generator=g) * 0.02
    scale = dk ** -0.5
    o_r, S_r = torch.empty(B, H, dv, device="cuda"), torch.empty_like(S_in)
    o_o, S_o = torch.empty_like(o_r), torch.empty_like(S_in)
    ref.forward(q, k, v, a, b, A_log, dtb, S_in, scale, o_r, S_r)
    ours.forward(q, k, v, a, b, A_log, dtb, S_in, scale, o_o, S_o)
    torch.cuda.synchronize()
    err_o = float((o_o - o_r).abs().max() / o_r.abs().max())
    err_s = float((S_o - S_r).norm() / S_r.norm())
    assert err_o < 1e-5 and err_s < 1e-6, (err_o, err_s)
    t_ref = _time_ms(lambda: ref.forward(q, k, v, a, b, A_log, dtb, S_in, scale, o_r, S_r))
    t_our = _time_ms(lambda: ours.forward(q, k, v, a, b, A_log, dtb, S_in, scale, o_o, S_o))
    alg = 2 * S_in.numel() * 4 + B * H * (2 * dk + dv + 2) * 2 + o_r.numel() * 4
    _report("decode", "B=256 H=32 dk=dv=128", t_our, t_ref, alg_bytes=alg)


def test_rmsnorm_vs_reference_kernel(cuda_device):
    import torch
    from gdn_18646_b200 import ops
    ref = _ref("gdn_ref_rmsnorm")
    ours = ops.exts()["rmsnorm"]
    R_, D = 16384, 2048
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(R_, D, device="cuda", generator=g).to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    y_r = ref.forward(x, gamma, 1e-6, 256, 2)
    y_o = ours.forward(x, gamma, 1e-6, 256, 2)
    torch.cuda.synchronize()
    yr, yo = y_r.float(), y_o.float()
    diff = (yo - yr).abs()
    assert bool((diff <= yr.abs() * 2.0 ** -7 + 1e-6).all()), "more than 1 bf16 ulp apart"
    assert float((yo != yr).float().mean()) <= 0.01
    t_ref = _time_ms(lambda: ref.forward(x, gamma, 1e-6, 256, 2))
    t_our = _time_ms(lambda: ours.forward(x, gamma, 1e-6, 256, 2))
    _report("rmsnorm", "R=16384 D=2048", t_our, t_ref, alg_bytes=2 * x.numel() * 2 + D * 2)


def test_proj_vs_reference_kernel(cuda_device):
    import torch
    from gdn_18646_b200 import ops
    ref = _ref("gdn_ref_proj")
    ours = ops.exts()["proj"]
    B, T, D, Dout = 2, 8192, 2048, 8192
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(B, T, D, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(Dout, D, device="cuda", generator=g) * D ** -0.5).to(torch.bfloat16)
    cw = (torch.randn(Dout, 4, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    y_r = ref.forward(x, W, cw)
    y_o = ours.forward(x, W, cw)
    torch.cuda.synchronize()
    yr, yo = y_r.float(), y_o.float()
    diff = (yo - yr).abs()
    # The reference kernel keeps the projection in fp32 through the conv
    # (kernels/fused_proj_conv_silu.cu:262-293) where its Python reference, and this
    # library, round it to bf16 first (reference/fused_proj_conv_silu_ref.py:54-66):
    # a few output ulps on many elements.  Gate: every element within 4 bf16 ulps
    # (the harness's absolute max-abs < 5e-2, tests/test_fused_proj_conv_silu.py:59,
    # is two ulps at outputs above 4, which these unit-variance inputs reach) and a
    # small relative norm.
    assert bool((diff <= yr.abs() * 2.0 ** -5 + 1e-2).all()), f"max diff {float(diff.max()):.3e}"
    assert float((yo - yr).norm() / yr.norm()) < 1e-2
    t_ref = _time_ms(lambda: ref.forward(x, W, cw), iters=10)
    t_our = _time_ms(lambda: ours.forward(x, W, cw), iters=10)
    _report("proj_conv_silu", "x [2,8192,2048] W [8192,2048]", t_our, t_ref, flops=2.0 * B * T * D * Dout)


def test_prefill_vs_reference_kernel(cuda_device):
    import torch
    from gdn_18646_b200 import ops
    from oracle import gdn_oracle as O
    from tests._util import to_np
    ref = _ref("gdn_ref_prefill")
    ours = ops.exts()["prefill"]
    B, T, H, dk, dv = 4, 4096, 16, 128, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    bf = torch.bfloat16
    q = torch.nn.functional.normalize(torch.randn(B, H, T, dk, device="cuda", generator=g), dim=-1).to(bf)
    k = torch.nn.functional.normalize(torch.randn(B, H, T, dk, device="cuda", generator=g), dim=-1).to(bf)
    v = torch.randn(B, H, T, dv, device="cuda", generator=g).to(bf)
    a = torch.randn(B, H, T, device="cuda", generator=g).to(bf)
    b = torch.randn(B, H, T, device="cuda", generator=g).to(bf)
    A_log = torch.full((H,), float(np.log(0.1)), device="cuda")
    mask = torch.ones(B, T, device="cuda")
    S0 = torch.randn(B, H, dk, dv, device="cuda", generator=g) * 0.02
    scale = dk ** -0.5
    o_r, S_r = ref.prefill(q, k, v, A_log, a, 0.0, b, mask, S0, scale)
    o_o, S_o = ours.prefill(q, k, v, A_log, a, 0.0, b, mask, S0, scale)
    torch.cuda.synchronize()
    # the library against the fp64 oracle on one sampled head (the north_star bar)
    bi, hi = 1, 5
    sl = lambda t: to_np(t[bi:bi + 1, hi:hi + 1])
    o_x, S_x = O.prefill(sl(q), sl(k), sl(v), to_np(A_log[hi:hi + 1]), sl(a), 0.0, sl(b), np.ones((1, T)),
                         state_in=sl(S0), scale=scale, chunk_size=64, dt=np.float64)
    err_o_ours = float(np.abs(O.bf16_to_f32(sl(o_o)) - o_x).max())
    err_s_ours = O.rel_fro(sl(S_o), S_x)
    err_o_ref = float(np.abs(O.bf16_to_f32(sl(o_r)) - o_x).max())
    err_s_ref = O.rel_fro(sl(S_r), S_x)
    print(f"REFCMP prefill vs fp64 oracle (b={bi}, h={hi}): library o {err_o_ours:.2e} state {err_s_ours:.2e}; "
          f"reference kernel o {err_o_ref:.2e} state {err_s_ref:.2e}")
    assert err_o_ours <= 2e-2 and err_s_ours <= 1e-3
    # the two GPU outputs against each other, with the reference harness's mixed
    # tolerance (tests/test_prefill.py:61-62) over every element
    diff = (o_o.float() - o_r.float()).abs()
    assert bool((diff < 1e-2 + 0.05 * o_r.float().abs()).all()), f"max diff {float(diff.max()):.3e}"
    t_ref = _time_ms(lambda: ref.prefill(q, k, v, A_log, a, 0.0, b, mask, S0, scale), iters=5, warmup=1)
    t_our = _time_ms(lambda: ours.prefill(q, k, v, A_log, a, 0.0, b, mask, S0, scale), iters=10)
    alg = B * H * T * (2 * dk * 2 + 2 * dv * 2 + 2 * 2) + 2 * B * H * dk * dv * 4
    _report("prefill", "B=4 T=4096 H=16 dk=128 dv=256", t_our, t_ref, alg_bytes=alg)
