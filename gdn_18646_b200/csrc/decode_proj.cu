// decode_proj.cu -- the input projections of one decode step as a single
// weight-streaming GEMV launch.
//
// For a decode step (one token per sequence, B <= 8 rows) the projections are
// bound by reading the weights once, not by math.  The reference layer instead
// re-runs the fused projection kernel over the last 4 inputs every step
// (gdn_layer.py:58-69, _decode_fused_proj_step) to rebuild the conv window.
// Here the conv window is a cache of the last 3 projected values per channel
// (the same history the prefill leaves behind), so each step projects one
// token and shifts the cache:
//
//   p       = bf16(x . W[c])                           (fp32 accumulate)
//   conv    = bf16(h0 w0 + h1 w1 + h2 w2 + p w3)       (conv segments)
//   y       = bf16(SiLU(conv))  or  bf16(p)            (plain segments: z, a, b, W_o)
//   y       = bf16(y / sqrt(sum_group y^2 + 1e-6))     (L2-normalised groups: q, k)
//   history = (h1, h2, p)
//
// with the bf16 rounding points of reference/fused_proj_conv_silu_ref.py:54-66
// (and of the prefill projection kernel).  An optional RMSNorm of x
// (reference/rmsnorm_ref.py:24-28) is fused in front: every CTA normalises the
// B rows it needs in shared memory.
//
// One launch covers up to kMaxSeg segments (e.g. q | k | v | z | a | b).  Every
// CTA (8 warps) owns 16 channels of one segment, so all CTAs carry the same
// work.  At entry the CTA bulk-copies (cp.async.bulk) its 16 weight rows into
// shared memory at a padded row stride, completing on one mbarrier, while it
// stages x.  The dot products run on tensor cores as warp-level
// mma.sync.m16n8k16 (A = 16 weight rows via ldmatrix, B = the token rows,
// N = 8 >= B): each warp takes one eighth of D, and the eight partial [16 x 8]
// results are added through shared memory.  (A tcgen05 MMA has a fixed cost of
// ~100 cycles per instruction, far more than this N = 8 GEMV needs per K step;
// per 256 weights this costs ~3 instructions instead of ~700 on CUDA cores.)
// An L2 group wider than a CTA (q/k heads of 128 channels) is split over the 8
// CTAs of one thread-block cluster, which exchange their partial sums of
// squares through distributed shared memory (mapa + ld.shared::cluster).

#include <mutex>

#include "common.cuh"

namespace gdn {
namespace {

constexpr int kMaxSeg = 8;
constexpr int kMaxRows = 8;
constexpr int kThreads = 256;
constexpr int kBs = 16;                   // channels per CTA (one MMA tile of rows)
constexpr int kSmemBudget = 205 * 1024;   // weight rows + x rows + partial sums per CTA
std::once_flag g_attr_once[64];
bool g_attr_ok[64];

struct Seg {
    const uint16_t* W;         // [C, D]
    uint16_t* y;               // [B, ldy]
    const uint16_t* conv_w;    // [C, 4] or null (plain GEMV)
    const uint16_t* conv_in;   // [B, C, 3] or null (zeros)
    uint16_t* conv_out;        // [B, C, 3] or null; may alias conv_in
    int C, ldy, l2, first_cta;
};

struct Args {
    const uint16_t* x;         // [B, D]
    const uint16_t* gamma;     // [D] or null (no RMSNorm)
    float eps;
    int B, D, nseg;
    int cluster;               // CTAs per cluster (1: no cluster barriers)
    int real_ctas;             // CTAs past this only join the cluster barriers
    unsigned int* err;         // device error word (bounded waits)
    Seg seg[kMaxSeg];
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// a float in the shared memory of cluster CTA `rank`, at the address `p` has in this CTA
__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

__device__ __forceinline__ float bf16r(float x) {
    return __uint_as_float(static_cast<uint32_t>(f32_to_bf16_bits(x)) << 16);
}

// A fragment of mma.m16n8k16 (16 x 16 bf16, row-major) from shared memory:
// lane l gives the address of row (l % 16), columns 8 * (l / 16) .. +8.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__global__ void __launch_bounds__(kThreads, 2)
decode_proj_kernel(const __grid_constant__ Args a) {
    const int B = a.B, D = a.D, bs = kBs;
    const int ld = D + 8;                              // padded row stride (elements): conflict-free ldmatrix
    extern __shared__ __align__(16) uint8_t smem[];
    uint16_t* ws = reinterpret_cast<uint16_t*>(smem);                           // [16][ld] weight rows
    uint16_t* xs = ws + kBs * ld;                                               // [8][ld] token rows
    float* acc_s = reinterpret_cast<float*>(xs + kMaxRows * ld);                // [8 warps][16][8] partials
    float* ys = acc_s + (kThreads / 32) * kBs * kMaxRows;                       // [8][16] (L2 groups)
    __shared__ float red[kThreads / 32][kMaxRows];
    __shared__ float part[kMaxRows];                                            // this CTA's sum of squares
    __shared__ __align__(8) uint64_t wbar;                                      // weight rows landed

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool real = static_cast<int>(blockIdx.x) < a.real_ctas;
    int s = 0;
    while (s + 1 < a.nseg && static_cast<int>(blockIdx.x) >= a.seg[s + 1].first_cta) ++s;
    const Seg& g = a.seg[s];
    const int c0 = (blockIdx.x - g.first_cta) * bs;
    const int nc = real ? max(0, min(bs, g.C - c0)) : 0;

    // ---- the CTA's weight rows -> shared memory, one bulk copy per row (lanes of warp 0)
    if (warp == 0) {
        if (lane == 0) {
            mbar_init(&wbar, 1);
            fence_mbar_init();
            if (nc > 0) mbar_arrive_expect_tx(&wbar, static_cast<uint32_t>(nc) * D * 2);
        }
        __syncwarp();
        if (lane < nc)
            bulk_load(ws + static_cast<long>(lane) * ld, g.W + static_cast<long>(c0 + lane) * D,
                      static_cast<uint32_t>(D) * 2, &wbar);
    }

    // ---- stage x (optionally RMS-normalised, reference/rmsnorm_ref.py:24-28) as bf16
    const int nchunk = D >> 3;
    for (int b = 0; b < B; ++b) {
        float ss = 0.f;
        for (int ch = tid; ch < nchunk; ch += kThreads) {
            const uint4 v = *reinterpret_cast<const uint4*>(a.x + static_cast<long>(b) * D + 8 * ch);
            *reinterpret_cast<uint4*>(xs + b * ld + 8 * ch) = v;
            if (a.gamma) {
                const float f0 = __uint_as_float(v.x << 16), f1 = __uint_as_float(v.x & 0xffff0000u);
                const float f2 = __uint_as_float(v.y << 16), f3 = __uint_as_float(v.y & 0xffff0000u);
                const float f4 = __uint_as_float(v.z << 16), f5 = __uint_as_float(v.z & 0xffff0000u);
                const float f6 = __uint_as_float(v.w << 16), f7 = __uint_as_float(v.w & 0xffff0000u);
                ss += f0 * f0 + f1 * f1 + f2 * f2 + f3 * f3 + f4 * f4 + f5 * f5 + f6 * f6 + f7 * f7;
            }
        }
        if (a.gamma) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp][b] = ss;
        }
    }
    for (int i = tid; i < (kMaxRows - B) * nchunk; i += kThreads)   // unused MMA columns read zeros
        *reinterpret_cast<uint4*>(xs + (B + i / nchunk) * ld + 8 * (i % nchunk)) = make_uint4(0, 0, 0, 0);
    __syncthreads();
    if (a.gamma) {
        for (int b = 0; b < B; ++b) {
            float ss = 0.f;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) ss += red[w][b];
            const float r = rsqrtf(ss / static_cast<float>(D) + a.eps);
            for (int ch = tid; ch < nchunk; ch += kThreads) {
                uint4* p = reinterpret_cast<uint4*>(xs + b * ld + 8 * ch);
                const uint4 v = *p;
                const uint4 gm = __ldg(reinterpret_cast<const uint4*>(a.gamma) + ch);
                const uint32_t xu[4] = {v.x, v.y, v.z, v.w}, gu[4] = {gm.x, gm.y, gm.z, gm.w};
                uint32_t o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    o[i] = pack_bf16x2((__uint_as_float(xu[i] << 16) * r) * __uint_as_float(gu[i] << 16),
                                       (__uint_as_float(xu[i] & 0xffff0000u) * r) *
                                           __uint_as_float(gu[i] & 0xffff0000u));
                *p = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
        __syncthreads();
    }

    // ---- [16 channels x 8 rows] = W x^T on tensor cores, warp w over K in [w D/8, (w+1) D/8)
    if (nc > 0) {
        mbar_wait(&wbar, 0, a.err);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int kw = D / (kThreads / 32);
        const int gq = lane >> 2, t4 = lane & 3;
        const uint16_t* arow = ws + (lane & 15) * ld + ((lane >> 4) << 3);
        const uint16_t* brow = xs + gq * ld + 2 * t4;
        for (int k0 = warp * kw; k0 < (warp + 1) * kw; k0 += 16) {
            uint32_t af[4];
            ldmatrix_x4(af, arow + k0);
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(brow + k0);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(brow + k0 + 8);
            mma_bf16_16816(acc, af, b0, b1);
        }
        // C fragment: rows gq, gq + 8 (channels), columns 2 t4, 2 t4 + 1 (token rows)
        float* pw = acc_s + warp * kBs * kMaxRows;
        pw[gq * kMaxRows + 2 * t4] = acc[0];
        pw[gq * kMaxRows + 2 * t4 + 1] = acc[1];
        pw[(gq + 8) * kMaxRows + 2 * t4] = acc[2];
        pw[(gq + 8) * kMaxRows + 2 * t4 + 1] = acc[3];
    }
    __syncthreads();

    // ---- epilogue per (channel, row): thread tid < 128 takes channel tid / 8, row tid % 8
    if (tid < kBs * kMaxRows) {
        const int cl = tid >> 3, b = tid & 7;
        if (cl < nc && b < B) {
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) sum += acc_s[(w * kBs + cl) * kMaxRows + b];
            const int c = c0 + cl;
            const float p = bf16r(sum);
            float yv = p;
            if (g.conv_w) {
                const uint2 cw = *reinterpret_cast<const uint2*>(g.conv_w + 4 * static_cast<long>(c));
                const long hb = (static_cast<long>(b) * g.C + c) * 3;
                float h0 = 0.f, h1 = 0.f, h2 = 0.f;
                if (g.conv_in) {
                    h0 = bf16_bits_to_f32(g.conv_in[hb]);
                    h1 = bf16_bits_to_f32(g.conv_in[hb + 1]);
                    h2 = bf16_bits_to_f32(g.conv_in[hb + 2]);
                }
                float conv = h0 * __uint_as_float(cw.x << 16);
                conv = fmaf(h1, __uint_as_float(cw.x & 0xffff0000u), conv);
                conv = fmaf(h2, __uint_as_float(cw.y << 16), conv);
                conv = fmaf(p, __uint_as_float(cw.y & 0xffff0000u), conv);
                const float cr = bf16r(conv);
                yv = bf16r(__fdividef(cr, 1.f + __expf(-cr)));              // SiLU
                if (g.conv_out) {
                    g.conv_out[hb] = f32_to_bf16_bits(h1);
                    g.conv_out[hb + 1] = f32_to_bf16_bits(h2);
                    g.conv_out[hb + 2] = f32_to_bf16_bits(p);
                }
            }
            if (g.l2) ys[b * bs + cl] = yv;
            else g.y[static_cast<long>(b) * g.ldy + c] = f32_to_bf16_bits(yv);
        }
    }

    // ---- per-group L2 norm (fp32, eps 1e-6), then the bf16 store.  Groups of at
    //      most bs channels stay in the CTA; wider ones (g = k * bs) span k
    //      consecutive CTAs of the cluster, which add up their partial sums.
    //      Every CTA of the launch takes part in both cluster barriers.
    const bool l2 = nc > 0 && g.l2 != 0;
    const bool wide = l2 && g.l2 > bs;
    if (a.cluster > 1) {
        __syncthreads();
        if (wide && warp < B) {                        // this CTA's sum of squares per row
            float ss = 0.f;
            for (int e = lane; e < nc; e += 32) ss += ys[warp * bs + e] * ys[warp * bs + e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) part[warp] = ss;
        }
        cluster_sync_all();                            // partials visible cluster-wide
        if (wide) {
            const int k = g.l2 / bs;                   // CTAs per group
            const uint32_t r0 = (cluster_rank() / k) * k;
            for (int item = tid; item < B * nc; item += kThreads) {
                const int b = item / nc, e = item - b * nc;
                float ss = 0.f;
                for (int r = 0; r < k; ++r) ss += ld_cluster_f32(&part[b], r0 + r);
                const float inv = 1.f / sqrtf(ss + 1e-6f);
                g.y[static_cast<long>(b) * g.ldy + c0 + e] = f32_to_bf16_bits(ys[b * bs + e] * inv);
            }
        }
        cluster_sync_all();                            // no CTA leaves while a peer reads it
    }
    if (l2 && !wide) {
        __syncthreads();
        const int ng = nc / g.l2;
        for (int item = warp; item < B * ng; item += kThreads / 32) {
            const int b = item / ng, gi = item - b * ng;
            const float* yr = ys + b * bs + gi * g.l2;
            float ss = 0.f;
            for (int e = lane; e < g.l2; e += 32) ss += yr[e] * yr[e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.f / sqrtf(ss + 1e-6f);
            for (int e = lane; e < g.l2; e += 32)
                g.y[static_cast<long>(b) * g.ldy + c0 + gi * g.l2 + e] = f32_to_bf16_bits(yr[e] * inv);
        }
    }
}

}  // namespace
}  // namespace gdn

namespace gdn {
namespace {
// weight rows and token rows (padded stride), partial sums and L2 scratch
int smem_bytes(int /*B*/, int D) {
    return (kBs + kMaxRows) * (D + 8) * 2 + (kThreads / 32) * kBs * kMaxRows * 4 + kMaxRows * kBs * 4;
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_decode_proj_fwd(const void* x, const void* norm_gamma, float eps, int B, int D,
                                   const gdn_proj_segment* segs, int nseg, void* stream) {
    using namespace gdn;
    if (!x || !segs) return fail(GDN_ERR_NULL, "gdn_decode_proj_fwd: x and segs are required");
    if (B < 1 || B > kMaxRows || D < 256 || D % 256 != 0 || smem_bytes(B, D) > kSmemBudget)
        return fail(GDN_ERR_SHAPE, "gdn_decode_proj_fwd: need 1 <= B <= %d, D %% 256 == 0 and D <= 4096 (got B=%d D=%d)",
                    kMaxRows, B, D);
    if (nseg < 1 || nseg > kMaxSeg)
        return fail(GDN_ERR_SHAPE, "gdn_decode_proj_fwd: 1..%d segments (got %d)", kMaxSeg, nseg);
    if (!aligned16(x) || (norm_gamma && !aligned16(norm_gamma)))
        return fail(GDN_ERR_ALIGN, "gdn_decode_proj_fwd: x and norm_gamma must be 16-byte aligned");
    Args a;
    a.x = static_cast<const uint16_t*>(x);
    a.gamma = static_cast<const uint16_t*>(norm_gamma);
    a.eps = eps;
    a.B = B;
    a.D = D;
    a.nseg = nseg;
    for (int i = 0; i < nseg; ++i) {
        const gdn_proj_segment& s = segs[i];
        if (!s.W || !s.y) return fail(GDN_ERR_NULL, "gdn_decode_proj_fwd: segment %d needs W and y", i);
        if (s.C < 16 || s.C % 16 != 0 || s.ldy < s.C)
            return fail(GDN_ERR_SHAPE, "gdn_decode_proj_fwd: segment %d: C %% 16 == 0 and ldy >= C (got C=%d ldy=%d)",
                        i, s.C, s.ldy);
        if (s.l2_group != 0 && (s.l2_group < 8 || 128 % s.l2_group != 0 || s.C % s.l2_group != 0))
            return fail(GDN_ERR_SHAPE,
                        "gdn_decode_proj_fwd: segment %d: l2_group %d must divide 128 and C (C=%d)", i, s.l2_group,
                        s.C);
        if (!s.conv_w && (s.conv_state_in || s.conv_state_out))
            return fail(GDN_ERR_NULL, "gdn_decode_proj_fwd: segment %d: conv states need conv_w", i);
        if (!aligned16(s.W) || (s.conv_w && (reinterpret_cast<uintptr_t>(s.conv_w) & 7u)))
            return fail(GDN_ERR_ALIGN, "gdn_decode_proj_fwd: segment %d: W 16-byte, conv_w 8-byte aligned", i);
        Seg& d = a.seg[i];
        d.W = static_cast<const uint16_t*>(s.W);
        d.y = static_cast<uint16_t*>(s.y);
        d.conv_w = static_cast<const uint16_t*>(s.conv_w);
        d.conv_in = static_cast<const uint16_t*>(s.conv_state_in);
        d.conv_out = static_cast<uint16_t*>(s.conv_state_out);
        d.C = s.C;
        d.ldy = s.ldy;
        d.l2 = s.l2_group;
    }
    int st = check_sm100();
    if (st != GDN_OK) return st;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: no current device");
    // CTA plan, 16 channels per CTA: an L2 group wider than that spans g/16 CTAs
    // of one cluster, so such a segment starts on a cluster boundary
    int cl = 1;
    for (int i = 0; i < nseg; ++i)
        if (a.seg[i].l2 > kBs) cl = cl > a.seg[i].l2 / kBs ? cl : a.seg[i].l2 / kBs;
    int n = 0;
    for (int i = 0; i < nseg; ++i) {
        if (a.seg[i].l2 > kBs) n = (n + cl - 1) / cl * cl;
        a.seg[i].first_cta = n;
        n += (a.seg[i].C + kBs - 1) / kBs;
    }
    a.cluster = cl;
    a.real_ctas = n;
    const int ctas = (n + cl - 1) / cl * cl;
    const int smem = smem_bytes(B, D);
    a.err = device_error_word();
    (void)sms;
    std::call_once(g_attr_once[dev], [dev] {
        g_attr_ok[dev] = cudaFuncSetAttribute(decode_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kSmemBudget) == cudaSuccess;
    });
    if (!g_attr_ok[dev]) return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: cannot grant shared memory");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_proj_kernel, a);
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: launch failed: %s", cudaGetErrorString(e));
    return launch_status("gdn_decode_proj_fwd");
}
