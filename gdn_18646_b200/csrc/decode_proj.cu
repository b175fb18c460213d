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
// One launch covers up to kMaxSeg segments (e.g. q | k | v | z | a | b).  The
// weights are cut into tiles of 16 rows (channels); a tile is the M side of
// warp-level tensor-core MMAs (mma.sync.m16n8k16) whose N side is the <= 8
// token rows.  The kernel is persistent, one CTA per SM, and warp-specialised
// so that the weight stream never waits for an epilogue:
//
//   producer warp   initialises the barriers, streams the first ring's worth
//                   of weight stages (2..8 stages of 16 rows x KC columns,
//                   KC <= 2048, one cp.async.bulk per row and stage, on
//                   full/empty mbarriers), waits for the kernels it depends
//                   on (griddepcontrol: under programmatic dependent launch
//                   the weights start streaming while the previous kernel
//                   still runs), bulk-copies the B token rows and the RMSNorm
//                   weight, then each conv tile's conv weights and history
//                   into a 4-deep side ring and the remaining weight stages.
//                   4 KB row copies stream at the HBM rate; 1 KB rows reached
//                   only ~30% of it.  Every global read of the kernel is one
//                   of these copies: a plain load issued behind the weight
//                   stream waited ~2 us;
//   8 MMA warps     RMS-normalise the token rows in place once, then each
//                   takes one eighth of every stage's K range (ldmatrix A
//                   fragments, B from the token rows) into a per-warp [16 x 8]
//                   accumulator, and hands the tile's eight partials to the
//                   epilogue through a double-buffered shared-memory slot;
//   4 epilogue      one thread per (channel, token row): sum of the partials,
//     warps         conv4 / SiLU / history update / L2 norm and the stores.
//
// (A tcgen05 MMA costs ~100 cycles per instruction whatever N is, which this
// N <= 8 product cannot amortise; mma.sync needs ~3 instructions per 256
// weights, so the SM's issue slots stay far from the limit.)
//
// L2 groups wider than a tile (q/k heads of 128 channels) are handled by a
// thread-block cluster of g/16 CTAs that walk the same sequence of 16*cl
// channel groups, CTA rank r taking tile r of each: every CTA sends its
// per-row partial sum of squares to all peers with st.async (completing on
// the peer's mbarrier), so no cluster-wide barrier is needed in the loop.

#include <mutex>
#include <vector>

#include "common.cuh"

namespace gdn {
namespace {

constexpr int kMaxSeg = 8;
constexpr int kMaxRows = 8;
constexpr int kBs = 16;                        // rows per tile
constexpr int kMmaWarps = 8;
constexpr int kEpiWarps = 4;                   // kBs * kMaxRows threads
constexpr int kProducerWarp = kMmaWarps + kEpiWarps;
constexpr int kThreads = (kProducerWarp + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kMaxKC = 2048;                   // columns per stage (4 KB rows)
constexpr int kMaxCluster = 8;
constexpr int kSide = 4;                       // conv side-ring slots
constexpr int kSideBytes = 128 + kMaxRows * 96; // conv_w [16][4] + history [8][16][3], bf16
constexpr int kSmemBudget = 226 * 1024;
std::once_flag g_attr_once[64];
bool g_attr_ok[64];

struct Seg {
    const uint16_t* W;         // [C, D]
    uint16_t* y;               // [B, ldy]
    const uint16_t* conv_w;    // [C, 4] or null (plain GEMV)
    const uint16_t* conv_in;   // [B, C, 3] or null (zeros)
    uint16_t* conv_out;        // [B, C, 3] or null; may alias conv_in
    int C, ldy, l2, first_group;
};

struct Args {
    const uint16_t* x;         // [B, D]
    const uint16_t* gamma;     // [D] or null (no RMSNorm)
    float eps;
    int B, D, KC, nst;         // KC: columns per ring stage; nst: ring stages
    int nseg, cl, ngroups;     // cl: CTAs per cluster = tiles per group
    int pdl;                   // launched with programmatic stream serialisation
    unsigned int* err;         // device error word (bounded waits)
    Seg seg[kMaxSeg];
};

// shared memory besides the ring: x rows | RMSNorm weight | partials (2 buffers) | L2 values (2) |
// exchanged sums (2) | conv side ring
int fixed_smem_bytes(int B, int D) {
    return B * (D + 8) * 2 + D * 2 + 2 * kMmaWarps * kBs * kMaxRows * 4 + 2 * kMaxRows * kBs * 4 +
           2 * kMaxCluster * kMaxRows * 4 + kSide * kSideBytes;
}
int stage_smem_bytes(int KC) { return kBs * (KC + 8) * 2; }

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Relaxed arrive: the only ordering the cluster barriers carry is that of the
// mbarrier initialisations, published by fence.mbarrier_init.release.cluster.
// (A release arrive issued while the CTA's weight copies were in flight took
// ~5 us to retire.)
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// v -> the float at `local` (an address of this CTA's shared memory) in cluster
// CTA `rank`, completing 4 bytes on that CTA's mbarrier `bar`
__device__ __forceinline__ void st_async_f32(const float* local, uint64_t* bar, uint32_t rank, float v) {
    uint32_t ra, rb;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"(smem_u32(bar)), "r"(rank));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(ra),
                 "r"(__float_as_uint(v)), "r"(rb)
                 : "memory");
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

// mbar_wait_or_abort with cluster-scope acquire (the data came from peers' st.async)
__device__ __forceinline__ bool mbar_wait_cluster_or_abort(uint64_t* bar, uint32_t parity, unsigned int* err,
                                                           volatile int* abort) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (*abort) return false;
        if (clock64() - t0 > (1ll << 31)) {
            if (err) atomicOr(err, DERR_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
}

// One exchange of per-row partial sums over the cluster (the 128 epilogue
// threads, index e): threads e = b < B send `part` to slot [rank][b] of every
// CTA, then all wait until this CTA has the cl * B values of this exchange.
// Buffers and mbarriers alternate between exchanges.  Thread e = 0 re-arms the
// mbarrier as soon as its phase completed: no peer can send into it again
// before this CTA's next exchange, which its 128 threads start only after
// reading this one, so the slots stay valid for the caller.  Returns this
// exchange's [cl][8] slots.
__device__ __forceinline__ const float* exchange(const Args& a, float* xsum, uint64_t* xbar, uint32_t rank,
                                                 uint32_t& nw, int e, float part, volatile int* abort_flag) {
    const uint32_t buf = nw & 1u;
    float* slot = xsum + buf * kMaxCluster * kMaxRows;
    if (e < a.B)
        for (int r = 0; r < a.cl; ++r) st_async_f32(slot + rank * kMaxRows + e, &xbar[buf], static_cast<uint32_t>(r), part);
    mbar_wait_cluster_or_abort(&xbar[buf], (nw >> 1) & 1u, a.err, abort_flag);
    if (e == 0) mbar_arrive_expect_tx(&xbar[buf], a.cl * a.B * 4);
    ++nw;
    return slot;
}

// The segment of group j and the first row of this CTA's tile in it (-1: no tile).
__device__ __forceinline__ int tile_of(const Args& a, int j, uint32_t rank, int& s) {
    s = 0;
    while (s + 1 < a.nseg && j >= a.seg[s + 1].first_group) ++s;
    const int row0 = ((j - a.seg[s].first_group) * a.cl + static_cast<int>(rank)) * kBs;
    return row0 < a.seg[s].C ? row0 : -1;
}

__global__ void __launch_bounds__(kThreads, 1)
decode_proj_kernel(const __grid_constant__ Args a) {
    const int B = a.B, D = a.D, KC = a.KC, nk = D / KC, nst = a.nst;
    const int lds = KC + 8, ldx = D + 8;               // padded strides (elements): conflict-free ldmatrix / B loads
    extern __shared__ __align__(16) uint8_t smem[];
    uint16_t* ring = reinterpret_cast<uint16_t*>(smem);                          // [nst][16][lds]
    uint16_t* xs = ring + nst * kBs * lds;                                       // [B][ldx]
    uint16_t* gs = xs + B * ldx;                                                 // [D] RMSNorm weight
    float* acc_s = reinterpret_cast<float*>(gs + D);                             // [2][8 warps][16][8]
    float* ys = acc_s + 2 * kMmaWarps * kBs * kMaxRows;                          // [2][8][16]
    float* xsum = ys + 2 * kMaxRows * kBs;                                       // [2][kMaxCluster][8]
    uint8_t* side = reinterpret_cast<uint8_t*>(xsum + 2 * kMaxCluster * kMaxRows);   // [kSide][kSideBytes]
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], xfull, accfull[2], accempty[2], xbar[2],
        sidefull[kSide], sideempty[kSide];
    __shared__ float red[kMmaWarps][kMaxRows];
    __shared__ int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank(), cid = cluster_id(), ncl = cluster_count();

    if (warp == kProducerWarp) {
        // ---------------- producer: barriers, token rows (+ RMSNorm weight), then weight rows -> ring
        if (lane == 0) {
            for (int i = 0; i < nst; ++i) {
                mbar_init(&full[i], 1);
                mbar_init(&empty[i], kMmaWarps);
            }
            mbar_init(&xfull, 1);
            for (int i = 0; i < 2; ++i) {
                mbar_init(&accfull[i], kMmaWarps);
                mbar_init(&accempty[i], kEpiWarps);
                mbar_init(&xbar[i], 1);
            }
            for (int i = 0; i < kSide; ++i) {
                mbar_init(&sidefull[i], 1);
                mbar_init(&sideempty[i], kEpiWarps);
            }
            abort_flag = 0;
            fence_mbar_init();
            if (a.cl > 1) {                            // both exchange buffers armed up front
                mbar_arrive_expect_tx(&xbar[0], a.cl * B * 4);
                mbar_arrive_expect_tx(&xbar[1], a.cl * B * 4);
            }
        }
        __syncwarp();
        named_bar(0, kThreads);                        // barriers initialised
        cluster_arrive();
        if (lane == 0) pdl_launch_dependents();        // the next kernel may launch (it waits for us)
        // token rows and RMSNorm weight: data of earlier kernels, so after the wait
        auto issue_x = [&]() {
            pdl_wait_prior();
            if (lane == 0) mbar_arrive_expect_tx(&xfull, static_cast<uint32_t>(B + (a.gamma ? 1 : 0)) * D * 2);
            __syncwarp();
            if (lane < B)
                bulk_load(xs + lane * ldx, a.x + static_cast<long>(lane) * D, static_cast<uint32_t>(D) * 2, &xfull);
            if (lane == kMaxRows && a.gamma) bulk_load(gs, a.gamma, static_cast<uint32_t>(D) * 2, &xfull);
        };
        if (!a.pdl) {
            // launched after the previous kernel completed: the token rows go first and
            // land before the weight stream starts (issued next to it they queue behind
            // ~20 MB of weight reads, ~5 us)
            issue_x();
            if (lane == 0) mbar_wait_or_abort(&xfull, 0, a.err, &abort_flag);
            __syncwarp();
        }
        // Phase A: the first ring's worth of weight stages.  Weights are constant
        // operands: under programmatic dependent launch they stream while the
        // previous kernel still runs.
        const uint32_t stage_bytes = static_cast<uint32_t>(kBs) * KC * 2;
        uint32_t pre = 0;
        for (int j = static_cast<int>(cid); j < a.ngroups && pre < static_cast<uint32_t>(nst);
             j += static_cast<int>(ncl)) {
            int s;
            const int row0 = tile_of(a, j, rank, s);
            if (row0 < 0) continue;
            const uint16_t* W = a.seg[s].W + static_cast<long>(row0 + lane) * D;
            for (int kc = 0; kc < nk && pre < static_cast<uint32_t>(nst); ++kc, ++pre) {
                if (lane == 0) mbar_arrive_expect_tx(&full[pre], stage_bytes);      // fresh slot
                __syncwarp();
                if (lane < kBs)
                    bulk_load(ring + (pre * kBs + lane) * lds, W + kc * KC, static_cast<uint32_t>(KC) * 2, &full[pre]);
            }
        }
        if (a.pdl) issue_x();
        // Phase B (after the wait: the conv history is data of earlier kernels): conv side data of every tile, and the weight stages past the first ring
        uint32_t q = 0, nsd = 0;
        for (int j = static_cast<int>(cid); j < a.ngroups; j += static_cast<int>(ncl)) {
            int s;
            const int row0 = tile_of(a, j, rank, s);
            if (row0 < 0) continue;
            const Seg& g = a.seg[s];
            if (g.conv_w) {                            // conv weights + history of the tile's channels
                const uint32_t sl = nsd % kSide, ph = (nsd / kSide) & 1u;
                uint8_t* sd = side + sl * kSideBytes;
                if (lane == 0) {
                    mbar_wait_or_abort(&sideempty[sl], ph ^ 1u, a.err, &abort_flag);
                    mbar_arrive_expect_tx(&sidefull[sl], 128u + (g.conv_in ? static_cast<uint32_t>(B) * 96u : 0u));
                }
                __syncwarp();
                if (lane == 0) bulk_load(sd, g.conv_w + 4 * static_cast<long>(row0), 128u, &sidefull[sl]);
                if (g.conv_in && lane >= 1 && lane <= B)
                    bulk_load(sd + 128 + (lane - 1) * 96, g.conv_in + (static_cast<long>(lane - 1) * g.C + row0) * 3, 96u,
                              &sidefull[sl]);
                ++nsd;
            }
            const uint16_t* W = g.W + static_cast<long>(row0 + lane) * D;
            for (int kc = 0; kc < nk; ++kc, ++q) {
                if (q < pre) continue;                 // issued in phase A
                const uint32_t st = q % nst, ph = (q / nst) & 1u;
                if (lane == 0) {
                    mbar_wait_or_abort(&empty[st], ph ^ 1u, a.err, &abort_flag);
                    mbar_arrive_expect_tx(&full[st], stage_bytes);
                }
                __syncwarp();
                if (lane < kBs)
                    bulk_load(ring + (st * kBs + lane) * lds, W + kc * KC, static_cast<uint32_t>(KC) * 2, &full[st]);
            }
        }
        cluster_wait();
    } else if (warp < kMmaWarps) {
        // ---------------- MMA warps
        named_bar(0, kThreads);                        // barriers initialised
        cluster_arrive();                              // peers' barriers exist before any st.async
        mbar_wait_or_abort(&xfull, 0, a.err, &abort_flag);
        if (a.gamma) {                                 // RMSNorm of the token rows, reference/rmsnorm_ref.py:24-28
            const int nchunk = D >> 3;
            for (int b = 0; b < B; ++b) {
                float ss = 0.f;
                for (int ch = tid; ch < nchunk; ch += kMmaWarps * 32) {
                    const uint4 v = *reinterpret_cast<const uint4*>(xs + b * ldx + 8 * ch);
                    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float f0 = __uint_as_float(u[i] << 16), f1 = __uint_as_float(u[i] & 0xffff0000u);
                        ss = fmaf(f0, f0, ss);
                        ss = fmaf(f1, f1, ss);
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                if (lane == 0) red[warp][b] = ss;
            }
            named_bar(1, kMmaWarps * 32);
            for (int b = 0; b < B; ++b) {
                float ss = 0.f;
#pragma unroll
                for (int w = 0; w < kMmaWarps; ++w) ss += red[w][b];
                const float r = rsqrtf(ss / static_cast<float>(D) + a.eps);
                for (int ch = tid; ch < nchunk; ch += kMmaWarps * 32) {
                    uint4* p = reinterpret_cast<uint4*>(xs + b * ldx + 8 * ch);
                    const uint4 v = *p;
                    const uint4 gm = *reinterpret_cast<const uint4*>(gs + 8 * ch);
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
            named_bar(1, kMmaWarps * 32);
        }
        cluster_wait();

        const int gq = lane >> 2, t4 = lane & 3;
        const bool brow_ok = gq < B;                   // MMA columns past B multiply zeros
        const uint16_t* brow = xs + (brow_ok ? gq : 0) * ldx + 2 * t4;
        const int kw = KC / kMmaWarps;                 // K columns of a stage per warp (a multiple of 32)
        uint32_t q = 0, nt = 0;
        for (int j = static_cast<int>(cid); j < a.ngroups; j += static_cast<int>(ncl)) {
            int s;
            if (tile_of(a, j, rank, s) < 0) continue;
            // [16 rows x 8 token rows] over this warp's share of every stage; two
            // accumulators halve the dependent MMA chain
            float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            for (int kc = 0; kc < nk; ++kc, ++q) {
                const uint32_t st = q % nst, ph = (q / nst) & 1u;
                mbar_wait_or_abort(&full[st], ph, a.err, &abort_flag);
                const uint16_t* arow = ring + (st * kBs + (lane & 15)) * lds + ((lane >> 4) << 3) + warp * kw;
                const uint16_t* bk = brow + kc * KC + warp * kw;
#pragma unroll 4
                for (int k0 = 0; k0 < kw; k0 += 32) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t af[4];
                        ldmatrix_x4(af, arow + k0 + 16 * h);
                        const uint32_t b0 = brow_ok ? *reinterpret_cast<const uint32_t*>(bk + k0 + 16 * h) : 0u;
                        const uint32_t b1 = brow_ok ? *reinterpret_cast<const uint32_t*>(bk + k0 + 16 * h + 8) : 0u;
                        mma_bf16_16816(acc[h], af, b0, b1);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
            // C fragment: rows gq, gq + 8 (channels), columns 2 t4, 2 t4 + 1 (token rows)
            const uint32_t buf = nt & 1u;
            mbar_wait_or_abort(&accempty[buf], ((nt >> 1) & 1u) ^ 1u, a.err, &abort_flag);
            float* pw = acc_s + (buf * kMmaWarps + warp) * kBs * kMaxRows;
            pw[gq * kMaxRows + 2 * t4] = acc[0][0] + acc[1][0];
            pw[gq * kMaxRows + 2 * t4 + 1] = acc[0][1] + acc[1][1];
            pw[(gq + 8) * kMaxRows + 2 * t4] = acc[0][2] + acc[1][2];
            pw[(gq + 8) * kMaxRows + 2 * t4 + 1] = acc[0][3] + acc[1][3];
            __syncwarp();
            if (lane == 0) mbar_arrive(&accfull[buf]);
            ++nt;
        }
    } else {
        // ---------------- epilogue warps: thread e takes channel e / 8, token row e % 8
        named_bar(0, kThreads);
        cluster_arrive();
        cluster_wait();
        const int e = tid - kMmaWarps * 32;
        const int ech = e >> 3, eb = e & 7;
        const bool epi = eb < B;
        uint32_t nt = 0, nw = 0, nsd = 0;
        for (int j = static_cast<int>(cid); j < a.ngroups; j += static_cast<int>(ncl)) {
            int s;
            const int row0 = tile_of(a, j, rank, s);
            const Seg& g = a.seg[s];
            const bool wide = g.l2 > kBs;
            if (row0 < 0) {
                // no tile here; a wide group still exchanges (zeros) so every CTA of
                // the cluster walks the same sequence of exchanges
                if (wide) exchange(a, xsum, xbar, rank, nw, e, 0.f, &abort_flag);
                continue;
            }
            const long hb = (static_cast<long>(eb) * g.C + row0 + ech) * 3;
            uint2 cw = make_uint2(0, 0);
            uint16_t hr0 = 0, hr1 = 0, hr2 = 0;
            if (g.conv_w) {                            // from the side ring
                const uint32_t sl = nsd % kSide;
                mbar_wait_or_abort(&sidefull[sl], (nsd / kSide) & 1u, a.err, &abort_flag);
                const uint8_t* sd = side + sl * kSideBytes;
                cw = *reinterpret_cast<const uint2*>(sd + ech * 8);
                if (g.conv_in && epi) {
                    const uint16_t* hs = reinterpret_cast<const uint16_t*>(sd + 128 + eb * 96) + ech * 3;
                    hr0 = hs[0];
                    hr1 = hs[1];
                    hr2 = hs[2];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sideempty[sl]);
                ++nsd;
            }
            const uint32_t buf = nt & 1u;
            mbar_wait_or_abort(&accfull[buf], (nt >> 1) & 1u, a.err, &abort_flag);
            float sum = 0.f;
            const float* pc = acc_s + (buf * kMmaWarps * kBs + ech) * kMaxRows + eb;
#pragma unroll
            for (int w = 0; w < kMmaWarps; ++w) sum += pc[w * kBs * kMaxRows];
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[buf]);
            float yv = 0.f;
            if (epi) {
                const float p = bf16r(sum);
                yv = p;
                if (g.conv_w) {
                    const float h0 = bf16_bits_to_f32(hr0), h1 = bf16_bits_to_f32(hr1), h2 = bf16_bits_to_f32(hr2);
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
                if (!g.l2) g.y[static_cast<long>(eb) * g.ldy + row0 + ech] = f32_to_bf16_bits(yv);
            }
            if (g.l2) {
                // per-group L2 norm (fp32, eps 1e-6), reference/fused_proj_conv_silu_ref.py:64-66;
                // the first barrier keeps a fast thread from overwriting values that a slow
                // one still reads for an earlier tile
                float* yb = ys + buf * kMaxRows * kBs;
                named_bar(2, kEpiWarps * 32);
                if (epi) yb[eb * kBs + ech] = yv;
                named_bar(2, kEpiWarps * 32);
                float ss = 0.f;
                if (!wide) {
                    if (epi) {
                        const float* yr = yb + eb * kBs + (ech / g.l2) * g.l2;
                        for (int i = 0; i < g.l2; ++i) ss = fmaf(yr[i], yr[i], ss);
                    }
                } else {
                    float part = 0.f;
                    if (e < B)
                        for (int i = 0; i < kBs; ++i) part = fmaf(yb[e * kBs + i], yb[e * kBs + i], part);
                    const float* slot = exchange(a, xsum, xbar, rank, nw, e, part, &abort_flag);
                    const int k = g.l2 / kBs;                           // CTAs of this L2 group
                    const int r0 = static_cast<int>(rank) / k * k;
                    if (epi)
                        for (int r = r0; r < r0 + k; ++r) ss += slot[r * kMaxRows + eb];
                }
                if (epi)
                    g.y[static_cast<long>(eb) * g.ldy + row0 + ech] = f32_to_bf16_bits(yv * (1.f / sqrtf(ss + 1e-6f)));
            }
            ++nt;
        }
    }
    cluster_arrive();                                  // no CTA leaves while a peer may still write to it
    cluster_wait();
}

struct ClusterFit {
    int dev, cl, smem, n;
};
std::mutex g_fit_mu;
std::vector<ClusterFit> g_fit;

}  // namespace
}  // namespace gdn

extern "C" int gdn_decode_proj_fwd(const void* x, const void* norm_gamma, float eps, int B, int D,
                                   const gdn_proj_segment* segs, int nseg, void* stream) {
    using namespace gdn;
    if (!x || !segs) return fail(GDN_ERR_NULL, "gdn_decode_proj_fwd: x and segs are required");
    // stage width: the widest multiple of 256 columns dividing D, at most 2048
    int KC = 256;
    for (int c = 256; c <= kMaxKC && c <= D; c += 256)
        if (D % c == 0) KC = c;
    const int fixed = B >= 1 && B <= kMaxRows ? fixed_smem_bytes(B, D) : 0;
    int nst = (kSmemBudget - fixed) / stage_smem_bytes(KC);
    nst = nst > kMaxStages ? kMaxStages : nst;
    if (B < 1 || B > kMaxRows || D < 256 || D % 256 != 0 || nst < 2)
        return fail(GDN_ERR_SHAPE,
                    "gdn_decode_proj_fwd: need 1 <= B <= %d, D %% 256 == 0 and B token rows of D plus two weight "
                    "stages within 226 KB of shared memory (got B=%d D=%d)",
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
    a.KC = KC;
    a.nst = nst;
    a.nseg = nseg;
    int cl = 1;
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
        if (!aligned16(s.W) || (s.conv_w && !aligned16(s.conv_w)) || (s.conv_state_in && !aligned16(s.conv_state_in)))
            return fail(GDN_ERR_ALIGN, "gdn_decode_proj_fwd: segment %d: W, conv_w and conv_state_in must be 16-byte aligned",
                        i);
        Seg& d = a.seg[i];
        d.W = static_cast<const uint16_t*>(s.W);
        d.y = static_cast<uint16_t*>(s.y);
        d.conv_w = static_cast<const uint16_t*>(s.conv_w);
        d.conv_in = static_cast<const uint16_t*>(s.conv_state_in);
        d.conv_out = static_cast<uint16_t*>(s.conv_state_out);
        d.C = s.C;
        d.ldy = s.ldy;
        d.l2 = s.l2_group;
        if (s.l2_group > kBs) cl = cl > s.l2_group / kBs ? cl : s.l2_group / kBs;
    }
    // groups of cl tiles; a wide L2 group (cl * 16 channels) is exactly one of them
    int ng = 0;
    for (int i = 0; i < nseg; ++i) {
        a.seg[i].first_group = ng;
        ng += (a.seg[i].C / kBs + cl - 1) / cl;
    }
    a.cl = cl;
    a.ngroups = ng;
    int st = check_sm100();
    if (st != GDN_OK) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: no current device");
    std::call_once(g_attr_once[dev], [dev] {
        g_attr_ok[dev] = cudaFuncSetAttribute(decode_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kSmemBudget) == cudaSuccess;
    });
    if (!g_attr_ok[dev]) return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: cannot grant shared memory");
    const int smem = fixed + nst * stage_smem_bytes(KC);
    a.err = device_error_word();

    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    a.pdl = launch_overlap() ? 1 : 0;
    cfg.numAttrs = a.pdl ? 2 : 1;
    // persistent grid: as many clusters as fit at once (cached per device, cluster size, shared memory)
    int fit = 0;
    {
        std::lock_guard<std::mutex> lk(g_fit_mu);
        for (const ClusterFit& f : g_fit)
            if (f.dev == dev && f.cl == cl && f.smem == smem) fit = f.n;
        if (fit == 0) {
            int sms = 0;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cfg.gridDim = dim3(cl * (sms / cl > 0 ? sms / cl : 1));
            if (cudaOccupancyMaxActiveClusters(&fit, decode_proj_kernel, &cfg) != cudaSuccess || fit < 1)
                return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: no cluster of %d CTAs fits", cl);
            g_fit.push_back({dev, cl, smem, fit});
        }
    }
    cfg.gridDim = dim3(cl * (ng < fit ? ng : fit));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_proj_kernel, a);
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_decode_proj_fwd: launch failed: %s", cudaGetErrorString(e));
    return launch_status("gdn_decode_proj_fwd");
}
