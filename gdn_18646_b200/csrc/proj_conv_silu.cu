// proj_conv_silu.cu -- fused input projection + causal depthwise conv1d (k=4) + SiLU
// (+ optional per-head L2 norm), on tcgen05 tensor cores.
//
// Math: reference/fused_proj_conv_silu_ref.py:33-67 with its bf16 rounding
// points (projection rounded to bf16, conv over bf16 values in fp32 rounded
// to bf16, SiLU rounded to bf16).  Replaces fused_proj_conv_silu_kernel
// (kernels/fused_proj_conv_silu.cu:105-295, WMMA + cp.async).
//
// The GEMM is computed TRANSPOSED: D[c, t] = sum_d W[c, d] x[t, d], with
// output channels on the TMEM lanes and 256 consecutive tokens on the TMEM
// columns (MMA N = 256).  Each epilogue thread therefore owns one channel
// across 256 tokens and the causal conv along tokens is a register-local
// sliding window.  A tile's GEMM rows start 3 tokens before its first output
// token (TMA zero-fills negative token coordinates, which is exactly the
// reference's causal zero padding), so each tile emits 253 tokens.
//
// The CTAs run in pairs (clusters of 2) issuing tcgen05 cta_group::2 MMAs of
// M = 256: each CTA loads its own 128 channel rows of W and HALF of the 256
// token rows of x, and the pair's MMA reads the other half from the peer's
// shared memory.  Per CTA that is 32 KB of operands per 64-deep k step instead
// of 48 KB for a one-CTA 128 x 256 tile, which is what bounded that version (its
// shared-memory fill plus the MMA reads exceeded the SM's shared-memory
// bandwidth).  No load is multicast.  The two channel tiles of a pair are
// independent (they may belong to different segments); with an odd number of
// channel tiles the last pair's second CTA repeats the last tile and stores
// nothing.
//
// Persistent, warp-specialised: warp 0 = TMA producer (W and x tiles, 128B
// swizzle, 5-stage ring, completion counted on the even CTA's barriers),
// warp 1 = MMA issuer (even CTA only; its commits arrive on both CTAs'
// barriers), warps 2-5 = epilogue (TMEM -> conv/SiLU/L2 -> smem -> TMA store;
// each CTA its own 128 channels).  Two TMEM accumulators (2 x 256 columns) let
// the epilogue of tile i overlap the MMAs of tile i+1.
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {
namespace {

constexpr int PM = 128;               // channels per tile (MMA M)
constexpr int PN = 256;               // token rows per tile (MMA N)
constexpr int POUT = PN - 3;          // output tokens per tile
constexpr int PK = 64;                // K per stage (one 128-byte swizzle atom of bf16)
constexpr int PSTAGES = 5;
constexpr int PNH = PN / 2;           // token rows of x each CTA of the pair loads
constexpr int A_BYTES = PM * PK * 2;  // 16 KB
constexpr int B_BYTES = PNH * PK * 2; // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int Y_SUB_BYTES = PN * 128; // one 64-channel output sub-tile: 256 rows x 128 B
constexpr int OFF_Y = PSTAGES * STAGE_BYTES;
constexpr int OFF_BAR = OFF_Y + 2 * Y_SUB_BYTES;
constexpr int PROJ_SMEM = OFF_BAR + 128 + 1024;
static_assert(PROJ_SMEM <= 232448, "proj shared memory exceeds 227 KB");
constexpr int kProjThreads = 192;     // 6 warps

constexpr int kProjMaxSeg = 6;

// One output-channel segment of a launch: its own weights, conv and output tensors.
struct ProjSeg {
    const uint16_t* conv_w;      // [Dout, 4], or null: plain projection y = bf16(x . W[c])
    const uint16_t* state_in;    // [B, Dout, 3] or null
    uint16_t* state_out;         // [B, Dout, 3] or null
    int Dout;
    int ct0;                     // first channel tile of the segment in the launch
    int l2;                      // 0 or group size
};

struct ProjArgs {
    unsigned int* err;
    int B, T, D;
    int n_ct, n_tt, ntiles;      // n_ct: channel tiles over all segments; ntiles: pair tiles
    int nseg;
    ProjSeg seg[kProjMaxSeg];
};

struct alignas(64) ProjMaps {
    CUtensorMap w[kProjMaxSeg];
    CUtensorMap y[kProjMaxSeg];
};

__device__ __forceinline__ int proj_seg_of(const ProjArgs& a, int ct) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kProjMaxSeg; ++i)
        if (i < a.nseg && ct >= a.seg[i].ct0) s = i;
    return s;
}

__device__ __forceinline__ float bf16r(float x) { return __uint_as_float(static_cast<uint32_t>(f32_to_bf16_bits(x)) << 16); }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kProjThreads, 1)
proj_conv_silu_kernel(const __grid_constant__ ProjMaps maps, const __grid_constant__ CUtensorMap map_x,
                      const __grid_constant__ ProjArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + OFF_BAR);   // [PSTAGES]
    uint64_t* empty = full + PSTAGES;                               // [PSTAGES]
    uint64_t* acc_full = empty + PSTAGES;                           // [2]
    uint64_t* acc_empty = acc_full + 2;                             // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* ysm = sm + OFF_Y;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int nk = args.D / PK;
    const uint32_t rank = cluster_ctarank();        // 0: the pair's MMA issuer
    const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
    const int n_cp = (args.n_ct + 1) >> 1;          // channel-tile pairs
    // this CTA's channel tile of pair tile `pt` (the last tile again when n_ct is odd: not stored)
    auto my_ct = [&](int pt, bool& valid) {
        const int ct = 2 * (pt % n_cp) + static_cast<int>(rank);
        valid = ct < args.n_ct;
        return valid ? ct : args.n_ct - 1;
    };

    if (tid == 0) {
        for (int s = 0; s < PSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], 8);            // even CTA's: 4 epilogue warps of each CTA
        }
        *abort_flag = 0;
        fence_mbar_init();
        for (int i = 0; i < args.nseg; ++i) {
            tma_prefetch_desc(&maps.w[i]);
            tma_prefetch_desc(&maps.y[i]);
        }
        tma_prefetch_desc(&map_x);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();                                 // both CTAs' barriers initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = pair; tile < args.ntiles; tile += npairs) {
                bool valid;
                const int ct = my_ct(tile, valid);
                const int rest = tile / n_cp;
                const int tt = rest % args.n_tt;
                const int b = rest / args.n_tt;
                const int ts = tt * POUT - 3;
                const int sg = proj_seg_of(args, ct);
                const CUtensorMap* mw = &maps.w[sg];
                const int lct = ct - args.seg[sg].ct0;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait_or_abort(&empty[stage], phase ^ 1u, args.err, abort_flag)) break;
                    uint8_t* st = sm + stage * STAGE_BYTES;
                    // both CTAs' bytes complete on the even CTA's barrier, which expects them all
                    const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
                    tma_load_2d_pair(st, mw, fb, kb * PK, lct * PM);
                    tma_load_3d_pair(st + A_BYTES, &map_x, fb, kb * PK, ts + static_cast<int>(rank) * PNH, b);
                    if (++stage == PSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (*abort_flag) break;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (the pair's even CTA)
        if (lane == 0 && rank == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            constexpr uint32_t idesc = idesc_bf16(2 * PM, PN, false, false);
            for (int tile = pair; tile < args.ntiles; tile += npairs, ++local) {
                const int abuf = local & 1;
                const uint32_t aphase = static_cast<uint32_t>(local >> 1) & 1u;
                if (!mbar_wait_or_abort(&acc_empty[abuf], aphase ^ 1u, args.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + abuf * PN;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait_or_abort(&full[stage], phase, args.err, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(sm + stage * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < PK / 16; ++k)
                        umma_bf16_ss_pair(d_tmem, sdesc_sw128(sa + k * 32, 16, 1024),
                                          sdesc_sw128(sb + k * 32, 16, 1024), idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    umma_commit_pair(&empty[stage]);
                    if (++stage == PSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (*abort_flag) break;
                umma_commit_pair(&acc_full[abuf]);
            }
        }
    } else {
        // ---------------- epilogue: 4 warps, TMEM lanes 32*(warp%4) .. +31
        const int quad = warp & 3;
        const int cl = quad * 32 + lane;            // channel within the tile (= TMEM lane)
        const int et = tid - 64;                    // 0..127
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        int local = 0;
        const uint32_t acc_empty_even[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0),
                                            mapa_shared(smem_u32(&acc_empty[1]), 0)};
        for (int tile = pair; tile < args.ntiles; tile += npairs, ++local) {
            bool valid;
            const int ct = my_ct(tile, valid);
            const int rest = tile / n_cp;
            const int tt = rest % args.n_tt;
            const int b = rest / args.n_tt;
            const int t0 = tt * POUT;
            const int ts = t0 - 3;
            const int sg = proj_seg_of(args, ct);
            const ProjSeg& S = args.seg[sg];
            const int lct = ct - S.ct0;
            const int c = lct * PM + cl;                // channel within the segment
            const int abuf = local & 1;
            const uint32_t aphase = static_cast<uint32_t>(local >> 1) & 1u;

            // previous tile's TMA store must have finished reading the staging buffer
            if (et == 0) bulk_wait_read0();
            named_bar(1, 128);

            const bool conv = S.conv_w != nullptr;
            float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f;
            if (conv) {
                const uint2 wraw = *reinterpret_cast<const uint2*>(S.conv_w + static_cast<long>(c) * 4);
                w0 = bf16_bits_to_f32(wraw.x & 0xffffu);
                w1 = bf16_bits_to_f32(wraw.x >> 16);
                w2 = bf16_bits_to_f32(wraw.y & 0xffffu);
                w3 = bf16_bits_to_f32(wraw.y >> 16);
            }
            const long sbase = (static_cast<long>(b) * S.Dout + c) * 3;

            const bool ok = mbar_wait_or_abort(&acc_full[abuf], aphase, args.err, abort_flag);
            tc_fence_after();
            float p1 = 0.f, p2 = 0.f, p3 = 0.f;     // projections of tokens i-3, i-2, i-1
            uint8_t* ysub = ysm + (cl >> 6) * Y_SUB_BYTES;
            const uint32_t ccol = cl & 63;
            // tiles that touch the conv history (first tile with state_in, last tile with state_out)
            const bool special = conv && ((tt == 0 && S.state_in) || (S.state_out && ts + PN > args.T - 3));
            uint16_t* const state_out = valid ? S.state_out : nullptr;    // a repeated tile writes nothing
#pragma unroll 1
            for (int blk = 0; blk < PN / 32; ++blk) {
                float acc[32];
                tmem_ld32(tmem + lane_off + abuf * PN + blk * 32, acc);
                tmem_ld_wait();
                if (!conv) {                               // plain projection: y = bf16(x . W[c])
#pragma unroll
                    for (int u = 0; u < 32; ++u) {
                        const int i = blk * 32 + u;
                        if (i >= 3)
                            *reinterpret_cast<uint16_t*>(ysub + sw128_off(i - 3, ccol)) = f32_to_bf16_bits(acc[u]);
                    }
                } else if (!special) {
#pragma unroll
                    for (int u = 0; u < 32; ++u) {
                        const int i = blk * 32 + u;
                        const float p = bf16r(acc[u]);
                        if (i >= 3) {
                            float conv = p1 * w0;
                            conv = fmaf(p2, w1, conv);
                            conv = fmaf(p3, w2, conv);
                            conv = fmaf(p, w3, conv);
                            const float cr = bf16r(conv);
                            const float y = __fdividef(cr, 1.f + __expf(-cr));   // SiLU
                            *reinterpret_cast<uint16_t*>(ysub + sw128_off(i - 3, ccol)) = f32_to_bf16_bits(y);
                        }
                        p1 = p2;
                        p2 = p3;
                        p3 = p;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 32; ++u) {
                        const int i = blk * 32 + u;
                        const int tok = ts + i;
                        float p = bf16r(acc[u]);
                        if (tok < 0) p = S.state_in ? bf16_bits_to_f32(S.state_in[sbase + (tok + 3)]) : 0.f;
                        if (state_out && tok < args.T && tok >= args.T - 3 && (i >= 3 || tt == 0))
                            state_out[sbase + (tok - (args.T - 3))] = f32_to_bf16_bits(p);
                        if (i >= 3) {
                            float conv = p1 * w0;
                            conv = fmaf(p2, w1, conv);
                            conv = fmaf(p3, w2, conv);
                            conv = fmaf(p, w3, conv);
                            const float cr = bf16r(conv);
                            const float y = __fdividef(cr, 1.f + __expf(-cr));   // SiLU
                            *reinterpret_cast<uint16_t*>(ysub + sw128_off(i - 3, ccol)) = f32_to_bf16_bits(y);
                        }
                        p1 = p2;
                        p2 = p3;
                        p3 = p;
                    }
                }
            }
            // accumulator buffer free for the MMA warp (on the even CTA's barrier)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty_even[abuf]);

            if (S.l2) {
                // per token row: the 128 channels as 16 chunks of 8 (16-byte shared-memory
                // accesses, conflict-free per quarter warp under the 128-byte swizzle), the
                // sum of squares per group of args.l2 channels, then every value scaled
                named_bar(1, 128);
                const int cpg = S.l2 >> 3;                     // chunks per group
                for (int r = et; r < POUT; r += 128) {
                    uint4 cw[16];
#pragma unroll
                    for (int c16 = 0; c16 < 16; ++c16)
                        cw[c16] = *reinterpret_cast<const uint4*>(ysm + (c16 >> 3) * Y_SUB_BYTES + sw128_chunk(r, c16 & 7));
                    float t[16];                                   // chunk sums of squares
#pragma unroll
                    for (int c16 = 0; c16 < 16; ++c16) {
                        const uint32_t u[4] = {cw[c16].x, cw[c16].y, cw[c16].z, cw[c16].w};
                        float ss = 0.f;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float f0 = __uint_as_float(u[i] << 16), f1 = __uint_as_float(u[i] & 0xffff0000u);
                            ss = fmaf(f0, f0, ss);
                            ss = fmaf(f1, f1, ss);
                        }
                        t[c16] = ss;
                    }
                    // group sums over aligned blocks of cpg chunks (cpg a power of two)
#pragma unroll
                    for (int w = 1; w < 16; w <<= 1) {
                        if (w < cpg) {
                            float n[16];
#pragma unroll
                            for (int c = 0; c < 16; ++c) n[c] = t[c] + t[c ^ w];
#pragma unroll
                            for (int c = 0; c < 16; ++c) t[c] = n[c];
                        }
                    }
                    float inv[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) inv[c] = 1.f / sqrtf(t[c] + 1e-6f);
#pragma unroll
                    for (int c16 = 0; c16 < 16; ++c16) {
                        const uint32_t u[4] = {cw[c16].x, cw[c16].y, cw[c16].z, cw[c16].w};
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            o[i] = (static_cast<uint32_t>(f32_to_bf16_bits(__uint_as_float(u[i] & 0xffff0000u) * inv[c16])) << 16) |
                                   f32_to_bf16_bits(__uint_as_float(u[i] << 16) * inv[c16]);
                        *reinterpret_cast<uint4*>(ysm + (c16 >> 3) * Y_SUB_BYTES + sw128_chunk(r, c16 & 7)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
            }
            fence_async_smem();
            named_bar(1, 128);
            if (et == 0 && ok && valid && !*abort_flag) {
                tma_store_3d(&maps.y[sg], ysm, lct * PM, t0, b);
                tma_store_3d(&maps.y[sg], ysm + Y_SUB_BYTES, lct * PM + 64, t0, b);
                bulk_commit();
            }
        }
        if (et == 0) bulk_wait_all0();
    }

    tc_fence_before();
    cluster_sync();                                 // the pair's MMAs and both epilogues are done with TMEM
    if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

std::once_flag g_proj_attr_once[64];
int g_proj_attr_status[64];
int g_sm_count[64];

}  // namespace

int check_proj_args(const void* x, const void* W, const void* conv_w, void* y, int B, int T, int D, int Dout,
                    const void* csi, const void* cso, int l2) {
    if (!x || !W || !conv_w || !y) return fail(GDN_ERR_NULL, "gdn_proj_conv_silu_fwd: x, W, conv_w and y are required");
    if (B <= 0 || T <= 0 || D <= 0 || Dout <= 0 || D % 64 != 0 || Dout % 128 != 0)
        return fail(GDN_ERR_SHAPE,
                    "gdn_proj_conv_silu_fwd: need B, T > 0, D %% 64 == 0 and Dout %% 128 == 0 (got B=%d T=%d D=%d Dout=%d)",
                    B, T, D, Dout);
    if (l2 != 0 && (l2 < 8 || l2 > 128 || Dout % l2 != 0 || 128 % l2 != 0))
        return fail(GDN_ERR_SHAPE, "gdn_proj_conv_silu_fwd: l2norm_group %d must divide 128 and Dout", l2);
    if (!aligned16(x) || !aligned16(W) || !aligned16(y) || (reinterpret_cast<uintptr_t>(conv_w) & 7u) ||
        (csi && (reinterpret_cast<uintptr_t>(csi) & 1u)) || (cso && (reinterpret_cast<uintptr_t>(cso) & 1u)))
        return fail(GDN_ERR_ALIGN, "gdn_proj_conv_silu_fwd: x, W, y must be 16-byte and conv_w 8-byte aligned");
    return GDN_OK;
}

}  // namespace gdn

namespace gdn {
namespace {
int run_proj(const void* x, int B, int T, int D, const gdn_proj_out_seg* segs, int nseg, void* stream) {
    int st = check_sm100();
    if (st != GDN_OK) return st;
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(g_proj_attr_once[dev & 63], [dev]() {
        g_proj_attr_status[dev & 63] =
            cudaFuncSetAttribute(proj_conv_silu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PROJ_SMEM) ==
                    cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_sm_count[dev & 63] = sms > 0 ? sms : 148;
    });
    if (g_proj_attr_status[dev & 63] != GDN_OK)
        return fail(GDN_ERR_CUDA, "gdn_proj_conv_silu_fwd: cannot grant %d B of shared memory", PROJ_SMEM);

    ProjMaps maps;
    memset(&maps, 0, sizeof(maps));
    CUtensorMap mx;
    {
        uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
        uint64_t strides[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(D) * 2 * T};
        uint32_t box[3] = {PK, PNH, 1};
        if ((st = make_map_bf16(&mx, x, 3, dims, strides, box, true)) != GDN_OK) return st;
    }
    ProjArgs a;
    memset(&a, 0, sizeof(a));
    a.err = device_error_word();
    a.B = B;
    a.T = T;
    a.D = D;
    a.nseg = nseg;
    int ct = 0;
    for (int i = 0; i < nseg; ++i) {
        const gdn_proj_out_seg& g = segs[i];
        {
            uint64_t dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(g.Dout)};
            uint64_t strides[1] = {static_cast<uint64_t>(D) * 2};
            uint32_t box[2] = {PK, PM};
            if ((st = make_map_bf16(&maps.w[i], g.W, 2, dims, strides, box, true)) != GDN_OK) return st;
        }
        {
            uint64_t dims[3] = {static_cast<uint64_t>(g.Dout), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
            uint64_t strides[2] = {static_cast<uint64_t>(g.Dout) * 2, static_cast<uint64_t>(g.Dout) * 2 * T};
            uint32_t box[3] = {64, POUT, 1};
            if ((st = make_map_bf16(&maps.y[i], g.y, 3, dims, strides, box, true)) != GDN_OK) return st;
        }
        a.seg[i].conv_w = static_cast<const uint16_t*>(g.conv_w);
        a.seg[i].state_in = g.conv_w ? static_cast<const uint16_t*>(g.conv_state_in) : nullptr;
        a.seg[i].state_out = g.conv_w ? static_cast<uint16_t*>(g.conv_state_out) : nullptr;
        a.seg[i].Dout = g.Dout;
        a.seg[i].ct0 = ct;
        a.seg[i].l2 = g.l2norm_group;
        ct += g.Dout / PM;
    }
    a.n_ct = ct;
    a.n_tt = (T + POUT - 1) / POUT;
    const long ntiles = static_cast<long>((a.n_ct + 1) / 2) * a.n_tt * B;    // pair tiles (256 channels)
    if (ntiles > 0x7fffffffL) return fail(GDN_ERR_SHAPE, "gdn_proj_conv_silu_fwd: too many tiles");
    a.ntiles = static_cast<int>(ntiles);
    const long pairs = g_sm_count[dev & 63] / 2;
    const int grid = 2 * static_cast<int>(ntiles < pairs ? ntiles : pairs);
    proj_conv_silu_kernel<<<grid, kProjThreads, PROJ_SMEM, static_cast<cudaStream_t>(stream)>>>(maps, mx, a);
    return launch_status("gdn_proj_conv_silu_fwd");
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_proj_conv_silu_fwd(const void* x, const void* W, const void* conv_w, void* y, int B, int T,
                                      int D, int Dout, const void* conv_state_in, void* conv_state_out,
                                      int l2norm_group, void* stream) {
    using namespace gdn;
    const int st = check_proj_args(x, W, conv_w, y, B, T, D, Dout, conv_state_in, conv_state_out, l2norm_group);
    if (st != GDN_OK) return st;
    gdn_proj_out_seg seg;
    seg.W = W;
    seg.y = y;
    seg.conv_w = conv_w;
    seg.conv_state_in = conv_state_in;
    seg.conv_state_out = conv_state_out;
    seg.Dout = Dout;
    seg.l2norm_group = l2norm_group;
    return run_proj(x, B, T, D, &seg, 1, stream);
}

extern "C" int gdn_proj_multi_fwd(const void* x, int B, int T, int D, const gdn_proj_out_seg* segs, int nseg,
                                  void* stream) {
    using namespace gdn;
    if (!x || !segs) return fail(GDN_ERR_NULL, "gdn_proj_multi_fwd: x and segs are required");
    if (nseg < 1 || nseg > kProjMaxSeg)
        return fail(GDN_ERR_SHAPE, "gdn_proj_multi_fwd: 1 to %d segments (got %d)", kProjMaxSeg, nseg);
    for (int i = 0; i < nseg; ++i) {
        const gdn_proj_out_seg& g = segs[i];
        if (!g.W || !g.y) return fail(GDN_ERR_NULL, "gdn_proj_multi_fwd: segment %d needs W and y", i);
        // the shared checks, with conv_w standing in for plain segments
        const int st = check_proj_args(x, g.W, g.conv_w ? g.conv_w : g.W, g.y, B, T, D, g.Dout,
                                       g.conv_state_in, g.conv_state_out, g.l2norm_group);
        if (st != GDN_OK) return st;
    }
    return run_proj(x, B, T, D, segs, nseg, stream);
}
