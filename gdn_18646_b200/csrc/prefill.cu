// prefill.cu -- chunked gated-delta-rule prefill on tcgen05 tensor cores.
//
// Math: reference/prefill_ref.py:11-132 (chunk C = 64, WY / UT form).  Replaces
// the reference's gdn_prefill_v2_kernel (kernels/prefill_chunked.cu:41-417),
// which runs fp32 CUDA-core loops with one thread per value column and
// hard-codes H=16, K=128, V=256.
//
// One CTA per (batch, value head, 128-wide value tile).  Per 64-token chunk,
// with Lambda the in-chunk cumulative log decay, beta' = beta * mask,
//   N[t,s] = -beta'_t (k_t . k_s) exp(Lambda_t - Lambda_s)  (t > s)
//   A      = (I - N)^-1                                      (prefill_ref.py:96-101)
//   U      = A diag(beta') V,  W = A diag(beta' e^Lambda) K  (prefill_ref.py:103-104)
//   dV     = U - W S                                         (:117-118)
//   O      = diag(m) [ scale diag(e^Lambda) Q S + P dV ],
//            P[t,s] = scale (q_t.k_s) exp(Lambda_t - Lambda_s), s <= t   (:120-122)
//   S     <- e^{Lambda_last} S + K^T diag(e^{Lambda_last - Lambda}) dV   (:124-126)
//
// The state is held TRANSPOSED in TMEM (S^T: value index = TMEM lane), so the
// value tile is the M = 128 dimension of every state-path product.
//
// Warp roles (288 threads):
//   warp 0      TMA producer: q/k chunk tiles (2-slot ring) and v tiles.
//   warps 1-4   PREP warpgroup, one chunk ahead of the chain: gates and the
//               in-chunk cumulative decay; [Q;K] K^T on tensor cores; P and N
//               (TMEM -> registers); the 64x64 unit-lower-triangular inverse
//               (16x16 diagonal blocks by substitution in registers, the
//               off-diagonal blocks with warp-level bf16 MMAs on hi/lo-split
//               operands); U^T = V^T (A diag beta')^T and
//               W^T = K^T (A diag(beta' e^Lambda))^T on tensor cores; W^T to
//               shared memory as a bf16 hi/lo pair.
//   warps 5-8   CHAIN warpgroup, the sequential state recurrence:
//               S^T -> bf16 hi/lo; dV^T = U^T - S^T W^T accumulated straight into
//               U^T's TMEM (negated B operand) and (Q S)^T; then
//               S^T = e^{Lambda_last} S^T + dV'^T K and (P dV)^T.  W^T is
//               split to shared memory by the chain (prep never waits on its
//               U/W MMA), and chunk c's output tile is staged in shared memory
//               and TMA-stored at the top of chunk c+1, while prep still runs.
// Each warpgroup issues its own tcgen05.mma from one elected thread and
// tracks completion with tcgen05.commit -> mbarrier.  fp32 values feeding the
// state path (S, W, A diag beta', A diag beta' e^Lambda, dV') are split into
// bf16 hi + lo pairs (~16 mantissa bits per product); q/k/v are exact bf16
// inputs; the output path (Q S_hi, P dV) uses single bf16.
// Decay ratios exp(Lambda_t - Lambda_s) are formed as u_t * w_s with
// u_t = 2^(l_t - m), w_s = 2^(m - l_s) around the chunk's mid decay m (never
// gamma_t / gamma_s); chunks whose total decay could overflow that product
// fall back to one exp2 per element.  Every mbarrier wait is bounded; a
// timeout raises a CTA-wide abort and all roles drain through their barriers.
#include <mutex>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {
namespace {

constexpr int kC = 64;                 // chunk length
constexpr int kThreads = 288;          // 9 warps
constexpr int kTmemCols = 512;

// TMEM column map (fp32, 128 lanes)
constexpr uint32_t COL_QKK = 0;        // prep: [Q;K] K^T (lanes 0-63 QK^T, 64-127 KK^T)
constexpr uint32_t COL_UT = 64;        // 2 x 64: U^T for chunk parity 0/1, becomes dV^T in place
constexpr uint32_t COL_QS = 192;       // (Q S_hi)^T
constexpr uint32_t COL_PDV = 256;      // (P dV)^T
constexpr uint32_t COL_ST = 320;       // S^T (fp32 state, dk columns)
constexpr uint32_t COL_WT = 448;       // W^T (lanes = key index d)

// named barriers
constexpr int BAR_PREP = 1, BAR_CHAIN = 2;

template <int DK>
struct PrefillSmem {
    static constexpr int CB = DK / 64;                    // 64-wide column blocks of q/k
    static constexpr int QK_BYTES = CB * 16384;           // slot: per block [Q 64 rows | K 64 rows] x 128 B
    static constexpr int V_BYTES = 2 * 8192;              // 2 blocks of 64 rows x 128 B
    static constexpr int SR_BYTES = (2 * CB * 16384 > 49152) ? 2 * CB * 16384 : 49152;
    static constexpr int OFF_QK0 = 0;
    static constexpr int OFF_QK1 = OFF_QK0 + QK_BYTES;
    static constexpr int OFF_V = OFF_QK1 + QK_BYTES;
    static constexpr int OFF_SR = OFF_V + V_BYTES;        // chain: S hi|lo; dV' hi|lo|dV bf16; o staging
    static constexpr int S_LO = CB * 16384;
    static constexpr int DVH = 0, DVL = 16384, DVB = 32768, OST = 0;
    static constexpr int OFF_X = OFF_SR + SR_BYTES;       // prep A1 hi/lo, A2 hi/lo; then W^T hi/lo
    static constexpr int X_A1H = 0, X_A1L = 8192, X_A2H = 16384, X_A2L = 24576;
    static constexpr int X_WTH = 0, X_WTL = 16384;
    static constexpr int OFF_P = OFF_X + 32768;           // P [2] x 8 KB
    static constexpr int NLD = 68;                        // fp32 row stride of N (16 B aligned rows)
    static constexpr int OFF_N = OFF_P + 16384;           // N; diagonal blocks replaced by D_i
    static constexpr int AOLD = 20;                       // fp32 row stride of 16x16 scratch blocks
    static constexpr int OFF_AO = OFF_N + 64 * NLD * 4;   // 6 off-diagonal blocks of A
    static constexpr int OFF_XS = OFF_AO + 6 * 16 * AOLD * 4;   // 3 per-warp 16x16 scratch blocks
    static constexpr int GSTRIDE = 9 * 64;                      // gate floats per parity slot
    static constexpr int OFF_G = OFF_XS + 3 * 16 * AOLD * 4;    // gates [2] x 9 x 64 floats
    static constexpr int OFF_OC = OFF_G + 2 * GSTRIDE * 4;      // chain copy of G_OC [2] x 64
    static constexpr int OFF_BAR = OFF_OC + 2 * 64 * 4;
    static constexpr int BYTES = OFF_BAR + 256;
    static constexpr int ALLOC = BYTES + 1024;
    static_assert(ALLOC <= 232448, "prefill shared memory exceeds 227 KB");
};

// per-chunk gate vectors (floats), 9 x 64 per parity slot
enum {
    G_LAM2 = 0,   // Lambda_t * log2(e)
    G_U = 1,      // 2^(l_t - m)
    G_W = 2,      // 2^(m - l_t)
    G_EDEC = 3,   // exp(Lambda_last - Lambda_t)
    G_BM = 4,     // beta_t * mask_t
    G_BME = 5,    // beta_t * mask_t * exp(Lambda_t)
    G_OC = 6,     // mask_t * scale * exp(Lambda_t)   (output coefficient of Q S)
    G_MK = 7,     // mask_t (0 for padding)
    G_TOT = 8     // [0,1] per-warp scan totals, [2] gamma_c, [3] direct-exp fallback flag
};

struct PrefillArgs {
    const void* a;
    const void* b;
    int gate_dtype;
    const float* A_log;
    float dt_bias;
    const float* dt_bias_vec;
    const float* mask;
    const float* state_in;
    float* state_out;
    unsigned int* err;
    int B, T, Hqk, Hv, dv, ntiles, layout;
    float scale;
};

struct Bars {
    uint64_t qk_full[2], qk_free[2], v_full, v_free;
    uint64_t qkk_done, uw_done, prep_done[2], chain_done[2];
    uint64_t ws_done, st_done, wt_read;
};

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    float a[32], b[32];
    tmem_ld32(taddr, a);
    tmem_ld32(taddr + 32, b);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        v[i] = a[i];
        v[32 + i] = b[i];
    }
}

// 8 fp32 -> one 16-byte chunk of hi and of lo bf16
__device__ __forceinline__ void split8(const float* v, uint4& h, uint4& l) {
    split2_bf16(v[0], v[1], h.x, l.x);
    split2_bf16(v[2], v[3], h.y, l.y);
    split2_bf16(v[4], v[5], h.z, l.z);
    split2_bf16(v[6], v[7], h.w, l.w);
}
__device__ __forceinline__ uint4 pack8(const float* v) {
    return make_uint4(cvt_bf16x2(v[0], v[1]), cvt_bf16x2(v[2], v[3]), cvt_bf16x2(v[4], v[5]),
                      cvt_bf16x2(v[6], v[7]));
}
// 64 fp32 -> one 128-byte row of a 128B-swizzled tile, bf16 hi and lo parts
__device__ __forceinline__ void store_row_split(uint8_t* hi_tile, uint8_t* lo_tile, int row, const float (&v)[64]) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
        uint4 h, l;
        split8(&v[8 * ch], h, l);
        const uint32_t off = sw128_chunk(row, ch);
        *reinterpret_cast<uint4*>(hi_tile + off) = h;
        *reinterpret_cast<uint4*>(lo_tile + off) = l;
    }
}

// ---------------------------------------------------------------------------
// 16x16 block product on one warp: acc (two 16x8 halves, C fragments) +=
// L (16x16 fp32, row stride ldl) * R (16x16 fp32, row stride ldr), with both
// operands split into bf16 hi + lo (3 MMAs per half: hi*hi + hi*lo + lo*hi).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void blk_mma_acc(float (&acc)[2][4], const float* L, int ldl, const float* R, int ldr,
                                            int lane) {
    const int g = lane >> 2, t4 = lane & 3;
    uint32_t ah[4], al[4];
    {
        const float2 v00 = *reinterpret_cast<const float2*>(L + g * ldl + 2 * t4);
        const float2 v10 = *reinterpret_cast<const float2*>(L + (g + 8) * ldl + 2 * t4);
        const float2 v01 = *reinterpret_cast<const float2*>(L + g * ldl + 2 * t4 + 8);
        const float2 v11 = *reinterpret_cast<const float2*>(L + (g + 8) * ldl + 2 * t4 + 8);
        split2_bf16(v00.x, v00.y, ah[0], al[0]);
        split2_bf16(v10.x, v10.y, ah[1], al[1]);
        split2_bf16(v01.x, v01.y, ah[2], al[2]);
        split2_bf16(v11.x, v11.y, ah[3], al[3]);
    }
#pragma unroll
    for (int hn = 0; hn < 2; ++hn) {
        const int n = 8 * hn + g;
        uint32_t bh0, bl0, bh1, bl1;
        split2_bf16(R[(2 * t4) * ldr + n], R[(2 * t4 + 1) * ldr + n], bh0, bl0);
        split2_bf16(R[(2 * t4 + 8) * ldr + n], R[(2 * t4 + 9) * ldr + n], bh1, bl1);
        mma_bf16_16816(acc[hn], ah, bh0, bh1);
        mma_bf16_16816(acc[hn], ah, bl0, bl1);
        mma_bf16_16816(acc[hn], al, bh0, bh1);
    }
}
__device__ __forceinline__ void blk_store(float* dst, int ld, const float (&acc)[2][4], int lane) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int hn = 0; hn < 2; ++hn) {
        *reinterpret_cast<float2*>(dst + g * ld + 8 * hn + 2 * t4) = make_float2(acc[hn][0], acc[hn][1]);
        *reinterpret_cast<float2*>(dst + (g + 8) * ld + 8 * hn + 2 * t4) = make_float2(acc[hn][2], acc[hn][3]);
    }
}

// slot of off-diagonal block (i, j), i > j, in the A scratch
__device__ __forceinline__ int ao_slot(int i, int j) {
    return (i - j == 1) ? j : (i - j == 2 ? 3 + j : 5);
}
__device__ __forceinline__ void blk_load(float (&acc)[2][4], const float* src, int ld, int lane) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int hn = 0; hn < 2; ++hn) {
        const float2 a = *reinterpret_cast<const float2*>(src + g * ld + 8 * hn + 2 * t4);
        const float2 b = *reinterpret_cast<const float2*>(src + (g + 8) * ld + 8 * hn + 2 * t4);
        acc[hn][0] = a.x;
        acc[hn][1] = a.y;
        acc[hn][2] = b.x;
        acc[hn][3] = b.y;
    }
}

// ---------------------------------------------------------------------------
// A = (I - N)^-1 for the 64x64 strictly-lower N held in Nsm (row stride NLD),
// by the 128 prep threads (4 warps):
//   1. warp w inverts the 16x16 diagonal block w by forward substitution in
//      registers (row i of the block becomes final at step i and is broadcast
//      by shuffles); D_w overwrites the diagonal block of Nsm;
//   2. off-diagonal blocks, A_ij = D_i sum_{k=j}^{i-1} N_ik A_kj (A_jj = D_j),
//      as warp-level MMAs on 16x16 blocks, with the D-only terms issued first:
//        a) Y_{i,i-1} = N_{i,i-1} D_{i-1};  Z20 = N20 D0, Z31 = N31 D1, Z30 = N30 D0
//        b) A_{i,i-1} = D_i Y_{i,i-1}
//        c) A20 = D2 (Z20 + N21 A10);  A31 = D3 (Z31 + N32 A21);  W30 = Z30 + N31 A10
//        d) A30 = D3 (W30 + N32 A20)
// ---------------------------------------------------------------------------
template <int NLD, int AOLD>
__device__ __forceinline__ void invert_unit_lower(float* Nsm, float* Ao, float* Xs, int pw, int lane) {
    {
        const int r = lane >> 1, hf = lane & 1;
        const int row0 = 16 * pw;
        float n[16], x[8];
        const float4* nr = reinterpret_cast<const float4*>(Nsm + (row0 + r) * NLD + row0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 t4 = nr[q];
            n[4 * q] = t4.x; n[4 * q + 1] = t4.y; n[4 * q + 2] = t4.z; n[4 * q + 3] = t4.w;
        }
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) x[cc] = (8 * hf + cc == r) ? 1.f : 0.f;
#pragma unroll
        for (int i = 0; i < 15; ++i) {
            float bi[8];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) bi[cc] = __shfl_sync(0xffffffffu, x[cc], 2 * i + hf);
            if (r > i) {
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) x[cc] = fmaf(n[i], bi[cc], x[cc]);
            }
        }
        __syncwarp();
        float4* dst = reinterpret_cast<float4*>(Nsm + (row0 + r) * NLD + row0 + 8 * hf);
        dst[0] = make_float4(x[0], x[1], x[2], x[3]);
        dst[1] = make_float4(x[4], x[5], x[6], x[7]);
    }
    named_bar(BAR_PREP, 128);
    auto Nb = [&](int i, int j) { return Nsm + (16 * i) * NLD + 16 * j; };   // N_ij (i > j) or D_i (i == j)
    auto Ab = [&](int i, int j) { return Ao + ao_slot(i, j) * 16 * AOLD; };
    float* xs = Xs + (pw < 3 ? pw : 0) * 16 * AOLD;
    // a) Y_{pw+1,pw} -> xs;  Z -> final slot of its block
    if (pw < 3) {
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        blk_mma_acc(acc, Nb(pw + 1, pw), NLD, Nb(pw, pw), NLD, lane);
        blk_store(xs, AOLD, acc, lane);
        const int zi = (pw == 2) ? 3 : pw + 2, zj = (pw == 2) ? 0 : pw;
        float acz[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        blk_mma_acc(acz, Nb(zi, zj), NLD, Nb(zj, zj), NLD, lane);
        blk_store(Ab(zi, zj), AOLD, acz, lane);
    }
    __syncwarp();
    // b) A_{pw+1,pw} = D_{pw+1} Y
    if (pw < 3) {
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        blk_mma_acc(acc, Nb(pw + 1, pw + 1), NLD, xs, AOLD, lane);
        blk_store(Ab(pw + 1, pw), AOLD, acc, lane);
    }
    named_bar(BAR_PREP, 128);
    // c) warp 0: A20, warp 1: A31, warp 2: W30 (partial sum of A30's X)
    if (pw < 3) {
        const int i = (pw == 2) ? 3 : pw + 2, j = (pw == 2) ? 0 : pw, k = (pw == 2) ? 1 : pw + 1;
        float acc[2][4];
        blk_load(acc, Ab(i, j), AOLD, lane);
        blk_mma_acc(acc, Nb(i, k), NLD, Ab(k, j), AOLD, lane);
        if (pw < 2) {
            blk_store(xs, AOLD, acc, lane);
            __syncwarp();
            float acc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            blk_mma_acc(acc2, Nb(i, i), NLD, xs, AOLD, lane);
            blk_store(Ab(i, j), AOLD, acc2, lane);
        } else {
            blk_store(Ab(i, j), AOLD, acc, lane);
        }
    }
    named_bar(BAR_PREP, 128);
    // d) A30 = D3 (W30 + N32 A20)
    if (pw == 0) {
        float acc[2][4];
        blk_load(acc, Ab(3, 0), AOLD, lane);
        blk_mma_acc(acc, Nb(3, 2), NLD, Ab(2, 0), AOLD, lane);
        blk_store(xs, AOLD, acc, lane);
        __syncwarp();
        float acc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        blk_mma_acc(acc2, Nb(3, 3), NLD, xs, AOLD, lane);
        blk_store(Ab(3, 0), AOLD, acc2, lane);
    }
    named_bar(BAR_PREP, 128);
}

template <int DK>
__global__ void __launch_bounds__(kThreads, 1)
prefill_chunk_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                     const PrefillArgs args) {
    using L = PrefillSmem<DK>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(sm + L::OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_BAR + sizeof(Bars));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* Nsm = reinterpret_cast<float*>(sm + L::OFF_N);
    float* Ao = reinterpret_cast<float*>(sm + L::OFF_AO);
    float* Xs = reinterpret_cast<float*>(sm + L::OFF_XS);
    float* gates = reinterpret_cast<float*>(sm + L::OFF_G);
    float* ocbuf = reinterpret_cast<float*>(sm + L::OFF_OC);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int tile = blockIdx.x % args.ntiles;
    const int bh = blockIdx.x / args.ntiles;       // b * Hv + h
    const int h = bh % args.Hv;
    const int bidx = bh / args.Hv;
    const int hq = h / (args.Hv / args.Hqk);
    const int T = args.T;
    const int nchunks = (T + kC - 1) / kC;
    const int v0 = tile * 128;
    const int dv_valid = min(128, args.dv - v0);
    const int nvb = (dv_valid + 63) / 64;
    unsigned int* err = args.err;

    if (tid == 0) {
        uint64_t* all = reinterpret_cast<uint64_t*>(bars);
        for (int i = 0; i < static_cast<int>(sizeof(Bars) / 8); ++i) mbar_init(&all[i], 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
        tma_prefetch_desc(&map_o);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ======================= TMA producer (lane 0: q/k ring, lane 1: v)
        if (lane == 0) {
            for (int c = 0; c < nchunks; ++c) {
                const int slot = c & 1;
                if (c >= 2 && !mbar_wait_or_abort(&bars->qk_free[slot], ((c >> 1) - 1) & 1, err, abort_flag)) break;
                uint8_t* dst = sm + (slot ? L::OFF_QK1 : L::OFF_QK0);
                mbar_arrive_expect_tx(&bars->qk_full[slot], 2 * L::CB * 8192);
#pragma unroll
                for (int cb = 0; cb < L::CB; ++cb) {
                    tma_load_4d(dst + cb * 16384, &map_q, &bars->qk_full[slot], cb * 64, c * kC, hq, bidx);
                    tma_load_4d(dst + cb * 16384 + 8192, &map_k, &bars->qk_full[slot], cb * 64, c * kC, hq, bidx);
                }
            }
        } else if (lane == 1) {
            for (int c = 0; c < nchunks; ++c) {
                if (c >= 1 && !mbar_wait_or_abort(&bars->v_free, (c - 1) & 1, err, abort_flag)) break;
                mbar_arrive_expect_tx(&bars->v_full, nvb * 8192);
                for (int vb = 0; vb < nvb; ++vb)
                    tma_load_4d(sm + L::OFF_V + vb * 8192, &map_v, &bars->v_full, v0 + vb * 64, c * kC, h, bidx);
            }
        }
    } else if (warp <= 4) {
        // ======================= PREP warpgroup
        const int pt = tid - 32;                           // 0..127
        const int pw = pt >> 5;                            // 0..3
        const int tl = ((warp & 3) << 5) | lane;           // TMEM lane of this thread
        const uint32_t lane_off = static_cast<uint32_t>(warp & 3) << 21;   // (32*(warp%4)) << 16
        const bool leader = (pt == 32);                    // MMA issuer: not on the gate warp (pw == 0)
        const float A_neg = -expf(args.A_log[h]);
        const float dtb = args.dt_bias_vec ? args.dt_bias_vec[h] : args.dt_bias;
        const float scale = args.scale;
        const long gate_base = static_cast<long>(bh) * T;
        constexpr float kLog2e = 1.4426950408889634f;
        // gate inputs (two tokens per lane of warp pw == 0), loaded one chunk ahead
        float pa0 = 0.f, pa1 = 0.f, pb0 = 0.f, pb1 = 0.f, pm0 = 0.f, pm1 = 0.f;
        auto load_gates = [&](int cc) {
            const int tok = cc * kC + 2 * lane;
            pa0 = pa1 = pb0 = pb1 = pm0 = pm1 = 0.f;
            if (pw == 0 && cc < nchunks) {
                if (tok < T) {
                    pa0 = load_gate(args.a, gate_base + tok, args.gate_dtype);
                    pb0 = load_gate(args.b, gate_base + tok, args.gate_dtype);
                    pm0 = args.mask ? args.mask[static_cast<long>(bidx) * T + tok] : 1.f;
                }
                if (tok + 1 < T) {
                    pa1 = load_gate(args.a, gate_base + tok + 1, args.gate_dtype);
                    pb1 = load_gate(args.b, gate_base + tok + 1, args.gate_dtype);
                    pm1 = args.mask ? args.mask[static_cast<long>(bidx) * T + tok + 1] : 1.f;
                }
            }
        };
        load_gates(0);
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
            const int par = c & 1;
            float* g = gates + par * L::GSTRIDE;
            if (c >= 2) mbar_wait_or_abort(&bars->chain_done[par], ((c >> 1) - 1) & 1, err, abort_flag);

            // ---- [Q;K] K^T on tensor cores (overlaps the gate computation below)
            mbar_wait_or_abort(&bars->qk_full[par], (c >> 1) & 1, err, abort_flag);
            uint8_t* qk_s = sm + (par ? L::OFF_QK1 : L::OFF_QK0);
            if (leader && !*abort_flag) {
                tc_fence_after();
                const uint32_t sqk = smem_u32(qk_s);
                constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
#pragma unroll
                for (int kk = 0; kk < DK / 16; ++kk) {
                    const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16_ss(tmem + COL_QKK, sdesc_sw128(sqk + o, 16, 1024),
                                 sdesc_sw128(sqk + o + 8192, 16, 1024), id64, kk > 0);
                }
                umma_commit(&bars->qkk_done);
            }

            // ---- gates (prefill_ref.py:49-64, 79-91) on one warp, two tokens per lane
            if (pw == 0) {
                const int t0 = 2 * lane;
                const int tok = c * kC + t0;
                float lg0 = 0.f, lg1 = 0.f, bm0 = 0.f, bm1 = 0.f;
                if (tok < T) {
                    lg0 = A_neg * softplus_fast(pa0 + dtb);
                    bm0 = sigmoid_fast(pb0) * pm0;
                }
                if (tok + 1 < T) {
                    lg1 = A_neg * softplus_fast(pa1 + dtb);
                    bm1 = sigmoid_fast(pb1) * pm1;
                }
                float sc = lg0 + lg1;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, sc, o);
                    if (lane >= o) sc += y;
                }
                const float ll2 = __shfl_sync(0xffffffffu, sc, 31) * kLog2e;
                const float m2 = 0.5f * ll2;
                const float l21 = sc * kLog2e, l20 = (sc - lg1) * kLog2e;
                const float el0 = ex2_approx(l20), el1 = ex2_approx(l21);
                *reinterpret_cast<float2*>(g + G_LAM2 * 64 + t0) = make_float2(l20, l21);
                *reinterpret_cast<float2*>(g + G_U * 64 + t0) = make_float2(ex2_approx(l20 - m2), ex2_approx(l21 - m2));
                *reinterpret_cast<float2*>(g + G_W * 64 + t0) = make_float2(ex2_approx(m2 - l20), ex2_approx(m2 - l21));
                *reinterpret_cast<float2*>(g + G_EDEC * 64 + t0) =
                    make_float2(ex2_approx(ll2 - l20), ex2_approx(ll2 - l21));
                *reinterpret_cast<float2*>(g + G_BM * 64 + t0) = make_float2(bm0, bm1);
                *reinterpret_cast<float2*>(g + G_BME * 64 + t0) = make_float2(bm0 * el0, bm1 * el1);
                *reinterpret_cast<float2*>(g + G_OC * 64 + t0) = make_float2(pm0 * scale * el0, pm1 * scale * el1);
                *reinterpret_cast<float2*>(g + G_MK * 64 + t0) = make_float2(pm0, pm1);
                if (lane == 0) {
                    g[G_TOT * 64 + 2] = ex2_approx(ll2);                  // gamma_c
                    g[G_TOT * 64 + 3] = (ll2 < -240.f) ? 1.f : 0.f;        // u_t * w_s could overflow
                }
                load_gates(c + 1);                         // prefetch the next chunk's gate inputs
            }
            named_bar(BAR_PREP, 128);      // gate vectors complete
            const bool direct = g[G_TOT * 64 + 3] != 0.f;
            mbar_wait_or_abort(&bars->qkk_done, c & 1, err, abort_flag);
            tc_fence_after();

            // ---- P (lanes 0-63) and N (lanes 64-127): only the lower triangle is computed
            {
                float row[64];
                tmem_ld64(tmem + lane_off + COL_QKK, row);
                const float* gw = g + G_W * 64;
                const float* gl2 = g + G_LAM2 * 64;
                if (tl < kC) {
                    const int t = tl;
                    const float coef = scale * g[G_MK * 64 + t];
                    const float cu = coef * g[G_U * 64 + t];
                    const float lt = gl2[t];
                    uint8_t* prow = sm + L::OFF_P + par * 8192;
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch) {
                        uint4 w4 = make_uint4(0u, 0u, 0u, 0u);
                        if (8 * ch <= t) {
                            float e[8];
                            if (!direct) {
#pragma unroll
                                for (int u = 0; u < 8; ++u) e[u] = (8 * ch + u <= t) ? row[8 * ch + u] * (cu * gw[8 * ch + u]) : 0.f;
                            } else {
#pragma unroll
                                for (int u = 0; u < 8; ++u)
                                    e[u] = (8 * ch + u <= t) ? row[8 * ch + u] * (coef * ex2_approx(lt - gl2[8 * ch + u])) : 0.f;
                            }
                            w4 = pack8(e);
                        }
                        *reinterpret_cast<uint4*>(prow + sw128_chunk(t, ch)) = w4;
                    }
                } else {
                    const int t = tl - kC;
                    const float coef = -g[G_BM * 64 + t];
                    const float cu = coef * g[G_U * 64 + t];
                    const float lt = gl2[t];
                    float* nrow = Nsm + t * L::NLD;
                    const int send = (t | 15) + 1;         // through the end of t's diagonal block
#pragma unroll
                    for (int s4 = 0; s4 < 16; ++s4) {
                        if (4 * s4 < send) {
                            float o4[4];
                            if (!direct) {
#pragma unroll
                                for (int u = 0; u < 4; ++u) o4[u] = (4 * s4 + u < t) ? row[4 * s4 + u] * (cu * gw[4 * s4 + u]) : 0.f;
                            } else {
#pragma unroll
                                for (int u = 0; u < 4; ++u)
                                    o4[u] = (4 * s4 + u < t) ? row[4 * s4 + u] * (coef * ex2_approx(lt - gl2[4 * s4 + u])) : 0.f;
                            }
                            *reinterpret_cast<float4*>(nrow + 4 * s4) = make_float4(o4[0], o4[1], o4[2], o4[3]);
                        }
                    }
                }
            }
            tc_fence_before();
            named_bar(BAR_PREP, 128);

            // ---- A = (I - N)^-1
            invert_unit_lower<L::NLD, L::AOLD>(Nsm, Ao, Xs, pw, lane);

            // ---- A1 = A diag(beta'), A2 = A diag(beta' e^Lambda) -> X (hi/lo rows [t][s])
            if (c >= 1) mbar_wait_or_abort(&bars->ws_done, (c - 1) & 1, err, abort_flag);
            {
                const int t = pt >> 1, hf = pt & 1;
                const int ib = t >> 4, r = t & 15;
                const float* bm = g + G_BM * 64;
                const float* bme = g + G_BME * 64;
                uint8_t* X = sm + L::OFF_X;
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    const int s0 = 32 * hf + 8 * ch;
                    const uint32_t off = sw128_chunk(t, 4 * hf + ch);
                    uint4 h1 = make_uint4(0u, 0u, 0u, 0u), l1 = h1, h2 = h1, l2 = h1;
                    if (s0 <= t) {
                        const int jb = s0 >> 4;
                        const float* src = (jb == ib) ? Nsm + t * L::NLD + s0
                                                      : Ao + ao_slot(ib, jb) * 16 * L::AOLD + r * L::AOLD + (s0 & 15);
                        const float4 x0 = *reinterpret_cast<const float4*>(src);
                        const float4 x1 = *reinterpret_cast<const float4*>(src + 4);
                        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                        float e1[8], e2[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float xa = (s0 + u <= t) ? xv[u] : 0.f;
                            e1[u] = xa * bm[s0 + u];
                            e2[u] = xa * bme[s0 + u];
                        }
                        split8(e1, h1, l1);
                        split8(e2, h2, l2);
                    }
                    *reinterpret_cast<uint4*>(X + L::X_A1H + off) = h1;
                    *reinterpret_cast<uint4*>(X + L::X_A1L + off) = l1;
                    *reinterpret_cast<uint4*>(X + L::X_A2H + off) = h2;
                    *reinterpret_cast<uint4*>(X + L::X_A2L + off) = l2;
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_bar(BAR_PREP, 128);

            // ---- U^T = V^T A1^T (into UT[par]), W^T = K^T A2^T (into COL_WT); the chain waits for them
            if (leader) {
                mbar_arrive(&bars->prep_done[par]);       // P, gates, A1/A2 are in shared memory
                if (c >= 1) mbar_wait_or_abort(&bars->wt_read, (c - 1) & 1, err, abort_flag);
                const bool okv = mbar_wait_or_abort(&bars->v_full, c & 1, err, abort_flag);
                tc_fence_after();
                if (okv && !*abort_flag) {
                    const uint32_t sv = smem_u32(sm + L::OFF_V);
                    const uint32_t sk = smem_u32(qk_s) + 8192;
                    const uint32_t sx = smem_u32(sm + L::OFF_X);
                    constexpr uint32_t id_mn = idesc_bf16(128, 64, true, false);
#pragma unroll
                    for (int p = 0; p < 2; ++p) {
                        const uint32_t b1 = sx + (p ? L::X_A1L : L::X_A1H);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_bf16_ss(tmem + COL_UT + par * 64, sdesc_sw128(sv + kk * 2048, 8192, 1024),
                                         sdesc_sw128(b1 + kk * 32, 16, 1024), id_mn, (p > 0 || kk > 0) ? 1u : 0u);
                    }
#pragma unroll
                    for (int p = 0; p < 2; ++p) {
                        const uint32_t b2 = sx + (p ? L::X_A2L : L::X_A2H);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_bf16_ss(tmem + COL_WT, sdesc_sw128(sk + kk * 2048, 16384, 1024),
                                         sdesc_sw128(b2 + kk * 32, 16, 1024), id_mn, (p > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&bars->uw_done);
                    umma_commit(&bars->v_free);
                }
            }
        }
    } else {
        // ======================= CHAIN warpgroup
        const int ct = tid - 160;                          // 0..127
        const int j = ((warp & 3) << 5) | lane;            // TMEM lane = value row j (or key row d for W^T)
        const uint32_t lane_off = static_cast<uint32_t>(warp & 3) << 21;
        const bool leader = (ct == 0);
        const long s_base = static_cast<long>(bh) * DK * args.dv + v0;
        uint8_t* sr = sm + L::OFF_SR;

        // output tile of chunk cc from (Q S)^T and (P dV)^T in TMEM:
        //   o[t, j] = oc_t (Q S)[t,j] + (P dV)[t,j]  -> smem [t][j] (128B swizzle) -> TMA store
        auto write_output = [&](int cc) {
            float qs[64], pd[64];
            tmem_ld64(tmem + lane_off + COL_QS, qs);
            tmem_ld64(tmem + lane_off + COL_PDV, pd);
            const float* oc = ocbuf + (cc & 1) * 64;
            uint8_t* ob = sr + L::OST + (j >> 6) * 8192;
            const uint32_t jj = j & 63;
#pragma unroll
            for (int t = 0; t < kC; ++t)
                *reinterpret_cast<uint16_t*>(ob + sw128_off(t, jj)) = f32_to_bf16_bits(fmaf(oc[t], qs[t], pd[t]));
            fence_async_smem();
            tc_fence_before();
            named_bar(BAR_CHAIN, 128);
            if (leader && !*abort_flag) {
                for (int vb = 0; vb < nvb; ++vb) tma_store_4d(&map_o, sr + L::OST + vb * 8192, v0 + vb * 64, cc * kC, h, bidx);
                bulk_commit();
            }
        };

        // initial state -> TMEM (S^T: lane j = value column, column d = key index)
#pragma unroll
        for (int blk = 0; blk < DK / 32; ++blk) {
            float vals[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int d = blk * 32 + i;
                vals[i] = (args.state_in && j < dv_valid) ? args.state_in[s_base + static_cast<long>(d) * args.dv + j]
                                                          : 0.f;
            }
            tmem_st32(tmem + lane_off + COL_ST + 32 * blk, vals);
        }
        tmem_st_wait();

#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
            const int par = c & 1;
            const float* g = gates + par * L::GSTRIDE;
            uint8_t* qk_s = sm + (par ? L::OFF_QK1 : L::OFF_QK0);
            if (c >= 1) write_output(c - 1);               // previous chunk's output, while prep runs
            mbar_wait_or_abort(&bars->prep_done[par], (c >> 1) & 1, err, abort_flag);
            mbar_wait_or_abort(&bars->uw_done, c & 1, err, abort_flag);
            tc_fence_after();

            // ---- W^T (lane d) -> X as MN-major B operand rows [d][t], hi/lo
            {
                float row[64];
                tmem_ld64(tmem + lane_off + COL_WT, row);
                store_row_split(sm + L::OFF_X + L::X_WTH, sm + L::OFF_X + L::X_WTL, j, row);
            }
            if (leader) bulk_wait_read0();                 // the output tile has left shared memory
            named_bar(BAR_CHAIN, 128);
            // ---- S^T -> bf16 hi/lo rows [j][d]; S^T *= gamma_c in TMEM
            const float gamma_c = g[G_TOT * 64 + 2];
#pragma unroll
            for (int blk = 0; blk < DK / 32; ++blk) {
                float vals[32];
                tmem_ld32(tmem + lane_off + COL_ST + 32 * blk, vals);
                tmem_ld_wait();
                const int cb = blk >> 1;
#pragma unroll
                for (int ch4 = 0; ch4 < 4; ++ch4) {
                    uint4 hw, lw;
                    split8(&vals[8 * ch4], hw, lw);
                    const uint32_t off = cb * 16384 + sw128_chunk(j, (blk & 1) * 4 + ch4);
                    *reinterpret_cast<uint4*>(sr + off) = hw;
                    *reinterpret_cast<uint4*>(sr + L::S_LO + off) = lw;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) vals[i] *= gamma_c;
                tmem_st32(tmem + lane_off + COL_ST + 32 * blk, vals);
            }
            tmem_st_wait();
            fence_async_smem();
            tc_fence_before();
            named_bar(BAR_CHAIN, 128);
            if (leader) mbar_arrive(&bars->wt_read);

            // ---- dV^T = U^T - S^T W^T (3 split terms, negated B, in place in UT[par]); (Q S_hi)^T
            if (leader && !*abort_flag) {
                tc_fence_after();
                const uint32_t ssr = smem_u32(sr);
                const uint32_t swt = smem_u32(sm + L::OFF_X);
                constexpr uint32_t id_ws = idesc_bf16(128, 64, false, true) | (1u << 14);   // negate B
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    const uint32_t sa = ssr + (p == 1 ? L::S_LO : 0);
                    const uint32_t sb = swt + (p == 2 ? L::X_WTL : L::X_WTH);
#pragma unroll
                    for (int kk = 0; kk < DK / 16; ++kk)
                        umma_bf16_ss(tmem + COL_UT + par * 64,
                                     sdesc_sw128(sa + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                                     sdesc_sw128(sb + kk * 2048, 16, 1024), id_ws, 1u);
                }
#pragma unroll
                for (int kk = 0; kk < DK / 16; ++kk) {
                    const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16_ss(tmem + COL_QS, sdesc_sw128(ssr + o, 16, 1024), sdesc_sw128(smem_u32(qk_s) + o, 16, 1024),
                                 idesc_bf16(128, 64, false, false), kk > 0);
                }
                umma_commit(&bars->ws_done);
            }
            mbar_wait_or_abort(&bars->ws_done, c & 1, err, abort_flag);
            tc_fence_after();

            // ---- dV (bf16) and dV' = dV * exp(Lambda_last - Lambda) (hi/lo) -> rows [j][t]
            {
                float row[64];
                tmem_ld64(tmem + lane_off + COL_UT + par * 64, row);
                const float* edec = g + G_EDEC * 64;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    const uint32_t off = sw128_chunk(j, ch);
                    *reinterpret_cast<uint4*>(sr + L::DVB + off) = pack8(&row[8 * ch]);
                    float e[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) e[u] = row[8 * ch + u] * edec[8 * ch + u];
                    uint4 hw, lw;
                    split8(e, hw, lw);
                    *reinterpret_cast<uint4*>(sr + L::DVH + off) = hw;
                    *reinterpret_cast<uint4*>(sr + L::DVL + off) = lw;
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_bar(BAR_CHAIN, 128);

            // ---- S^T += dV'^T K (K as MN-major B);  (P dV)^T = dV^T P^T
            if (leader && !*abort_flag) {
                tc_fence_after();
                const uint32_t ssr = smem_u32(sr);
                const uint32_t sk = smem_u32(qk_s) + 8192;
                const uint32_t sp = smem_u32(sm + L::OFF_P + par * 8192);
                constexpr uint32_t idst = idesc_bf16(128, DK, false, true);
                constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const uint32_t ra = ssr + (p ? L::DVL : L::DVH);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16_ss(tmem + COL_ST, sdesc_sw128(ra + kk * 32, 16, 1024),
                                     sdesc_sw128(sk + kk * 2048, 16384, 1024), idst, 1u);
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + COL_PDV, sdesc_sw128(ssr + L::DVB + kk * 32, 16, 1024),
                                 sdesc_sw128(sp + kk * 32, 16, 1024), id64, kk > 0);
                umma_commit(&bars->st_done);
                umma_commit(&bars->qk_free[par]);
            }
            mbar_wait_or_abort(&bars->st_done, c & 1, err, abort_flag);
            tc_fence_after();
            if (ct < kC) ocbuf[par * 64 + ct] = g[G_OC * 64 + ct];
            named_bar(BAR_CHAIN, 128);
            if (leader) mbar_arrive(&bars->chain_done[par]);
        }
        if (nchunks >= 1) write_output(nchunks - 1);
        if (leader) bulk_wait_all0();

        // ---- final state S^T -> state_out [dk][dv]
        if (!*abort_flag && args.state_out) {
#pragma unroll
            for (int blk = 0; blk < DK / 32; ++blk) {
                float vals[32];
                tmem_ld32(tmem + lane_off + COL_ST + 32 * blk, vals);
                tmem_ld_wait();
                if (j < dv_valid) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        args.state_out[s_base + static_cast<long>(blk * 32 + i) * args.dv + j] = vals[i];
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

std::once_flag g_attr_once[2][64];
int g_attr_status[2][64];

template <int DK>
int launch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                   const PrefillArgs& args, int grid, cudaStream_t st) {
    using L = PrefillSmem<DK>;
    int dev = 0;
    cudaGetDevice(&dev);
    const int which = DK == 128 ? 1 : 0;
    std::call_once(g_attr_once[which][dev & 63], [&]() {
        g_attr_status[which][dev & 63] =
            cudaFuncSetAttribute(prefill_chunk_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) ==
                    cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
    });
    if (g_attr_status[which][dev & 63] != GDN_OK)
        return fail(GDN_ERR_CUDA, "gdn_prefill_fwd: cannot grant %d B of shared memory", L::ALLOC);
    prefill_chunk_kernel<DK><<<grid, kThreads, L::ALLOC, st>>>(mq, mk, mv, mo, args);
    return launch_status("gdn_prefill_fwd");
}

// q/k/v/o map: dims (D, T, H, B) innermost first, box (64, 64, 1, 1), 128B swizzle.
int make_act_map(CUtensorMap* m, const void* base, int D, int T, int H, int B, int layout) {
    uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(T), static_cast<uint64_t>(H),
                        static_cast<uint64_t>(B)};
    uint64_t strides[3];
    const uint64_t e = 2;
    if (layout == GDN_LAYOUT_BHTD) {
        strides[0] = e * D;                  // T
        strides[1] = e * D * T;              // H
        strides[2] = e * D * T * H;          // B
    } else {
        strides[0] = e * D * H;              // T
        strides[1] = e * D;                  // H
        strides[2] = e * D * H * T;          // B
    }
    uint32_t box[4] = {64, 64, 1, 1};
    return make_map_bf16(m, base, 4, dims, strides, box, true);
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_fwd(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                               const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                               const float* mask, const float* state_in, void* out, float* state_out, int B, int T,
                               int Hqk, int Hv, int dk, int dv, int layout, float scale, void* stream) {
    using namespace gdn;
    if (!q || !k || !v || !A_log || !a || !b_logits || !out)
        return fail(GDN_ERR_NULL, "gdn_prefill_fwd: q, k, v, A_log, a, b_logits and out are required");
    if (B <= 0 || T <= 0 || Hqk <= 0 || Hv <= 0 || Hv % Hqk != 0)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_fwd: bad B=%d T=%d Hqk=%d Hv=%d (need > 0 and Hv %% Hqk == 0)", B, T,
                    Hqk, Hv);
    if (gate_dtype != GDN_DTYPE_BF16 && gate_dtype != GDN_DTYPE_F32)
        return fail(GDN_ERR_DTYPE, "gdn_prefill_fwd: gate_dtype must be GDN_DTYPE_BF16 or GDN_DTYPE_F32");
    if (layout != GDN_LAYOUT_BHTD && layout != GDN_LAYOUT_BTHD)
        return fail(GDN_ERR_DTYPE, "gdn_prefill_fwd: layout must be GDN_LAYOUT_BHTD or GDN_LAYOUT_BTHD");
    if (!(dk == 64 || dk == 128) || !(dv == 64 || dv == 128 || dv == 256))
        return fail(GDN_ERR_UNSUPPORTED, "gdn_prefill_fwd: dk=%d dv=%d not supported (dk in {64,128}, dv in {64,128,256})",
                    dk, dv);
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || (state_in && !aligned16(state_in)) ||
        (state_out && !aligned16(state_out)))
        return fail(GDN_ERR_ALIGN, "gdn_prefill_fwd: q, k, v, out and states must be 16-byte aligned");
    const long ntiles = (dv + 127) / 128;
    if (static_cast<long>(B) * Hv * ntiles > 0x7fffffffL)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_fwd: B*Hv too large");
    int st = check_sm100();
    if (st != GDN_OK) return st;
    if (scale == 0.f) scale = 1.f / sqrtf(static_cast<float>(dk));

    CUtensorMap mq, mk, mv, mo;
    if ((st = make_act_map(&mq, q, dk, T, Hqk, B, layout)) != GDN_OK) return st;
    if ((st = make_act_map(&mk, k, dk, T, Hqk, B, layout)) != GDN_OK) return st;
    if ((st = make_act_map(&mv, v, dv, T, Hv, B, layout)) != GDN_OK) return st;
    if ((st = make_act_map(&mo, out, dv, T, Hv, B, layout)) != GDN_OK) return st;

    PrefillArgs args;
    args.a = a;
    args.b = b_logits;
    args.gate_dtype = gate_dtype;
    args.A_log = A_log;
    args.dt_bias = dt_bias;
    args.dt_bias_vec = dt_bias_vec;
    args.mask = mask;
    args.state_in = state_in;
    args.state_out = state_out;
    args.err = device_error_word();
    args.B = B;
    args.T = T;
    args.Hqk = Hqk;
    args.Hv = Hv;
    args.dv = dv;
    args.ntiles = static_cast<int>(ntiles);
    args.layout = layout;
    args.scale = scale;
    const int grid = static_cast<int>(B * Hv * ntiles);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dk == 128) return launch_prefill<128>(mq, mk, mv, mo, args, grid, s);
    return launch_prefill<64>(mq, mk, mv, mo, args, grid, s);
}
