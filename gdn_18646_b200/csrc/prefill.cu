// prefill.cu -- chunked gated-delta-rule prefill on tcgen05 tensor cores.
//
// Math: reference/prefill_ref.py:11-132 (chunk C = 64, WY / UT form).  Replaces
// the reference's gdn_prefill_v2_kernel (kernels/prefill_chunked.cu:41-417),
// which runs fp32 CUDA-core loops with one thread per value column and
// hard-codes H=16, K=128, V=256.
//
// Per 64-token chunk, with Lambda the in-chunk cumulative log decay and
// beta' = beta * mask:
//   N[t,s] = -beta'_t (k_t . k_s) exp(Lambda_t - Lambda_s)  (t > s)
//   A      = (I - N)^-1                                      (prefill_ref.py:96-101)
//   U      = A diag(beta') V,  W = A diag(beta' e^Lambda) K  (prefill_ref.py:103-104)
//   dV     = U - W S                                         (:117-118)
//   O      = diag(m) [ scale diag(e^Lambda) Q S + P dV ],
//            P[t,s] = scale (q_t.k_s) exp(Lambda_t - Lambda_s), s <= t   (:120-122)
//   S     <- e^{Lambda_last} S + K^T diag(e^{Lambda_last - Lambda}) dV   (:124-126)
//
// Everything that does not involve S is independent per chunk, so the work is
// split into two launches:
//
// 1. prefill_prep_kernel: one task per (batch, value head, chunk), all in
//    parallel (persistent CTAs, 3 per SM).  Gates, [Q;K] K^T on tensor cores,
//    P and N, the 64x64 inverse, A1 = A diag(beta'), A2 = A diag(beta' e^Lambda),
//    W^T = K^T A2^T on tensor cores.  It writes one chunk record to a workspace:
//    A1 as bf16 hi/lo pairs, W in tf32, P in bf16, and the gate vectors the
//    recurrence needs -- each operand already in the 128-byte-swizzled shared
//    memory image the second kernel's MMAs read, so it is fetched with one
//    bulk copy.
// 2. prefill_chain_kernel: one CTA per (batch, value head, 128-wide value
//    tile) walks the chunks in order.  The fp32 state lives in TMEM,
//    TRANSPOSED (S^T: value index = TMEM lane, so the value tile is the
//    M = 128 dimension of every product), for the whole sequence.  Per chunk:
//      [U_l^T | U_h^T] = V^T [A1_lo^T | A1_hi^T]   (A, B from shared memory; one N=128 MMA per K step)
//      [U_h^T | O^T] -= S^T [W^T | -Q~^T]          (tf32: A = the fp32 state straight from TMEM,
//                                                   B = W from the record and -oc Q built in place)
//      dV^T = U_l^T + U_h^T -> bf16 and dV'^T = dV^T diag(e^{Lambda_last - Lambda}) -> hi/lo, in TMEM;
//      S^T <- gamma S^T in place                  (CUDA cores, TMEM -> TMEM)
//      S^T  += dV'^T K                             (A from TMEM, K as MN-major B)
//      O^T  += dV^T P^T                            (A from TMEM)
//      o     = O -> bf16 tile -> TMA store
//    with warp roles: warp 0 the copies, warp 1 the MMA issuer, warps 2-9 the
//    state path (each TMEM lane quadrant twice, one token half each) and the
//    output tile, warps 10-13 the -oc Q image.  Only the state path's
//    CUDA-core work and the [W | Q~] S and update MMAs sit on the sequential
//    critical path; the chunk buffers in TMEM are double-buffered so P dV of
//    one chunk and U of the next run in the tensor pipe meanwhile.
//
// Precision: A diag(beta') and dV' enter their products as bf16 hi + lo pairs
// (~16 mantissa bits), W S runs in tf32 straight from the fp32 state (fp32
// accumulation), q/k/v are exact bf16 inputs, P dV uses single bf16 (o is bf16).  Decay ratios
// exp(Lambda_t - Lambda_s) are formed as u_t * w_s with u_t = 2^(l_t - m),
// w_s = 2^(m - l_s) around the chunk's mid decay m (never gamma_t / gamma_s);
// chunks whose total decay could overflow that product fall back to one exp2
// per element.  Every mbarrier wait is bounded; a timeout raises a CTA-wide
// abort and all roles drain through their barriers.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {
namespace {

constexpr int kC = 64;                 // chunk length
// Test hook (gdn_test_prefill_hooks): a record whose ready flag the streamed
// schedule's prep workers leave unset, or -1.
static __device__ long long g_unpublished_record = -1;
constexpr int BAR_PREP = 1;            // named barrier of the prep kernel's 128 threads
constexpr int BAR_OUT = 2;             // named barrier of the chain kernel's Q~ warps
constexpr int BAR_STATE = 3;           // named barrier of the chain kernel's state-path warps

// ---------------------------------------------------------------------------
// Chunk record (bytes, 1024-aligned images), written by the gate and prep kernels:
//   GB        gate vectors of the chunk for the prep kernel (PrepGate layout)
//   A1        A diag(beta') as bf16 lo then hi images, rows t, cols s
//             (one K-major B of [U_l^T | U_h^T] = V^T [A1_lo^T | A1_hi^T])
//   W         W, rows t, cols d, tf32 (rounded to nearest), 32-column blocks
//             (rows 0-63 of the K-major B of S^T [W^T | Q~^T])
//   P         rows t, cols s                       (K-major B of dV^T P^T)
//   G         floats: [0,64) oc_t = m_t scale e^Lambda_t, [64,128) e^{Lambda_last - Lambda_t},
//             [128] gamma = e^{Lambda_last}
// The chain fetches A1, W (one copy per 32-key block) and P | G per chunk with bulk copies.
// ---------------------------------------------------------------------------
template <int DK>
struct Rec {
    static constexpr int GB = 0;                      // gate vectors for the prep kernel (PrepGate)
    static constexpr int A1 = 2048;                   // lo, then hi at + 8192
    static constexpr int W = A1 + 16384;
    static constexpr int P = W + DK * 256;
    static constexpr int G = P + 8192;
    static constexpr int BYTES = G + 1024;
    static_assert(BYTES % 1024 == 0, "record images must stay 1024-aligned");
};

// ---------------------------------------------------------------------------
// prep kernel layout
// ---------------------------------------------------------------------------
constexpr int kPrepThreads = 128;
constexpr int kPrepCtasPerSm = 3;
constexpr int kPrepTmemCols = 128;
constexpr int kPrepPerCta = 3;         // prep workers per CTA of the overlap kernel
constexpr uint32_t P_COL_QKK = 0;      // [Q;K] K^T (lanes 0-63 QK^T, 64-127 KK^T)
constexpr uint32_t P_COL_WT = 64;      // W^T (lanes = key index d)

template <int DK>
struct PrepSmem {
    static constexpr int CB = DK / 64;                    // 64-wide column blocks of q/k
    static constexpr int QK_BYTES = CB * 16384;           // per block [Q 64 rows | K 64 rows] x 128 B
    static constexpr int OFF_A2H = 0;                     // A2 hi over the dead Q block 0
    static constexpr int OFF_A2L = (DK == 128) ? 16384 : QK_BYTES;   // over Q block 1, or its own 8 KB
    static constexpr int END_A = (DK == 128) ? QK_BYTES : QK_BYTES + 8192;
    static constexpr int NLD = 68;                        // fp32 row stride of N (16 B aligned rows)
    static constexpr int OFF_N = END_A;                   // N; diagonal blocks replaced by D_i
    static constexpr int AOLD = 20;                       // fp32 row stride of 16x16 scratch blocks
    static constexpr int OFF_AO = OFF_N + 64 * NLD * 4;   // 6 off-diagonal blocks of A
    static constexpr int OFF_XS = OFF_AO + 6 * 16 * AOLD * 4;   // 3 per-warp 16x16 scratch blocks
    static constexpr int OFF_G = OFF_XS + 3 * 16 * AOLD * 4;    // gate vectors (record part GB)
    static constexpr int OFF_BAR = OFF_G + 2048;
    static constexpr int BYTES = OFF_BAR + 64;
    static constexpr int ALLOC = BYTES + 1024;
    // the M=128 W^T MMA reads a second 64-row block of K^T at +16384 (unused lanes when DK = 64)
    static_assert(DK == 128 || 8192 + 16384 + 8192 <= BYTES, "W^T operand window leaves shared memory");
    static_assert(kPrepCtasPerSm * (ALLOC + 1024) <= 233472, "prep kernel does not fit 3 CTAs per SM");
};

// per-chunk gate vectors for the prep kernel (floats, 64 per entry), record part GB
enum PrepGate {
    G_LAM2 = 0,   // Lambda_t * log2(e)
    G_U = 1,      // 2^(l_t - m), m = Lambda_last * log2(e) / 2
    G_W = 2,      // 2^(m - l_t)
    G_BM = 3,     // beta_t * mask_t
    G_BME = 4,    // beta_t * mask_t * exp(Lambda_t)
    G_MK = 5,     // mask_t (0 for padding)
    G_FLAG = 6,   // [0]: 1 when u_t * w_s could overflow (direct exp2 per element instead)
    G_COUNT = 7
};
constexpr int kGateBytes = G_COUNT * 64 * 4;     // 1792, bulk-copied with the q/k tiles

struct GateArgs {
    const void* a;
    const void* b;
    int gate_dtype;
    const float* A_log;
    float dt_bias;
    const float* dt_bias_vec;
    const float* mask;
    uint8_t* rec;
    int ntasks, T, Hv, nchunks;
    float scale;
    const int* cu;       // varlen: sequence b is packed tokens [cu[b], cu[b+1]); a, b_logits [Hv, Ttot]
    int Ttot;
    unsigned int* err;
    unsigned int* ready; // streamed schedule: per-record ready flags, cleared here
    long gate_ld;        // elements between the rows of mask [B rows]
    long g_b, g_h, g_t;  // element strides of a, b_logits over (batch, value head, token)
};

struct PrepArgs {
    uint8_t* rec;
    unsigned int* err;
    int ntasks;          // B * Hv * ncp: the chunks [c0, c0 + ncp) of every sequence
    int Hqk, Hv, nchunks, c0, ncp;
    float scale;
    const int* cu;       // varlen sequence offsets or null
    int Ttot;
    unsigned int* ready; // streamed schedule: set once a record is complete in global memory
    int chunk_major;     // task order: chunk-major (all sequences' chunk 0 first) for the streamed schedule
};

// ---------------------------------------------------------------------------
// chain kernel layout
// ---------------------------------------------------------------------------
constexpr int kChainThreads = 448;     // 14 warps
constexpr int kChainTmemCols = 512;
// TMEM columns (128 lanes; lane j = value column of the tile):
constexpr uint32_t C_X = 0;            // S^T fp32 (DK columns): A operand of [W | Q~] S (tf32)
constexpr uint32_t C_BUF = 128;        // two chunk buffers of 192 columns, buffer c & 1 for chunk c:
                                       //   +0   U_l^T = V^T A1_lo^T (64 token columns); after the state-path
                                       //        pass: dV^T bf16 pairs, token half g at 32g (16 columns)
                                       //   +64  U_h^T = V^T A1_hi^T, then - (W S)^T: U_l + U_h = dV^T; after the
                                       //        state-path pass: dV'^T hi/lo pairs, half g hi at 32g, lo at 32g + 16
                                       //   +128 O^T: (Q~ S)^T in the same MMAs as W S, + (P dV)^T; zeroed after read
constexpr uint32_t C_BUF_STRIDE = 192;
static_assert(C_BUF + 2 * C_BUF_STRIDE <= kChainTmemCols, "chain TMEM map exceeds 512 columns");

template <int DK>
struct ChainSmem {
    static constexpr int CB = DK / 64;      // 64-column bf16 blocks of the q/k tiles
    // q/k ring, 2 slots: K tile (TMA; MN-major B of the state update) and q tile (TMA; read once
    // to build Q~); a slot is refilled once the state update and the Q~ build have read it
    static constexpr int KQ_K = 0;
    static constexpr int KQ_Q = CB * 8192;
    static constexpr int KQ_BYTES = 2 * CB * 8192;
    static constexpr int OFF_KQ = 0;
    // record ring, 3 slots: P (K-major B of dV^T P^T) and the chunk's gate floats, as they lie
    // in the record; P dV of chunk c is issued during chunk c + 1, so this ring is one deeper
    static constexpr int PG_P = 0;
    static constexpr int PG_G = 8192;
    static constexpr int PG_BYTES = 8192 + 1024;
    static constexpr int OFF_PG = 2 * KQ_BYTES;
    // [W | -Q~] image of the current chunk, K-major tf32: key block kb (32 keys) at kb * 16 KB,
    // rows 0-63 W (bulk-copied from the record), rows 64-127 -oc Q (built by the Q~ warps)
    static constexpr int OFF_IMG = OFF_PG + 3 * PG_BYTES;
    static constexpr int OFF_V = OFF_IMG + DK * 512;       // v tile, 2 blocks of 64 columns
    static constexpr int OFF_A1 = OFF_V + 16384;           // A1 lo | hi
    static constexpr int OFF_O = OFF_A1 + 16384;           // output staging, 2 x (2 blocks x 8 KB)
    static constexpr int OFF_BAR = OFF_O + 32768;
    static constexpr int BYTES = OFF_BAR + 256;
    static constexpr int ALLOC = BYTES + 1024;
    static_assert(KQ_BYTES % 1024 == 0 && PG_BYTES % 1024 == 0, "slot images must stay 1024-aligned");
    static_assert(ALLOC <= 232448, "chain kernel shared memory exceeds 227 KB");
};

struct ChainBars {
    uint64_t kq_full[2], kq_free[2], pg_full[3], pg_free[3], va_full, va_free, w_full;
    uint64_t ws_done, dv_done, st_done, pdv_done, qt_ready, o_free, init_done, mma_drain;
};
static_assert(sizeof(ChainBars) + 8 <= 256, "chain barriers exceed their shared-memory block");

struct ChainArgs {
    const uint8_t* rec;
    const float* state_in;
    float* state_out;
    unsigned int* err;
    int T, Hqk, Hv, dv, ntiles;
    int nchunks_total;   // chunks of the whole sequence (record indexing)
    int c0, nchunks;     // this launch walks chunks [c0, c0 + nchunks)
    const int* cu;       // varlen sequence offsets or null
    uint16_t* out;       // varlen: o [Ttot, Hv, dv], written directly for each sequence's last chunk
    int Ttot;
    const unsigned int* ready;   // streamed schedule: wait for a record's flag before loading it
};

// ---------------------------------------------------------------------------
// Streamed schedule: prep workers and chain CTAs in one cooperative launch; a
// prep worker publishes each finished record with a release flag, a chain CTA
// acquires it before its bulk loads.  The record bytes are written by the
// async proxy (bulk stores), so both sides fence the async proxy around the flag.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void publish_record(unsigned int* flag) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(1u) : "memory");
}
// Current value of a record flag (no ordering: only decides whether to prefetch the record)
__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned int* flag) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    return v;
}
// Non-blocking check of a record flag: true (with the async-proxy fence taken) once it is set;
// the caller bounds how long it keeps polling.
__device__ __forceinline__ bool record_ready(const unsigned int* flag) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v == 0) return false;
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return true;
}

// Varlen: first token and length of sequence b.  Offsets that are negative,
// decreasing or past Ttot make the sequence empty (nothing read or written for
// it beyond its state) and raise DERR_VARLEN in the device error word.
__device__ __forceinline__ int varlen_seq(const int* cu, int b, int Ttot, int& start, unsigned int* err) {
    start = cu[b];
    const int end = cu[b + 1];
    if (start < 0 || end < start || end > Ttot) {
        if (err) atomicOr(err, DERR_VARLEN);
        start = 0;
        return 0;
    }
    return end - start;
}
// chunks of a sequence of `len` tokens (at least one, so an empty sequence still
// passes its state on), at most the launch's chunk count
__device__ __forceinline__ int varlen_chunks(int len, int nchunks_total) {
    const int n = len > 0 ? (len + kC - 1) / kC : 1;
    return n < nchunks_total ? n : nchunks_total;
}

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
//   1. warps 0 and 1 invert the four 16x16 diagonal blocks by forward
//      substitution, one column of D_i per lane (16 lanes per block, the rows
//      of N_ii read as shared-memory broadcasts); D_i overwrites the diagonal
//      block of Nsm;
//   2. off-diagonal blocks, A_ij = D_i sum_{k=j}^{i-1} N_ik A_kj (A_jj = D_j),
//      as warp-level MMAs on 16x16 blocks, with the D-only terms issued first:
//        a) Y_{i,i-1} = N_{i,i-1} D_{i-1};  Z20 = N20 D0, Z31 = N31 D1, Z30 = N30 D0
//        b) A_{i,i-1} = D_i Y_{i,i-1}
//        c) A20 = D2 (Z20 + N21 A10);  A31 = D3 (Z31 + N32 A21);  W30 = Z30 + N31 A10
//        d) A30 = D3 (W30 + N32 A20)
// ---------------------------------------------------------------------------
template <int NLD, int AOLD>
__device__ __forceinline__ void invert_unit_lower(float* Nsm, float* Ao, float* Xs, int pw, int lane, int bar_id) {
    if (pw < 2) {
        // diagonal block blk = 2 pw + (lane >> 4); lane j = lane & 15 computes column j of D:
        // x_i = delta_ij + sum_{k<i} N_ik x_k (x_k = 0 for k < j), N rows read as shared-memory
        // broadcasts, no cross-lane exchange
        const int blk = 2 * pw + (lane >> 4), j = lane & 15, row0 = 16 * blk;
        float* nb = Nsm + row0 * NLD + row0;
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float a0 = (i == j) ? 1.f : 0.f, a1 = 0.f;
#pragma unroll
            for (int k4 = 0; k4 < i; k4 += 4) {
                const float4 n4 = *reinterpret_cast<const float4*>(nb + i * NLD + k4);
                a0 = fmaf(n4.x, x[k4], a0);
                if (k4 + 1 < i) a1 = fmaf(n4.y, x[k4 + 1], a1);
                if (k4 + 2 < i) a0 = fmaf(n4.z, x[k4 + 2], a0);
                if (k4 + 3 < i) a1 = fmaf(n4.w, x[k4 + 3], a1);
            }
            x[i] = a0 + a1;
        }
        __syncwarp();                              // every lane has read its block's rows
#pragma unroll
        for (int i = 0; i < 16; ++i) nb[i * NLD + j] = x[i];
    }
    named_bar(bar_id, 128);
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
    named_bar(bar_id, 128);
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
    named_bar(bar_id, 128);
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
    named_bar(bar_id, 128);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ===========================================================================
// Kernel 0: gate vectors of every chunk, one warp per (batch, value head, chunk)
// (prefill_ref.py:49-64, 79-91): g_t = -exp(A_log) softplus(a_t + dt_bias),
// beta_t = sigmoid(b_t) * mask_t, Lambda = in-chunk cumulative sum of g.
// ===========================================================================
template <int DK>
__global__ void __launch_bounds__(128)
prefill_gates_kernel(const GateArgs args) {
    using R = Rec<DK>;
    constexpr float kLog2e = 1.4426950408889634f;
    const int lane = threadIdx.x & 31;
    const int task = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (task >= args.ntasks) return;
    const int bh = task / args.nchunks, c = task - bh * args.nchunks;
    const int h = bh % args.Hv, bidx = bh / args.Hv;
    // valid tokens of this sequence and the offset of its gates (varlen: [Hv, Ttot], packed)
    int start = 0;
    const int T = args.cu ? varlen_seq(args.cu, bidx, args.Ttot, start, args.err) : args.T;
    const long base = args.cu ? static_cast<long>(h) * args.Ttot + start
                              : static_cast<long>(bidx) * args.g_b + static_cast<long>(h) * args.g_h;
    const long gt = args.cu ? 1 : args.g_t;
    const int t0 = 2 * lane;
    const int tok = c * kC + t0;
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f, m0 = 0.f, m1 = 0.f;
    if (tok < T) {
        a0 = load_gate(args.a, base + tok * gt, args.gate_dtype);
        b0 = load_gate(args.b, base + tok * gt, args.gate_dtype);
        m0 = args.mask ? args.mask[static_cast<long>(bidx) * args.gate_ld + tok] : 1.f;
    }
    if (tok + 1 < T) {
        a1 = load_gate(args.a, base + (tok + 1) * gt, args.gate_dtype);
        b1 = load_gate(args.b, base + (tok + 1) * gt, args.gate_dtype);
        m1 = args.mask ? args.mask[static_cast<long>(bidx) * args.gate_ld + tok + 1] : 1.f;
    }
    const float A_neg = -expf(args.A_log[h]);
    const float dtb = args.dt_bias_vec ? args.dt_bias_vec[h] : args.dt_bias;
    float lg0 = 0.f, lg1 = 0.f, bm0 = 0.f, bm1 = 0.f;
    if (tok < T) {
        lg0 = A_neg * softplus_f(a0 + dtb);
        bm0 = sigmoid_f(b0) * m0;
    }
    if (tok + 1 < T) {
        lg1 = A_neg * softplus_f(a1 + dtb);
        bm1 = sigmoid_f(b1) * m1;
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
    uint8_t* rec = args.rec + static_cast<long>(task) * R::BYTES;
    float* g = reinterpret_cast<float*>(rec + R::GB);
    *reinterpret_cast<float2*>(g + G_LAM2 * 64 + t0) = make_float2(l20, l21);
    *reinterpret_cast<float2*>(g + G_U * 64 + t0) = make_float2(ex2_approx(l20 - m2), ex2_approx(l21 - m2));
    *reinterpret_cast<float2*>(g + G_W * 64 + t0) = make_float2(ex2_approx(m2 - l20), ex2_approx(m2 - l21));
    *reinterpret_cast<float2*>(g + G_BM * 64 + t0) = make_float2(bm0, bm1);
    *reinterpret_cast<float2*>(g + G_BME * 64 + t0) = make_float2(bm0 * el0, bm1 * el1);
    *reinterpret_cast<float2*>(g + G_MK * 64 + t0) = make_float2(m0, m1);
    *reinterpret_cast<float2*>(g + G_FLAG * 64 + t0) =
        make_float2(lane == 0 && ll2 < -240.f ? 1.f : 0.f, 0.f);          // u_t * w_s could overflow
    float* G = reinterpret_cast<float*>(rec + R::G);
    *reinterpret_cast<float2*>(G + t0) = make_float2(m0 * args.scale * el0, m1 * args.scale * el1);
    *reinterpret_cast<float2*>(G + 64 + t0) = make_float2(ex2_approx(ll2 - l20), ex2_approx(ll2 - l21));
    if (lane == 0) G[128] = ex2_approx(ll2);                              // gamma_c
    if (args.ready && lane == 0) args.ready[task] = 0;                    // record not prepared yet
}

// ===========================================================================
// Kernel 1: per-chunk preparation, all chunks in parallel
// ===========================================================================
// One prep worker: 128 threads (tid 0..127) with their own shared memory
// (PrepSmem at `sm`, 1024-aligned), 128 TMEM columns and named barrier
// `bar_id`; it takes tasks vblock, vblock + vgrid, ...
template <int DK>
__device__ __forceinline__ void prep_body(const CUtensorMap* map_q, const CUtensorMap* map_k, const PrepArgs& args,
                                          uint8_t* sm, const int tid, const int vblock, const int vgrid,
                                          const int bar_id, const bool relinquish) {
    using L = PrepSmem<DK>;
    using R = Rec<DK>;
    uint64_t* bar_qk = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);      // q/k tiles landed
    uint64_t* bar_qkk = bar_qk + 1;                                        // [Q;K] K^T done
    uint64_t* bar_w = bar_qk + 2;                                          // W^T done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_qk + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* Nsm = reinterpret_cast<float*>(sm + L::OFF_N);
    float* Ao = reinterpret_cast<float*>(sm + L::OFF_AO);
    float* Xs = reinterpret_cast<float*>(sm + L::OFF_XS);
    const float* gates = reinterpret_cast<const float*>(sm + L::OFF_G);

    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int pw = warp;
    const uint32_t lane_off = static_cast<uint32_t>(warp) << 21;
    const bool leader = (tid == 32);                    // MMA/TMA issuer: not on the gate warp
    const int nchunks = args.nchunks;
    const int group = args.Hv / args.Hqk;
    const float scale = args.scale;
    unsigned int* err = args.err;

    if (tid == 0) {
        mbar_init(bar_qk, 1);
        mbar_init(bar_qkk, 1);
        mbar_init(bar_w, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(map_q);
        tma_prefetch_desc(map_k);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kPrepTmemCols);
        if (relinquish) tmem_relinquish();
    }
    tc_fence_before();
    named_bar(bar_id, kPrepThreads);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // task -> (sequence-head bh, chunk c); chunk-major order for the streamed schedule
    auto coords = [&](int task, int& bh, int& c) {
        if (args.chunk_major) {
            const int nbh = args.ntasks / args.ncp;
            const int cc = task / nbh;
            bh = task - cc * nbh;
            c = args.c0 + cc;
        } else {
            bh = task / args.ncp;
            c = args.c0 + (task - bh * args.ncp);
        }
    };
    // varlen: the next task at or after `task` (stride vgrid) inside its sequence's chunks
    auto next_task = [&](int task) {
        if (args.cu)
            for (; task < args.ntasks; task += vgrid) {
                int bh, c;
                coords(task, bh, c);
                int st0;
                if (c < varlen_chunks(varlen_seq(args.cu, bh / args.Hv, args.Ttot, st0, nullptr), nchunks)) break;
            }
        return task;
    };
    // q/k tiles and the gate vectors of `task` -> shared memory, completing on bar_qk
    auto issue_qk = [&](int task) {
        int bh, c;
        coords(task, bh, c);
        const int hq = (bh % args.Hv) / group, bidx = bh / args.Hv;
        // token row and batch coordinates (varlen: packed tokens, one batch)
        int st0 = 0;
        if (args.cu) varlen_seq(args.cu, bidx, args.Ttot, st0, nullptr);
        const int trow = st0 + c * kC, bco = args.cu ? 0 : bidx;
        mbar_arrive_expect_tx(bar_qk, 2 * L::CB * 8192 + kGateBytes);
#pragma unroll
        for (int cb = 0; cb < L::CB; ++cb) {
            tma_load_4d(sm + cb * 16384, map_q, bar_qk, cb * 64, trow, hq, bco);
            tma_load_4d(sm + cb * 16384 + 8192, map_k, bar_qk, cb * 64, trow, hq, bco);
        }
        bulk_load(sm + L::OFF_G, args.rec + (static_cast<long>(bh) * nchunks + c) * R::BYTES + R::GB, kGateBytes,
                  bar_qk);
    };
    const int first = next_task(vblock);
    if (leader && first < args.ntasks) issue_qk(first);

    int it = 0;
    long published = -1;                               // streamed: record whose flag is still to be set
#pragma unroll 1
    for (int task = first; task < args.ntasks; task = next_task(task + vgrid), ++it) {
        const uint32_t ph = it & 1;
        int tbh, tc;
        coords(task, tbh, tc);
        const long rec_idx = static_cast<long>(tbh) * nchunks + tc;
        uint8_t* rec = args.rec + rec_idx * R::BYTES;
        const float* g = gates;                           // this task's gate vectors (landed with q/k)

        // ---- [Q;K] K^T on tensor cores
        mbar_wait_or_abort(bar_qk, ph, err, abort_flag);
        if (leader && !*abort_flag) {
            tc_fence_after();
            const uint32_t sqk = smem_u32(sm);
            constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
#pragma unroll
            for (int kk = 0; kk < DK / 16; ++kk) {
                const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tmem + P_COL_QKK, sdesc_sw128(sqk + o, 16, 1024),
                             sdesc_sw128(sqk + o + 8192, 16, 1024), id64, kk > 0);
            }
            umma_commit(bar_qkk);
        }
        if (leader && args.ready && published >= 0) {
            // streamed: publish the previous task's record once its bulk stores have completed;
            // after this task's MMAs are issued, so that waiting for the stores does not delay them
            bulk_wait_all0();
            if (published != g_unpublished_record) publish_record(args.ready + published);
            published = -1;
        }

        const bool direct = g[G_FLAG * 64] != 0.f;
        mbar_wait_or_abort(bar_qkk, ph, err, abort_flag);
        tc_fence_after();

        // ---- P (lanes 0-63) -> image over the dead q block 0 (bulk-stored to the record),
        //      N (lanes 64-127) -> shared; lower triangle only
        {
            float row[64];
            tmem_ld64(tmem + lane_off + P_COL_QKK, row);
            const float* gw = g + G_W * 64;
            const float* gl2 = g + G_LAM2 * 64;
            if (tid < kC) {
                const int t = tid;
                const float coef = scale * g[G_MK * 64 + t];
                const float cu = coef * g[G_U * 64 + t];
                const float lt = gl2[t];
                uint8_t* prow = sm + L::OFF_A2H;
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
                const int t = tid - kC;
                const float coef = -g[G_BM * 64 + t];
                const float cu = coef * g[G_U * 64 + t];
                const float lt = gl2[t];
                float* nrow = Nsm + t * L::NLD;
                const int send = (t | 15) + 1;             // through the end of t's diagonal block
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
        fence_async_smem();
        tc_fence_before();
        named_bar(bar_id, kPrepThreads);
        if (leader) {
            bulk_store(rec + R::P, sm + L::OFF_A2H, 8192);
            bulk_commit();
        }

        // ---- A = (I - N)^-1
        invert_unit_lower<L::NLD, L::AOLD>(Nsm, Ao, Xs, pw, lane, bar_id);

        // ---- A1 = A diag(beta'), A2 = A diag(beta' e^Lambda), bf16 hi/lo images (rows [t][s]):
        //      computed into registers, then A2 over the q blocks (W MMA operand) and A1 over
        //      N (bulk-stored to the record) once every thread has read N and the off-diagonal blocks
        {
            const int t = tid >> 1, hf = tid & 1;
            const int ib = t >> 4, r = t & 15;
            const float* bm = g + G_BM * 64;
            const float* bme = g + G_BME * 64;
            uint4 h1[4], l1[4], h2[4], l2[4];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const int s0 = 32 * hf + 8 * ch;
                h1[ch] = l1[ch] = h2[ch] = l2[ch] = make_uint4(0u, 0u, 0u, 0u);
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
                    split8(e1, h1[ch], l1[ch]);
                    split8(e2, h2[ch], l2[ch]);
                }
            }
            if (leader) bulk_wait_read0();                // the P image has left the q block
            named_bar(bar_id, kPrepThreads);              // N and the A blocks are no longer read
            uint8_t* a1 = reinterpret_cast<uint8_t*>(Nsm);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const uint32_t off = sw128_chunk(t, 4 * hf + ch);
                *reinterpret_cast<uint4*>(a1 + off) = l1[ch];
                *reinterpret_cast<uint4*>(a1 + 8192 + off) = h1[ch];
                *reinterpret_cast<uint4*>(sm + L::OFF_A2H + off) = h2[ch];
                *reinterpret_cast<uint4*>(sm + L::OFF_A2L + off) = l2[ch];
            }
        }
        fence_async_smem();
        tc_fence_before();
        named_bar(bar_id, kPrepThreads);
        if (leader) {
            bulk_store(rec + R::A1, Nsm, 16384);
            bulk_commit();
        }

        // ---- W^T = K^T A2^T (K as MN-major A, A2 as K-major B), 2 split terms
        if (leader && !*abort_flag) {
            tc_fence_after();
            const uint32_t sk = smem_u32(sm) + 8192;
            constexpr uint32_t id_mn = idesc_bf16(128, 64, true, false);
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const uint32_t b2 = smem_u32(sm + (p ? L::OFF_A2L : L::OFF_A2H));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + P_COL_WT, sdesc_sw128(sk + kk * 2048, 16384, 1024),
                                 sdesc_sw128(b2 + kk * 32, 16, 1024), id_mn, (p > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(bar_w);
        }
        mbar_wait_or_abort(bar_w, ph, err, abort_flag);
        tc_fence_after();

        // ---- W (rows t, columns d) as a K-major tf32 image over the dead q/k tiles -> record;
        //      TMEM row d of W^T is column d of W (a warp stores 128 contiguous bytes per row t)
        if (tid < DK) {
            float row[64];
            tmem_ld64(tmem + lane_off + P_COL_WT, row);
#pragma unroll
            for (int t = 0; t < kC; ++t) *reinterpret_cast<float*>(sm + sw128_f32(t, tid, kC)) = round_tf32(row[t]);
        }
        fence_async_smem();
        tc_fence_before();
        named_bar(bar_id, kPrepThreads);
        bool pending = false;
        if (leader) {
            bulk_store(rec + R::W, sm, DK * 256);
            bulk_commit();
            bulk_wait_read0();                        // the images (and A1 over N) have been read out
            if (args.ready) published = rec_idx;       // published once the next task's q/k have landed
            // q/k shared memory is free: fetch the next task's tiles
            const int nt = next_task(task + vgrid);
            if (!*abort_flag && nt < args.ntasks) {
                issue_qk(nt);
                pending = true;
            }
        }
        named_bar(bar_id, kPrepThreads);
        if (*abort_flag) {
            if (pending) mbar_wait(bar_qk, ph ^ 1u, err);   // let the issued copy land before exiting
            break;
        }
    }

    if (leader) {
        bulk_wait_all0();                              // record stores complete before the worker ends
        if (args.ready && published >= 0 && published != g_unpublished_record) publish_record(args.ready + published);
    }
    tc_fence_before();
    named_bar(bar_id, kPrepThreads);
    if (warp == 0) tmem_dealloc(tmem, kPrepTmemCols);
}

template <int DK>
__global__ void __launch_bounds__(kPrepThreads, kPrepCtasPerSm)
prefill_prep_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const PrepArgs args) {
    extern __shared__ uint8_t smem_raw[];
    prep_body<DK>(&map_q, &map_k, args, align1024(smem_raw), threadIdx.x, blockIdx.x, gridDim.x, BAR_PREP, true);
}

// ===========================================================================
// Kernel 2: the sequential state recurrence, one CTA per (b, h, value tile)
// ===========================================================================
// One chain CTA (all 448 threads), working on (b, h, value tile) number `cta`.
//
// Per chunk c (S^T in TMEM, lane j = value column; buffer c & 1 of [U | O]):
//   U^T  = V^T A1_lo^T + V^T A1_hi^T                    8 bf16 MMAs (N = 64), issued one chunk ahead
//   [U^T | O^T] -= S^T [W^T | -Q~^T]                    DK/8 tf32 MMAs (N = 128), A = the fp32
//                                                       state straight from TMEM, B = [W | -oc Q]
//   state path: dV = U -> bf16 and dV' = dV e^{Lambda_last - Lambda} -> hi/lo;
//               S <- gamma_c S in place
//   S^T += dV'^T K                                      8 bf16 MMAs (hi and lo)
//   O^T += dV^T P^T                                     4 bf16 MMAs, issued after the next
//                                                       chunk's [W | Q~] S; o = O -> bf16 -> TMA store
// The critical path per chunk is [W | Q~] S -> state-path pass -> state update -> the next
// [W | Q~] S; P dV of the previous chunk and U of the next one fill the tensor pipe while
// the state path works, which is why U, O and the bf16 dV are double-buffered in TMEM.
// Barrier arrivals from a group of warps are one per warp (after __syncwarp).
template <int DK>
__device__ __forceinline__ void chain_body(const CUtensorMap* map_q, const CUtensorMap* map_k,
                                           const CUtensorMap* map_v, const CUtensorMap* map_o, const ChainArgs& args,
                                           uint8_t* sm, const int cta) {
    using L = ChainSmem<DK>;
    using R = Rec<DK>;
    constexpr int HALF = DK / 2;                   // key columns per state-path thread group
    constexpr int NBLK = HALF / 32;                // 32-column blocks per group
    ChainBars* bars = reinterpret_cast<ChainBars*>(sm + L::OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int tile = cta % args.ntiles;
    const int bh = cta / args.ntiles;              // b * Hv + h
    const int h = bh % args.Hv;
    const int bidx = bh / args.Hv;
    const int hq = h / (args.Hv / args.Hqk);
    // varlen: this sequence's first token row and length, its own chunk count
    // (single-piece schedule), batch coordinate 0 of the packed tensors
    int trow0 = 0;
    const int seq_len = args.cu ? varlen_seq(args.cu, bidx, args.Ttot, trow0, nullptr) : args.T;
    const int bco = args.cu ? 0 : bidx;
    const int nchunks = args.cu ? varlen_chunks(seq_len, args.nchunks_total) : args.nchunks;
    const int v0 = tile * 128;
    const int dv_valid = min(128, args.dv - v0);
    const int nvb = (dv_valid + 63) / 64;
    unsigned int* err = args.err;
    const int c0 = args.c0;
    const uint8_t* rec0 = args.rec + (static_cast<long>(bh) * args.nchunks_total + c0) * R::BYTES;
    const unsigned int* flags = args.ready ? args.ready + static_cast<long>(bh) * args.nchunks_total + c0 : nullptr;

    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bars->kq_full[s], 1);
            mbar_init(&bars->kq_free[s], 2);       // state-update commit + Q~ warps (q tile read)
        }
        for (int s = 0; s < 3; ++s) {
            mbar_init(&bars->pg_full[s], 1);
            mbar_init(&bars->pg_free[s], 2);       // P dV commit + Q~ warps (gates read)
        }
        mbar_init(&bars->va_full, 1);
        mbar_init(&bars->va_free, 1);
        mbar_init(&bars->w_full, 1);
        mbar_init(&bars->ws_done, 1);
        mbar_init(&bars->dv_done, 8);              // one arrival per state-path warp
        mbar_init(&bars->st_done, 1);
        mbar_init(&bars->pdv_done, 1);
        mbar_init(&bars->qt_ready, 1);
        mbar_init(&bars->o_free, 8);               // one arrival per state-path warp (O read and zeroed)
        mbar_init(&bars->init_done, 8);
        mbar_init(&bars->mma_drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(map_q);
        tma_prefetch_desc(map_k);
        tma_prefetch_desc(map_v);
        tma_prefetch_desc(map_o);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kChainTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto kq_of = [&](int c) { return sm + L::OFF_KQ + (c & 1) * L::KQ_BYTES; };
    auto pg_of = [&](int c) { return sm + L::OFF_PG + (c % 3) * L::PG_BYTES; };
    auto gates_of = [&](int c) { return reinterpret_cast<const float*>(pg_of(c) + L::PG_G); };

    if (warp == 0) {
        // ======================= producer: one thread drives the four streams of copies, polling
        // their barriers without blocking (lanes of one warp spinning on different barriers would
        // take turns); the W rows of the image go first, being on the critical path
        if (lane == 0) {
            uint8_t* img = sm + L::OFF_IMG;
            int nw = 0, nkq = 0, npg = 0, nva = 0;      // next chunk of each stream
            const long long budget = wait_budget();
            long long t_moved = clock64();
            while ((nw < nchunks || nkq < nchunks || npg < nchunks || nva < nchunks) && !*abort_flag) {
                bool moved = false;
                // W rows of the image: chunk nw once [W | Q~] S of chunk nw - 1 has read it
                if (nw < nchunks && (nw == 0 || mbar_test_wait(&bars->ws_done, (nw - 1) & 1)) &&
                    (!flags || record_ready(flags + nw))) {
                    const uint8_t* rec = rec0 + static_cast<long>(nw) * R::BYTES;
                    mbar_arrive_expect_tx(&bars->w_full, DK * 256);
#pragma unroll
                    for (int kb = 0; kb < DK / 32; ++kb)
                        bulk_load(img + kb * 16384, rec + R::W + kb * 8192, 8192, &bars->w_full);
                    // the next chunk's W waits for this chunk's product: bring it into L2 now
                    if (nw + 1 < nchunks && (!flags || ld_relaxed_u32(flags + nw + 1)))
                        bulk_prefetch_l2(rec + R::BYTES + R::W, DK * 256);
                    ++nw;
                    moved = true;
                }
                // q/k ring (inputs, no record): chunk nkq into slot nkq & 1
                if (nkq < nchunks && (nkq < 2 || mbar_test_wait(&bars->kq_free[nkq & 1], ((nkq >> 1) - 1) & 1))) {
                    const int s = nkq & 1;
                    uint8_t* dst = kq_of(nkq);
                    mbar_arrive_expect_tx(&bars->kq_full[s], L::KQ_BYTES);
#pragma unroll
                    for (int cb = 0; cb < L::CB; ++cb) {
                        tma_load_4d(dst + L::KQ_Q + cb * 8192, map_q, &bars->kq_full[s], cb * 64,
                                    trow0 + (c0 + nkq) * kC, hq, bco);
                        tma_load_4d(dst + L::KQ_K + cb * 8192, map_k, &bars->kq_full[s], cb * 64,
                                    trow0 + (c0 + nkq) * kC, hq, bco);
                    }
                    ++nkq;
                    moved = true;
                }
                // P | gates ring: chunk npg into slot npg % 3
                if (npg < nchunks && (npg < 3 || mbar_test_wait(&bars->pg_free[npg % 3], ((npg / 3) - 1) & 1)) &&
                    (!flags || record_ready(flags + npg))) {
                    mbar_arrive_expect_tx(&bars->pg_full[npg % 3], L::PG_BYTES);
                    bulk_load(pg_of(npg), rec0 + static_cast<long>(npg) * R::BYTES + R::P, L::PG_BYTES,
                              &bars->pg_full[npg % 3]);
                    ++npg;
                    moved = true;
                }
                // V tile and A1 (single buffer): chunk nva once U of chunk nva - 1 has read them
                if (nva < nchunks && (nva == 0 || mbar_test_wait(&bars->va_free, (nva - 1) & 1)) &&
                    (!flags || record_ready(flags + nva))) {
                    mbar_arrive_expect_tx(&bars->va_full, nvb * 8192 + 16384);
                    for (int vb = 0; vb < nvb; ++vb)
                        tma_load_4d(sm + L::OFF_V + vb * 8192, map_v, &bars->va_full, v0 + vb * 64,
                                    trow0 + (c0 + nva) * kC, h, bco);
                    bulk_load(sm + L::OFF_A1, rec0 + static_cast<long>(nva) * R::BYTES + R::A1, 16384, &bars->va_full);
                    ++nva;
                    moved = true;
                }
                if (moved) {
                    t_moved = clock64();
                } else if (clock64() - t_moved > budget) {
                    atomicOr(err, DERR_TIMEOUT);
                    *abort_flag = 1;
                }
            }
            // every copy issued lands before the CTA can exit (bounded waits)
            if (nw > 0) mbar_wait(&bars->w_full, (nw - 1) & 1, err);
            for (int c = max(nkq - 2, 0); c < nkq; ++c) mbar_wait(&bars->kq_full[c & 1], (c >> 1) & 1, err);
            for (int c = max(npg - 3, 0); c < npg; ++c) mbar_wait(&bars->pg_full[c % 3], (c / 3) & 1, err);
            if (nva > 0) mbar_wait(&bars->va_full, (nva - 1) & 1, err);
        }
    } else if (warp == 1) {
        // ======================= MMA issuer (one thread)
        if (lane == 0) {
            const uint32_t sv = smem_u32(sm + L::OFF_V);
            const uint32_t sa1 = smem_u32(sm + L::OFF_A1);
            const uint32_t simg = smem_u32(sm + L::OFF_IMG);
            // [U_l^T | U_h^T] of chunk c = V^T [A1_lo^T | A1_hi^T] into buffer c & 1: V as MN-major A,
            // the two A1 parts as one 128-row K-major B
            auto issue_u = [&](int c) {
                const bool ok = mbar_spin_or_abort(&bars->va_full, c & 1, err, abort_flag);
                tc_fence_after();
                if (!ok || *abort_flag) return;
                constexpr uint32_t id_u = idesc_bf16(128, 128, true, false);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + C_BUF + (c & 1) * C_BUF_STRIDE, sdesc_sw128(sv + kk * 2048, 8192, 1024),
                                 sdesc_sw128(sa1 + kk * 32, 16, 1024), id_u, kk > 0 ? 1u : 0u);
                umma_commit(&bars->va_free);
            };
            // O^T += dV^T P^T of chunk c into the O columns of buffer c & 1; frees its P | gates slot
            auto issue_pdv = [&](int c) {
                const bool ok = mbar_spin_or_abort(&bars->pg_full[c % 3], (c / 3) & 1, err, abort_flag);
                tc_fence_after();
                if (!ok || *abort_flag) return;
                constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
                const uint32_t sp = smem_u32(pg_of(c) + L::PG_P);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ts(tmem + C_BUF + (c & 1) * C_BUF_STRIDE + 128,
                                 tmem + C_BUF + (c & 1) * C_BUF_STRIDE + (kk >> 1) * 32 + (kk & 1) * 8,
                                 sdesc_sw128(sp + kk * 32, 16, 1024), id64, 1u);
                umma_commit(&bars->pdv_done);
                umma_commit(&bars->pg_free[c % 3]);
            };
            if (nchunks > 0) issue_u(0);
            mbar_spin_or_abort(&bars->init_done, 0, err, abort_flag);
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c) {
                mbar_spin_or_abort(&bars->w_full, c & 1, err, abort_flag);
                mbar_spin_or_abort(&bars->qt_ready, c & 1, err, abort_flag);
                if (c >= 1) mbar_spin_or_abort(&bars->st_done, (c - 1) & 1, err, abort_flag);
                if (c >= 2) mbar_spin_or_abort(&bars->o_free, c & 1, err, abort_flag);   // O of chunk c - 2 read
                tc_fence_after();
                if (!*abort_flag) {
                    // [U^T | O^T] -= S^T [W^T | -Q~^T]: tf32, A = the fp32 state, B negated
                    constexpr uint32_t id_w = idesc_tf32(128, 128, false, false) | (1u << 14);
#pragma unroll
                    for (int kk = 0; kk < DK / 8; ++kk)
                        umma_tf32_ts(tmem + C_BUF + (c & 1) * C_BUF_STRIDE + 64, tmem + C_X + 8 * kk,
                                     sdesc_sw128(simg + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), id_w, 1u);
                    umma_commit(&bars->ws_done);
                }
                // the tensor pipe is idle while the state path works: P dV of the previous chunk and
                // U of the next one go here
                if (c >= 1) issue_pdv(c - 1);
                if (c + 1 < nchunks) issue_u(c + 1);
                mbar_spin_or_abort(&bars->dv_done, c & 1, err, abort_flag);
                mbar_spin_or_abort(&bars->kq_full[c & 1], (c >> 1) & 1, err, abort_flag);
                tc_fence_after();
                if (!*abort_flag) {
                    // S^T = gamma_c S^T (scaled in place by the state path) + dV'^T K, K as MN-major B;
                    // dV' hi/lo per 32-token half over U_h of buffer c & 1
                    constexpr uint32_t idst = idesc_bf16(128, DK, false, true);
                    const uint32_t dvh = tmem + C_BUF + (c & 1) * C_BUF_STRIDE + 64;
                    const uint32_t sk = smem_u32(kq_of(c) + L::KQ_K);
#pragma unroll
                    for (int p = 0; p < 2; ++p) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_bf16_ts(tmem + C_X, dvh + (kk >> 1) * 32 + p * 16 + (kk & 1) * 8,
                                         sdesc_sw128(sk + kk * 2048, 8192, 1024), idst, 1u);
                    }
                    umma_commit(&bars->st_done);
                    umma_commit(&bars->kq_free[c & 1]);
                }
            }
            if (nchunks > 0) issue_pdv(nchunks - 1);
            // every MMA issued has completed before TMEM is released (also after an abort)
            umma_commit(&bars->mma_drain);
            mbar_wait(&bars->mma_drain, 0, err);
        }
    } else if (warp < 10) {
        // ======================= state path: 256 threads, lane j twice (token half / key half grp)
        const int ct = tid - 64;
        const int grp = ct >> 7;
        const int j = ((warp & 3) << 5) | lane;
        const uint32_t lane_off = static_cast<uint32_t>(warp & 3) << 21;
        const long s_base = static_cast<long>(bh) * DK * args.dv + v0;

        const bool sleader = (ct == 0);
        // ---- o of chunk cc, tokens [32 grp, 32 grp + 32) of value column j: O^T -> bf16 ->
        //      staging image -> TMA store; O is zeroed for chunk cc + 2
        auto store_o = [&](int cc) {
            mbar_wait_or_abort(&bars->pdv_done, cc & 1, err, abort_flag);
            tc_fence_after();
            uint32_t ob2[16];                              // bf16 results, tokens 32 grp + (2i, 2i+1)
            {
                const uint32_t ocol = tmem + lane_off + C_BUF + (cc & 1) * C_BUF_STRIDE + 128 + grp * 32;
                float o[32], z[32];
                tmem_ld32(ocol, o);
#pragma unroll
                for (int i = 0; i < 32; ++i) z[i] = 0.f;
                tmem_ld_wait();
                tmem_st32(ocol, z);
#pragma unroll
                for (int i = 0; i < 16; ++i) ob2[i] = cvt_bf16x2(o[2 * i], o[2 * i + 1]);
                tmem_st_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->o_free);
            // varlen: a sequence's last chunk is stored row by row, only its own tokens (the
            // rows past its end belong to the next sequence); coalesced over the 128 columns
            const int cabs = c0 + cc;
            const bool tail = args.cu && (cabs + 1) * kC > seq_len;
            if (tail && j < dv_valid && !*abort_flag) {
                const int nvalid = seq_len - cabs * kC - 32 * grp;
                uint16_t* orow = args.out + (static_cast<long>(trow0 + cabs * kC + 32 * grp) * args.Hv + h) * args.dv + v0 + j;
                const long ostride = static_cast<long>(args.Hv) * args.dv;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    if (2 * i < nvalid) orow[(2 * i) * ostride] = static_cast<uint16_t>(ob2[i] & 0xffffu);
                    if (2 * i + 1 < nvalid) orow[(2 * i + 1) * ostride] = static_cast<uint16_t>(ob2[i] >> 16);
                }
            }
            if (sleader) bulk_wait_read1();                // the store of two chunks ago left this buffer
            named_bar(BAR_STATE, 256);
            uint8_t* ob = sm + L::OFF_O + (cc & 1) * 16384 + (j >> 6) * 8192;
            const uint32_t jj = j & 63;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t t = 32 * grp + 2 * i;
                *reinterpret_cast<uint16_t*>(ob + sw128_off(t, jj)) = static_cast<uint16_t>(ob2[i] & 0xffffu);
                *reinterpret_cast<uint16_t*>(ob + sw128_off(t + 1, jj)) = static_cast<uint16_t>(ob2[i] >> 16);
            }
            fence_async_smem();
            named_bar(BAR_STATE, 256);
            if (sleader) {
                if (!*abort_flag && !tail)
                    for (int vb = 0; vb < nvb; ++vb)
                        tma_store_4d(map_o, sm + L::OFF_O + (cc & 1) * 16384 + vb * 8192, v0 + vb * 64,
                                     trow0 + cabs * kC, h, bco);
                bulk_commit();
            }
        };

        // initial state -> TMEM (S^T: lane j = value column, column d = key index)
#pragma unroll
        for (int blk = 0; blk < NBLK; ++blk) {
            float vals[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int d = grp * HALF + blk * 32 + i;
                vals[i] = (args.state_in && j < dv_valid) ? args.state_in[s_base + static_cast<long>(d) * args.dv + j]
                                                          : 0.f;
            }
            tmem_st32(tmem + lane_off + C_X + grp * HALF + blk * 32, vals);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->init_done);

#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
            const float* G = gates_of(c);
            mbar_wait_or_abort(&bars->pg_full[c % 3], (c / 3) & 1, err, abort_flag);
            mbar_wait_or_abort(&bars->ws_done, c & 1, err, abort_flag);
            tc_fence_after();
            const float gamma_c = G[128];
            {
                // dV = U_l + U_h (bf16, for P dV) and dV' = dV e^{Lambda_last - Lambda} (hi/lo), tokens
                // [32 grp, 32 grp + 32), written over the U columns this thread has just read
                const uint32_t buf = tmem + lane_off + C_BUF + (c & 1) * C_BUF_STRIDE;
                float ul[32], uh[32];
                tmem_ld32(buf + grp * 32, ul);
                tmem_ld32(buf + 64 + grp * 32, uh);
                tmem_ld_wait();
                const float* edec = G + 64 + grp * 32;
                uint32_t bw[16], hi[16], lo[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float d0 = ul[2 * i] + uh[2 * i], d1 = ul[2 * i + 1] + uh[2 * i + 1];
                    bw[i] = cvt_bf16x2(d0, d1);
                    split2_bf16(d0 * edec[2 * i], d1 * edec[2 * i + 1], hi[i], lo[i]);
                }
                tmem_st16(buf + 64 + grp * 32, hi);
                tmem_st16(buf + 64 + grp * 32 + 16, lo);
                tmem_st16(buf + grp * 32, bw);
            }
            // S <- gamma_c S in place, key columns of half grp ([W | Q~] S has read S)
#pragma unroll
            for (int blk = 0; blk < NBLK; ++blk) {
                float v[32];
                tmem_ld32(tmem + lane_off + C_X + grp * HALF + blk * 32, v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] *= gamma_c;
                tmem_st32(tmem + lane_off + C_X + grp * HALF + blk * 32, v);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->dv_done);
            // the previous chunk's output while the state update and the next [W | Q~] S run
            if (c >= 1) store_o(c - 1);
        }
        if (nchunks > 0) store_o(nchunks - 1);

        // ---- final state -> state_out [dk][dv]
        if (nchunks > 0) mbar_wait_or_abort(&bars->st_done, (nchunks - 1) & 1, err, abort_flag);
        tc_fence_after();
        if (!*abort_flag && args.state_out) {
#pragma unroll
            for (int blk = 0; blk < NBLK; ++blk) {
                float vals[32];
                tmem_ld32(tmem + lane_off + C_X + grp * HALF + blk * 32, vals);
                tmem_ld_wait();
                if (j < dv_valid) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        args.state_out[s_base + static_cast<long>(grp * HALF + blk * 32 + i) * args.dv + j] = vals[i];
                }
            }
        }
        if (sleader) bulk_wait_all0();
    } else {
        // ======================= Q~ warps (4): -Q~ = -oc Q of every chunk into the image
        const int ot = tid - 320;
        const bool oleader = (ot == 0);
        uint8_t* img = sm + L::OFF_IMG;
        {
            // O accumulates from each chunk's [W | Q~] S: both buffers start at zero
            const uint32_t lane_off = static_cast<uint32_t>(warp & 3) << 21;
            float z[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) z[i] = 0.f;
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                tmem_st32(tmem + lane_off + C_BUF + b * C_BUF_STRIDE + 128, z);
                tmem_st32(tmem + lane_off + C_BUF + b * C_BUF_STRIDE + 160, z);
            }
            tmem_st_wait();
            tc_fence_before();
        }
        // rows 64-127 of the image (K-major tf32; the tensor core reads the top 19 bits) for
        // chunk cc, once [W | Q~] S of chunk cc - 1 has read them
#pragma unroll 1
        for (int cc = 0; cc < nchunks; ++cc) {
            const uint8_t* qsrc = kq_of(cc) + L::KQ_Q;
            const float* oc = gates_of(cc);
            mbar_wait_or_abort(&bars->kq_full[cc & 1], (cc >> 1) & 1, err, abort_flag);
            mbar_wait_or_abort(&bars->pg_full[cc % 3], (cc / 3) & 1, err, abort_flag);
            if (cc >= 1) mbar_wait_or_abort(&bars->ws_done, (cc - 1) & 1, err, abort_flag);
            constexpr int CPR = DK / 8;                    // 16-byte bf16 chunks per token row
#pragma unroll
            for (int task = ot; task < kC * CPR; task += 128) {
                const int t = task / CPR, ch = task % CPR;
                const uint4 w = *reinterpret_cast<const uint4*>(qsrc + (ch >> 3) * 8192 + sw128_chunk(t, ch & 7));
                const float s = -oc[t];
                const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
                float f[8];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    f[2 * u] = __uint_as_float(wv[u] << 16) * s;
                    f[2 * u + 1] = __uint_as_float(wv[u] & 0xffff0000u) * s;
                }
                uint8_t* row = img + (ch >> 2) * 16384 + 8192 + t * 128;
                *reinterpret_cast<float4*>(row + ((((2 * ch) & 7) ^ (t & 7)) << 4)) = make_float4(f[0], f[1], f[2], f[3]);
                *reinterpret_cast<float4*>(row + ((((2 * ch + 1) & 7) ^ (t & 7)) << 4)) =
                    make_float4(f[4], f[5], f[6], f[7]);
            }
            fence_async_smem();
            named_bar(BAR_OUT, 128);
            if (oleader) {
                mbar_arrive(&bars->qt_ready);
                mbar_arrive(&bars->kq_free[cc & 1]);       // the q tile has been read
                mbar_arrive(&bars->pg_free[cc % 3]);       // the gates have been read
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kChainTmemCols);
}

template <int DK>
__global__ void __launch_bounds__(kChainThreads, 1)
prefill_chain_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                     const ChainArgs args) {
    extern __shared__ uint8_t smem_raw[];
    chain_body<DK>(&map_q, &map_k, &map_v, &map_o, args, align1024(smem_raw), blockIdx.x);
}

// Shared memory of one overlap CTA: a chain CTA, or kPrepPerCta prep workers.
template <int DK>
struct OverlapSmem {
    static constexpr int PREP_STRIDE = (PrepSmem<DK>::BYTES + 1023) / 1024 * 1024;
    static constexpr int PREP_BYTES = kPrepPerCta * PREP_STRIDE + 1024;
    static constexpr int ALLOC = ChainSmem<DK>::ALLOC > PREP_BYTES ? ChainSmem<DK>::ALLOC : PREP_BYTES;
    static_assert(ALLOC <= 232448, "overlap kernel shared memory exceeds 227 KB");
};

// Chain piece k and prep piece k+1 in one launch: roles [0, nchain) run the
// recurrence over the chunks prepared by the previous launch; every other role
// hosts kPrepPerCta independent prep workers (128 threads each) preparing the
// next piece.  With one CTA per SM the two roles run side by side.
//
// A CTA's role is its block index, or with by_smid its SM id.  Chain and prep
// CTAs on neighbouring SMs slow each other down: with roles by block index
// the prep workers of the streamed schedule ran ~1.5x slower than alone while
// the chain ran, and the step took 13 % longer than with the chain on SMs
// [0, nchain) and prep on the rest.  by_smid is set only for the cooperative
// launch, where every CTA holds its own SM for the whole launch, and applies
// only when the SM ids are exactly [0, gridDim.x) (%nsmid == gridDim.x), so
// the roles are a permutation of the block indices.
template <int DK>
__global__ void __launch_bounds__(kChainThreads, 1)
prefill_overlap_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                       const ChainArgs ca, const PrepArgs pa, const int nchain, const int by_smid) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    int role = static_cast<int>(blockIdx.x);
    if (by_smid) {
        unsigned smid, nsmid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        asm volatile("mov.u32 %0, %%nsmid;" : "=r"(nsmid));
        if (nsmid == gridDim.x) role = static_cast<int>(smid);
    }
    if (role < nchain) {
        chain_body<DK>(&map_q, &map_k, &map_v, &map_o, ca, sm, role);
    } else {
        const int wg = threadIdx.x >> 7;
        if (wg < kPrepPerCta) {
            const int vblock = (role - nchain) * kPrepPerCta + wg;
            const int vgrid = (gridDim.x - nchain) * kPrepPerCta;
            prep_body<DK>(&map_q, &map_k, pa, sm + wg * OverlapSmem<DK>::PREP_STRIDE, threadIdx.x & 127, vblock, vgrid,
                          BAR_PREP + wg, false);
        }
    }
}


std::once_flag g_attr_once[2][64];
int g_attr_status[2][64];
int g_sm_count[64];

constexpr int kMaxPieces = 4;
thread_local int t_schedule = GDN_SCHEDULE_AUTO;   // gdn_prefill_set_schedule: the calling thread's default

// Predicted time (us) of the two schedules, from per-unit costs measured on
// B200 (config-1 shapes): a round of prep tasks takes ~10 us in the prep
// kernel (3 workers per SM) and ~13 us in the overlap kernel, a worker's first
// task ~4 us more; a chain chunk ~2.8 us, a chain launch ~7 us of state
// load/store and pipeline fill.  The pieced schedule wins when the chain is
// long and the sequences few (e.g. a head-sharded long-context prefill), not
// at config 1 where prep rounds, not the chain, would bound each overlap launch.
bool use_pieces(int nbh, int nchunks, int chain_grid, int sms) {
    if (2 * chain_grid > sms || nchunks < 4 * kMaxPieces) return false;
    auto rounds = [](long tasks, long workers) { return static_cast<double>((tasks + workers - 1) / workers); };
    const double prep_round = 10.0, ovl_round = 13.0, first = 4.0, chunk = 2.8, launch = 7.0;
    const long w_all = static_cast<long>(sms) * kPrepCtasPerSm;
    const long w_free = static_cast<long>(sms - chain_grid) * kPrepPerCta;
    const double unpieced = rounds(static_cast<long>(nbh) * nchunks, w_all) * prep_round + first + nchunks * chunk + launch;
    const int per = (nchunks + kMaxPieces - 1) / kMaxPieces;
    double pieced = rounds(static_cast<long>(nbh) * per, w_all) * prep_round + first;
    for (int c0 = 0; c0 < nchunks; c0 += per) {
        const int nc = nchunks - c0 < per ? nchunks - c0 : per;
        const int nn = nchunks - (c0 + nc) < per ? nchunks - (c0 + nc) : per;
        const double ch = nc * chunk + launch;
        const double pr = nn > 0 ? rounds(static_cast<long>(nbh) * nn, w_free) * ovl_round + first : 0.0;
        pieced += ch > pr ? ch : pr;
    }
    return pieced < 0.95 * unpieced;
}

// Predicted time (us) of the streamed schedule when the first `lead` chunks of
// every sequence are prepared by a prep launch on all SMs (~12 us a round of 3
// workers per SM) and the rest by the free SMs' workers inside the cooperative
// launch (~11 us a round, with the roles placed by SM id) while the chain CTAs
// consume them (~3.3 us a chunk): the lead, then the slower of the two
// streams.  Per-unit costs from traces of config 1 on B200 (clock stamps per
// record and per chain chunk); at config 1 it picks no lead, which measured
// fastest of leads 0-32.  The chunk cost is the chain's pace inside the streamed
// launch, where record production sets it; the chain alone (SINGLE) now runs a
// chunk in ~2.2 us.  With these constants the choices match the measured
// schedules: STREAM at config 1 (0.237 ms against 0.286 ms SINGLE), SINGLE for
// the 128-chain head shard of config 4 (2.97 ms against 8.7-12.5 ms streamed).
double streamed_time(int nbh, int nchunks, int chain_grid, int sms, int lead) {
    const long w_all = static_cast<long>(sms) * kPrepCtasPerSm;
    const long w_free = static_cast<long>(sms - chain_grid) * kPrepPerCta;
    const double prep_round = 12.0, ovl_round = 11.0, first = 4.0, chunk = 3.3, launch = 7.0;
    const long t_lead = static_cast<long>(nbh) * lead, t_rest = static_cast<long>(nbh) * (nchunks - lead);
    const double head = lead > 0 ? static_cast<double>((t_lead + w_all - 1) / w_all) * prep_round + first + launch : 0.0;
    const double prep = static_cast<double>((t_rest + w_free - 1) / w_free) * ovl_round + chunk;
    const double chain = first + (lead > 0 ? 0.0 : ovl_round) + nchunks * chunk;
    return head + (prep > chain ? prep : chain) + launch;
}
// The lead (chunks prepared before the cooperative launch) the model likes best.
int stream_lead(int nbh, int nchunks, int chain_grid, int sms) {
    int best = 0;
    double tbest = streamed_time(nbh, nchunks, chain_grid, sms, 0);
    for (int lead = 1; lead < nchunks; ++lead) {
        const double t = streamed_time(nbh, nchunks, chain_grid, sms, lead);
        if (t < tbest) {
            tbest = t;
            best = lead;
        }
    }
    return best;
}
double unpieced_time(int nbh, int nchunks, int sms) {
    const long w_all = static_cast<long>(sms) * kPrepCtasPerSm;
    return static_cast<double>((static_cast<long>(nbh) * nchunks + w_all - 1) / w_all) * 12.0 + 4.0 + nchunks * 3.2 +
           7.0;
}

// The schedule a call runs under the process-wide mode.  The streamed schedule
// needs one free SM besides the chain CTAs (all CTAs co-resident, one per SM);
// the pieced one equal-length sequences.
int pick_schedule(int mode, int nbh, int nchunks, int chain_grid, int sms, bool varlen) {
    const bool can_stream = chain_grid < sms && nchunks >= 2;
    if (mode == GDN_SCHEDULE_STREAM) return can_stream ? GDN_SCHEDULE_STREAM : GDN_SCHEDULE_SINGLE;
    if (mode == GDN_SCHEDULE_PIECED) return (!varlen && nchunks >= 2) ? GDN_SCHEDULE_PIECED : GDN_SCHEDULE_SINGLE;
    if (mode == GDN_SCHEDULE_SINGLE) return GDN_SCHEDULE_SINGLE;
    // STREAM only on a clear predicted win: where the free SMs' prep workers cannot keep up
    // with the chain (a long lead launch does most of the prep), the model is within its
    // error of SINGLE, and the config-4 head shard on 2 GPUs (128 chains, predicted 0.95 of
    // SINGLE) measured 4.0 ms streamed against 3.2 ms single
    if (can_stream &&
        streamed_time(nbh, nchunks, chain_grid, sms, stream_lead(nbh, nchunks, chain_grid, sms)) <
            0.85 * unpieced_time(nbh, nchunks, sms))
        return GDN_SCHEDULE_STREAM;
    if (!varlen && use_pieces(nbh, nchunks, chain_grid, sms)) return GDN_SCHEDULE_PIECED;
    return GDN_SCHEDULE_SINGLE;
}

// The schedule, all on the caller's stream.  Gates (one launch), then prep and
// chain.  When the chain kernel leaves at least half of the SMs idle (few
// sequences), the sequence is cut into up to 4 pieces of chunks:
//   prep(piece 0) -> overlap(chain piece 0 | prep piece 1) -> ... -> chain(last piece)
// with the state carried between chain pieces through `state_tmp`; otherwise
// one prep and one chain launch over all chunks.
template <int DK>
int launch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                   GateArgs ga, PrepArgs pa, ChainArgs ca, int chain_grid, float* state_tmp, unsigned int* ready,
                   int mode, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int which = DK == 128 ? 1 : 0;
    std::call_once(g_attr_once[which][dev & 63], [&]() {
        int sms = 0;
        const bool ok =
            cudaFuncSetAttribute(prefill_prep_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PrepSmem<DK>::ALLOC) == cudaSuccess &&
            cudaFuncSetAttribute(prefill_chain_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ChainSmem<DK>::ALLOC) == cudaSuccess &&
            cudaFuncSetAttribute(prefill_overlap_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 OverlapSmem<DK>::ALLOC) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0;
        g_sm_count[dev & 63] = sms;
        g_attr_status[which][dev & 63] = ok ? GDN_OK : GDN_ERR_CUDA;
    });
    if (g_attr_status[which][dev & 63] != GDN_OK)
        return fail(GDN_ERR_CUDA, "gdn_prefill_fwd: cannot configure the prefill kernels (%d / %d / %d B shared memory)",
                    PrepSmem<DK>::ALLOC, ChainSmem<DK>::ALLOC, OverlapSmem<DK>::ALLOC);
    const int sms = g_sm_count[dev & 63];
    const int nchunks = ca.nchunks_total;
    const int nbh = ga.ntasks / nchunks;                     // B * Hv
    const int sched = pick_schedule(mode, nbh, nchunks, chain_grid, sms, ca.cu != nullptr);
    if (sched == GDN_SCHEDULE_STREAM) ga.ready = ready;

    prefill_gates_kernel<DK><<<(ga.ntasks + 3) / 4, 128, 0, st>>>(ga);
    int s = launch_status("gdn_prefill_fwd (gates)");
    if (s != GDN_OK) return s;

    auto set_piece = [&](int c0, int nc, const float* sin, float* sout, int pc0, int pnc) {
        ca.c0 = c0;
        ca.nchunks = nc;
        ca.state_in = sin;
        ca.state_out = sout;
        pa.c0 = pc0;
        pa.ncp = pnc;
        pa.ntasks = nbh * pnc;
    };
    auto prep_only = [&](int ctas) {
        const int grid = pa.ntasks < ctas ? pa.ntasks : ctas;
        prefill_prep_kernel<DK><<<grid, kPrepThreads, PrepSmem<DK>::ALLOC, st>>>(mq, mk, pa);
        return launch_status("gdn_prefill_fwd (prep)");
    };
    auto chain_only = [&]() {
        prefill_chain_kernel<DK><<<chain_grid, kChainThreads, ChainSmem<DK>::ALLOC, st>>>(mq, mk, mv, mo, ca);
        return launch_status("gdn_prefill_fwd (chain)");
    };
    const float* user_in = ca.state_in;
    float* user_out = ca.state_out;

    if (sched == GDN_SCHEDULE_STREAM) {
        // the first `lead` chunks of every sequence on all SMs (their records published too),
        // then one cooperative launch (all CTAs co-resident: chain CTAs wait on prep workers):
        // chain CTAs over all chunks, prep workers on every other SM for the rest, chunk-major
        const int lead = stream_lead(nbh, nchunks, chain_grid, sms);
        pa.ready = ready;
        if (lead > 0) {
            set_piece(0, 0, nullptr, nullptr, 0, lead);
            if ((s = prep_only(sms * kPrepCtasPerSm)) != GDN_OK) return s;
        }
        set_piece(0, nchunks, user_in, user_out, lead, nchunks - lead);
        pa.chunk_major = 1;
        ca.ready = ready;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(sms);
        cfg.blockDim = dim3(kChainThreads);
        cfg.dynamicSmemBytes = OverlapSmem<DK>::ALLOC;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e =
            cudaLaunchKernelEx(&cfg, prefill_overlap_kernel<DK>, mq, mk, mv, mo, ca, pa, chain_grid, 1);
        if (e != cudaSuccess)
            return fail(GDN_ERR_CUDA, "gdn_prefill_fwd (streamed): cooperative launch of %d CTAs failed: %s", sms,
                        cudaGetErrorString(e));
        return launch_status("gdn_prefill_fwd (streamed)");
    }
    if (sched == GDN_SCHEDULE_SINGLE) {
        set_piece(0, nchunks, user_in, user_out, 0, nchunks);
        if ((s = prep_only(sms * kPrepCtasPerSm)) != GDN_OK) return s;
        return chain_only();
    }
    const int per = (nchunks + kMaxPieces - 1) / kMaxPieces;
    const int pieces = (nchunks + per - 1) / per;
    auto piece_len = [&](int k) { return (nchunks - k * per) < per ? (nchunks - k * per) : per; };
    set_piece(0, 0, nullptr, nullptr, 0, piece_len(0));
    if ((s = prep_only(sms * kPrepCtasPerSm)) != GDN_OK) return s;
    for (int k = 0; k + 1 < pieces; ++k) {
        set_piece(k * per, piece_len(k), k == 0 ? user_in : state_tmp, state_tmp, (k + 1) * per, piece_len(k + 1));
        // chain CTAs first, prep workers on the remaining SMs (at least one CTA of them)
        const int grid = chain_grid + (sms - chain_grid > 1 ? sms - chain_grid : 1);
        prefill_overlap_kernel<DK><<<grid, kChainThreads, OverlapSmem<DK>::ALLOC, st>>>(mq, mk, mv, mo, ca, pa,
                                                                                       chain_grid, 0);
        if ((s = launch_status("gdn_prefill_fwd (overlap)")) != GDN_OK) return s;
    }
    const int kl = pieces - 1;
    set_piece(kl * per, piece_len(kl), kl == 0 ? user_in : state_tmp, user_out, 0, 0);
    return chain_only();
}

// q/k/v/o map: dims (D, T, H, B) innermost first, box (64, 64, 1, 1), 128B swizzle.
// tld: tokens per row of the tensor the map reads (T for a whole tensor; the full
// length when the map covers a token window starting at `base`).
int make_act_map(CUtensorMap* m, const void* base, int D, int T, int H, int B, int layout, long tld = 0) {
    uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(T), static_cast<uint64_t>(H),
                        static_cast<uint64_t>(B)};
    uint64_t strides[3];
    const uint64_t e = 2, L = static_cast<uint64_t>(tld > 0 ? tld : T);
    if (layout == GDN_LAYOUT_BHTD) {
        strides[0] = e * D;                  // T
        strides[1] = e * D * L;              // H
        strides[2] = e * D * L * H;          // B
    } else {
        strides[0] = e * D * H;              // T
        strides[1] = e * D;                  // H
        strides[2] = e * D * H * L;          // B
    }
    uint32_t box[4] = {64, 64, 1, 1};
    return make_map_bf16(m, base, 4, dims, strides, box, true);
}

size_t record_bytes(int dk) { return dk == 128 ? Rec<128>::BYTES : Rec<64>::BYTES; }

}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_launch_count_ex(int B, int T, int Hv, int dk, int dv, int schedule) {
    if (schedule < GDN_SCHEDULE_AUTO || schedule > GDN_SCHEDULE_STREAM) return -1;
    if (B <= 0 || T <= 0 || Hv <= 0 || !(dk == 64 || dk == 128) || !(dv == 64 || dv == 128 || dv == 256)) return -1;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return -1;
    const int nchunks = (T + gdn::kC - 1) / gdn::kC;
    const int nbh = B * Hv, chain_grid = nbh * ((dv + 127) / 128);
    const int sched = gdn::pick_schedule(schedule, nbh, nchunks, chain_grid, sms, false);
    if (sched == GDN_SCHEDULE_STREAM)                     // gates, (lead prep), the cooperative prep + chain launch
        return gdn::stream_lead(nbh, nchunks, chain_grid, sms) > 0 ? 3 : 2;
    if (sched == GDN_SCHEDULE_SINGLE) return 3;
    const int per = (nchunks + gdn::kMaxPieces - 1) / gdn::kMaxPieces;
    return 2 + (nchunks + per - 1) / per;                // gates, prep(piece 0), overlaps, last chain
}

extern "C" int gdn_prefill_launch_count(int B, int T, int Hv, int dk, int dv) {
    return gdn_prefill_launch_count_ex(B, T, Hv, dk, dv, gdn::t_schedule);
}

// Test hooks of the prefill kernels on the current device: the cycle budget of
// their bounded waits (0: the default, ~2^31) and a streamed-schedule record left
// unpublished (-1: none).
extern "C" int gdn_test_prefill_hooks(long long wait_budget_cycles, long long unpublished_record) {
    if (wait_budget_cycles < 0 || unpublished_record < -1)
        return gdn::fail(GDN_ERR_ARG, "gdn_test_prefill_hooks: budget %lld / record %lld out of range",
                         wait_budget_cycles, unpublished_record);
    const long long budget = wait_budget_cycles > 0 ? wait_budget_cycles : (1ll << 31);
    if (cudaMemcpyToSymbol(gdn::g_wait_budget, &budget, sizeof(budget)) != cudaSuccess ||
        cudaMemcpyToSymbol(gdn::g_unpublished_record, &unpublished_record, sizeof(unpublished_record)) != cudaSuccess)
        return gdn::fail(GDN_ERR_CUDA, "gdn_test_prefill_hooks: %s", cudaGetErrorString(cudaGetLastError()));
    return GDN_OK;
}

// The calling host thread's default schedule (other threads keep theirs).
extern "C" int gdn_prefill_set_schedule(int mode) {
    if (mode != GDN_SCHEDULE_AUTO && mode != GDN_SCHEDULE_SINGLE && mode != GDN_SCHEDULE_PIECED &&
        mode != GDN_SCHEDULE_STREAM)
        return gdn::fail(GDN_ERR_ARG, "gdn_prefill_set_schedule: unknown mode %d", mode);
    gdn::t_schedule = mode;
    return GDN_OK;
}

extern "C" size_t gdn_prefill_workspace_bytes(int B, int T, int Hv, int dk, int dv) {
    if (B <= 0 || T <= 0 || Hv <= 0 || !(dk == 64 || dk == 128) || !(dv == 64 || dv == 128 || dv == 256)) return 0;
    const size_t nchunks = (static_cast<size_t>(T) + gdn::kC - 1) / gdn::kC;
    // chunk records, an fp32 state buffer [B, Hv, dk, dv] for the pieced schedule, and one
    // ready flag per record for the streamed schedule
    return static_cast<size_t>(B) * Hv * nchunks * gdn::record_bytes(dk) + static_cast<size_t>(B) * Hv * dk * dv * 4 +
           (static_cast<size_t>(B) * Hv * nchunks * 4 + 127) / 128 * 128;
}

namespace gdn {
namespace {
// Argument checks shared by both prefill entry points (no device access).
int validate_prefill(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                     const void* b_logits, int gate_dtype, const float* state_in, const void* out,
                     const float* state_out, int B, int T, int Hqk, int Hv, int dk, int dv, int layout) {
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
    const long nchunks = (static_cast<long>(T) + kC - 1) / kC;
    if (static_cast<long>(B) * Hv * ntiles > 0x7fffffffL || static_cast<long>(B) * Hv * nchunks > 0x7fffffffL)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_fwd: B*Hv*chunks too large");
    return GDN_OK;
}
}  // namespace
}  // namespace gdn

namespace gdn {
namespace {
// One prefill over B sequences of T tokens, or (cu != null) over B packed
// sequences of at most T tokens each in tensors of Ttot tokens (layout BTHD,
// batch 1), already validated.  gate_ld: elements between rows of a, b_logits
// and mask (0 = T, dense); tld: tokens per row of q, k, v and out (0 = T, dense;
// larger when the call covers a token window of longer tensors).
int run_prefill(const void* q, const void* k, const void* v, const float* A_log, const void* a, const void* b_logits,
                int gate_dtype, float dt_bias, const float* dt_bias_vec, const float* mask, const float* state_in,
                void* out, float* state_out, int B, int T, int Hqk, int Hv, int dk, int dv, int layout, float scale,
                void* workspace, size_t workspace_bytes, void* stream, const int* cu, int Ttot, long gate_ld = 0,
                long tld = 0, int schedule = -1, int gate_layout = GDN_GATES_BHT, long gate_tok_ld = 0) {
    int st = GDN_OK;
    const long ntiles = (dv + 127) / 128;
    const long nchunks = (static_cast<long>(T) + kC - 1) / kC;
    const size_t need = gdn_prefill_workspace_bytes(B, T, Hv, dk, dv);
    if (!workspace || workspace_bytes < need)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_fwd: workspace of %zu B required, %zu B given", need,
                    workspace ? workspace_bytes : static_cast<size_t>(0));
    if ((reinterpret_cast<uintptr_t>(workspace) & 127u) != 0)
        return fail(GDN_ERR_ALIGN, "gdn_prefill_fwd: workspace must be 128-byte aligned");
    st = check_sm100();
    if (st != GDN_OK) return st;
    if (scale == 0.f) scale = 1.f / sqrtf(static_cast<float>(dk));

    // varlen: the packed tensors are one batch of Ttot tokens
    const int mT = cu ? Ttot : T, mB = cu ? 1 : B;
    CUtensorMap mq, mk, mv, mo;
    if ((st = make_act_map(&mq, q, dk, mT, Hqk, mB, layout, tld)) != GDN_OK) return st;
    if ((st = make_act_map(&mk, k, dk, mT, Hqk, mB, layout, tld)) != GDN_OK) return st;
    if ((st = make_act_map(&mv, v, dv, mT, Hv, mB, layout, tld)) != GDN_OK) return st;
    if ((st = make_act_map(&mo, out, dv, mT, Hv, mB, layout, tld)) != GDN_OK) return st;

    GateArgs ga;
    ga.a = a;
    ga.b = b_logits;
    ga.gate_dtype = gate_dtype;
    ga.A_log = A_log;
    ga.dt_bias = dt_bias;
    ga.dt_bias_vec = dt_bias_vec;
    ga.mask = mask;
    ga.rec = static_cast<uint8_t*>(workspace);
    ga.ntasks = static_cast<int>(static_cast<long>(B) * Hv * nchunks);
    ga.T = T;
    ga.Hv = Hv;
    ga.nchunks = static_cast<int>(nchunks);
    ga.scale = scale;
    ga.cu = cu;
    ga.Ttot = mT;
    ga.err = device_error_word();
    ga.ready = nullptr;
    ga.gate_ld = gate_ld > 0 ? gate_ld : T;
    if (gate_layout == GDN_GATES_BTH) {            // [B, T, gate_tok_ld], head h at column h
        ga.g_t = gate_tok_ld;
        ga.g_h = 1;
        ga.g_b = static_cast<long>(T) * gate_tok_ld;
    } else {                                        // [B, Hv, T] rows gate_ld apart
        ga.g_t = 1;
        ga.g_h = ga.gate_ld;
        ga.g_b = static_cast<long>(Hv) * ga.gate_ld;
    }

    PrepArgs pa;
    pa.rec = static_cast<uint8_t*>(workspace);
    pa.err = device_error_word();
    pa.ntasks = ga.ntasks;
    pa.Hqk = Hqk;
    pa.Hv = Hv;
    pa.nchunks = ga.nchunks;
    pa.c0 = 0;
    pa.ncp = ga.nchunks;
    pa.scale = scale;
    pa.cu = cu;
    pa.Ttot = mT;
    pa.ready = nullptr;
    pa.chunk_major = 0;

    ChainArgs ca;
    ca.rec = static_cast<const uint8_t*>(workspace);
    ca.state_in = state_in;
    ca.state_out = state_out;
    ca.err = pa.err;
    ca.T = T;
    ca.Hqk = Hqk;
    ca.Hv = Hv;
    ca.dv = dv;
    ca.ntiles = static_cast<int>(ntiles);
    ca.nchunks_total = static_cast<int>(nchunks);
    ca.c0 = 0;
    ca.nchunks = ca.nchunks_total;
    ca.cu = cu;
    ca.out = static_cast<uint16_t*>(out);
    ca.Ttot = mT;
    ca.ready = nullptr;
    float* state_tmp = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                                static_cast<size_t>(ga.ntasks) * record_bytes(dk));

    const int grid = static_cast<int>(B * Hv * ntiles);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int* ready = reinterpret_cast<unsigned int*>(reinterpret_cast<uint8_t*>(state_tmp) +
                                                          static_cast<size_t>(B) * Hv * dk * dv * 4);
    const int mode = schedule >= 0 ? schedule : t_schedule;
    if (dk == 128) return launch_prefill<128>(mq, mk, mv, mo, ga, pa, ca, grid, state_tmp, ready, mode, s);
    return launch_prefill<64>(mq, mk, mv, mo, ga, pa, ca, grid, state_tmp, ready, mode, s);
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_fwd_ws(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                                  const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                                  const float* mask, const float* state_in, void* out, float* state_out, int B,
                                  int T, int Hqk, int Hv, int dk, int dv, int layout, float scale, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    using namespace gdn;
    const int st = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, B, T, Hqk, Hv,
                                    dk, dv, layout);
    if (st != GDN_OK) return st;
    return run_prefill(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, mask, state_in, out, state_out,
                       B, T, Hqk, Hv, dk, dv, layout, scale, workspace, workspace_bytes, stream, nullptr, 0);
}

// gdn_prefill_fwd_ws with per-call options: the launch schedule and the gate layout
// ([B, Hv, T], or token rows [B, T, gate_ld] read in place).
extern "C" int gdn_prefill_fwd_ex(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                                  const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                                  const float* mask, const float* state_in, void* out, float* state_out, int B,
                                  int T, int Hqk, int Hv, int dk, int dv, int layout, float scale,
                                  const gdn_prefill_opts* opts, void* workspace, size_t workspace_bytes,
                                  void* stream) {
    using namespace gdn;
    const int st = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, B, T, Hqk, Hv,
                                    dk, dv, layout);
    if (st != GDN_OK) return st;
    const int schedule = opts ? opts->schedule : GDN_SCHEDULE_AUTO;
    const int gl = opts ? opts->gate_layout : GDN_GATES_BHT;
    const long gld = opts ? opts->gate_ld : 0;
    if (schedule < GDN_SCHEDULE_AUTO || schedule > GDN_SCHEDULE_STREAM)
        return fail(GDN_ERR_ARG, "gdn_prefill_fwd_ex: unknown schedule %d", schedule);
    if (gl != GDN_GATES_BHT && gl != GDN_GATES_BTH)
        return fail(GDN_ERR_ARG, "gdn_prefill_fwd_ex: unknown gate layout %d", gl);
    if (gl == GDN_GATES_BTH && gld < Hv)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_fwd_ex: gate_ld %ld below Hv=%d", gld, Hv);
    return run_prefill(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, mask, state_in, out, state_out,
                       B, T, Hqk, Hv, dk, dv, layout, scale, workspace, workspace_bytes, stream, nullptr, 0, 0, 0,
                       schedule, gl, gld);
}

namespace gdn {
// gdn_prefill_fwd_ws over gates and mask whose rows are gate_ld elements apart
// (a token segment of wider [B*Hv, T] / [B, T] arrays): the host pipeline's
// per-segment call.
int prefill_segment(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                    const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec, const float* mask,
                    const float* state_in, void* out, float* state_out, int B, int T, int Hqk, int Hv, int dk, int dv,
                    int layout, float scale, void* workspace, size_t workspace_bytes, void* stream, long gate_ld) {
    const int st = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, B, T, Hqk, Hv,
                                    dk, dv, layout);
    if (st != GDN_OK) return st;
    if (gate_ld < T) return fail(GDN_ERR_SHAPE, "prefill segment: gate row stride %ld below T=%d", gate_ld, T);
    return run_prefill(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, mask, state_in, out, state_out,
                       B, T, Hqk, Hv, dk, dv, layout, scale, workspace, workspace_bytes, stream, nullptr, 0, gate_ld);
}
}  // namespace gdn

// Tokens [t0, t0 + Tw) of tensors holding T tokens per sequence: q, k, v, out,
// the gates and the mask are the whole tensors, read and written in place (no
// copies); state_in is the state before token t0, state_out the state after token
// t0 + Tw - 1.  Consecutive windows chained through their states give the whole
// call's result; with window bounds on 64-token chunk boundaries, bit for bit.
extern "C" int gdn_prefill_window_ws(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                                     const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                                     const float* mask, const float* state_in, void* out, float* state_out, int B,
                                     int T, int t0, int Tw, int Hqk, int Hv, int dk, int dv, int layout, float scale,
                                     void* workspace, size_t workspace_bytes, void* stream) {
    using namespace gdn;
    const int st = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, B, T, Hqk, Hv,
                                    dk, dv, layout);
    if (st != GDN_OK) return st;
    if (t0 < 0 || Tw <= 0 || static_cast<long>(t0) + Tw > T)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_window_ws: window [%d, %d + %d) outside T=%d", t0, t0, Tw, T);
    const bool bhtd = layout == GDN_LAYOUT_BHTD;
    const long tq = bhtd ? dk : static_cast<long>(Hqk) * dk;     // elements between tokens
    const long tv = bhtd ? dv : static_cast<long>(Hv) * dv;
    const size_t ge = gate_dtype == GDN_DTYPE_BF16 ? 2 : 4;
    const auto at = [](const void* p, size_t bytes) {
        return static_cast<const void*>(static_cast<const uint8_t*>(p) + bytes);
    };
    return run_prefill(at(q, t0 * tq * 2), at(k, t0 * tq * 2), at(v, t0 * tv * 2), A_log, at(a, t0 * ge),
                       at(b_logits, t0 * ge), gate_dtype, dt_bias, dt_bias_vec, mask ? mask + t0 : nullptr, state_in,
                       static_cast<uint8_t*>(out) + t0 * tv * 2, state_out, B, Tw, Hqk, Hv, dk, dv, layout, scale,
                       workspace, workspace_bytes, stream, nullptr, 0, T, T);
}

// Same call with the workspace taken from the stream-ordered allocator for the
// duration of the call.
extern "C" int gdn_prefill_fwd(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                               const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                               const float* mask, const float* state_in, void* out, float* state_out, int B, int T,
                               int Hqk, int Hv, int dk, int dv, int layout, float scale, void* stream) {
    using namespace gdn;
    int st0 = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, B, T, Hqk, Hv, dk,
                               dv, layout);
    if (st0 != GDN_OK) return st0;
    const size_t need = gdn_prefill_workspace_bytes(B, T, Hv, dk, dv);
    void* ws = nullptr;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (need > 0) {
        const int st = check_sm100();
        if (st != GDN_OK) return st;
        const cudaError_t e = cudaMallocAsync(&ws, need, s);
        if (e != cudaSuccess)
            return fail(GDN_ERR_CUDA, "gdn_prefill_fwd: workspace of %zu B: %s", need, cudaGetErrorString(e));
    }
    const int st = gdn_prefill_fwd_ws(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, mask, state_in,
                                      out, state_out, B, T, Hqk, Hv, dk, dv, layout, scale, ws, need, stream);
    if (ws) cudaFreeAsync(ws, s);
    return st;
}

// ---------------------------------------------------------------------------
// Variable-length prefill: N sequences packed along the token axis, sequence i
// being tokens [cu_seqlens[i], cu_seqlens[i+1]) of q/k/v/out and of the gate
// rows, with its own initial and final state.  Chunks restart at every
// sequence start; a sequence's last chunk is stored row by row so that the
// next sequence's rows are never written.
// ---------------------------------------------------------------------------
extern "C" size_t gdn_prefill_varlen_workspace_bytes(int N, int max_len, int Hv, int dk, int dv) {
    return gdn_prefill_workspace_bytes(N, max_len, Hv, dk, dv);
}

namespace gdn {
namespace {
int validate_varlen(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                    const void* b_logits, int gate_dtype, const int* cu_seqlens, int N, int Ttot, int max_len,
                    const float* state_in, const void* out, const float* state_out, int Hqk, int Hv, int dk, int dv) {
    if (!cu_seqlens) return fail(GDN_ERR_NULL, "gdn_prefill_varlen_fwd: cu_seqlens is required");
    if ((reinterpret_cast<uintptr_t>(cu_seqlens) & 3u) != 0)
        return fail(GDN_ERR_ALIGN, "gdn_prefill_varlen_fwd: cu_seqlens must be 4-byte aligned int32");
    if (N < 1 || Ttot < 1 || max_len < 1 || max_len > Ttot)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_varlen_fwd: need N >= 1 and 1 <= max_len <= Ttot (got N=%d Ttot=%d max_len=%d)",
                    N, Ttot, max_len);
    // tensors: [Ttot, H, D] = layout BTHD with one batch; states [N, Hv, dk, dv]
    const int st = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, 1, Ttot, Hqk,
                                    Hv, dk, dv, GDN_LAYOUT_BTHD);
    if (st != GDN_OK) return st;
    const long nchunks = (static_cast<long>(max_len) + kC - 1) / kC;
    if (static_cast<long>(N) * Hv * nchunks > 0x7fffffffL || static_cast<long>(N) * Hv * ((dv + 127) / 128) > 0x7fffffffL)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_varlen_fwd: N * Hv * chunks exceeds the launch limits");
    return GDN_OK;
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_varlen_fwd_ws(const void* q, const void* k, const void* v, const float* A_log,
                                         const void* a, const void* b_logits, int gate_dtype, float dt_bias,
                                         const float* dt_bias_vec, const int* cu_seqlens, int N, int Ttot, int max_len,
                                         const float* state_in, void* out, float* state_out, int Hqk, int Hv, int dk,
                                         int dv, float scale, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace gdn;
    const int st = validate_varlen(q, k, v, A_log, a, b_logits, gate_dtype, cu_seqlens, N, Ttot, max_len, state_in,
                                   out, state_out, Hqk, Hv, dk, dv);
    if (st != GDN_OK) return st;
    return run_prefill(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, nullptr, state_in, out,
                       state_out, N, max_len, Hqk, Hv, dk, dv, GDN_LAYOUT_BTHD, scale, workspace, workspace_bytes,
                       stream, cu_seqlens, Ttot);
}

extern "C" int gdn_prefill_varlen_fwd(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                                      const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                                      const int* cu_seqlens, int N, int Ttot, int max_len, const float* state_in,
                                      void* out, float* state_out, int Hqk, int Hv, int dk, int dv, float scale,
                                      void* stream) {
    using namespace gdn;
    const int st0 = validate_varlen(q, k, v, A_log, a, b_logits, gate_dtype, cu_seqlens, N, Ttot, max_len, state_in,
                                    out, state_out, Hqk, Hv, dk, dv);
    if (st0 != GDN_OK) return st0;
    const size_t need = gdn_prefill_varlen_workspace_bytes(N, max_len, Hv, dk, dv);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = check_sm100();
    if (st != GDN_OK) return st;
    void* ws = nullptr;
    const cudaError_t e = cudaMallocAsync(&ws, need, s);
    if (e != cudaSuccess)
        return fail(GDN_ERR_CUDA, "gdn_prefill_varlen_fwd: workspace of %zu B: %s", need, cudaGetErrorString(e));
    st = gdn_prefill_varlen_fwd_ws(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, cu_seqlens, N, Ttot,
                                   max_len, state_in, out, state_out, Hqk, Hv, dk, dv, scale, ws, need, stream);
    cudaFreeAsync(ws, s);
    return st;
}

// ---------------------------------------------------------------------------
// Allocation-free prefill, for callers that cannot allocate device memory at
// call time (an engine that reserved the GPU's memory for its own pools, a
// plugin whose host forbids allocation in its execute callback).  The
// workspace is a static device array of kStaticScratchBytes (32 MiB, held on
// every GPU that loads the library), enough for ~540 chunk records at dk=128
// (e.g. B*Hv = 8 sequences of 4096 tokens).  Every record value and the carried
// state are written by a call before that call uses them, so the array's
// contents from the previous call need no clearing; calls that overlap on the
// GPU race on it.
// ---------------------------------------------------------------------------
namespace gdn {
constexpr size_t kStaticScratchBytes = size_t(32) << 20;
static __device__ __align__(256) uint8_t g_prefill_scratch[kStaticScratchBytes];
namespace {
std::once_flag g_scratch_once[64];
void* g_scratch_ptr[64];
int g_scratch_status[64];
}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                                       const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                                       const float* mask, const float* state_in, void* out, float* state_out, int B,
                                       int T, int Hqk, int Hv, int dk, int dv, int layout, float scale, void* stream) {
    using namespace gdn;
    int st = validate_prefill(q, k, v, A_log, a, b_logits, gate_dtype, state_in, out, state_out, B, T, Hqk, Hv, dk,
                              dv, layout);
    if (st != GDN_OK) return st;
    const size_t need = gdn_prefill_workspace_bytes(B, T, Hv, dk, dv);
    if (need > kStaticScratchBytes)
        return fail(GDN_ERR_UNSUPPORTED,
                    "gdn_prefill_fwd_noalloc: this problem needs %zu B of workspace, the static scratch holds %zu B "
                    "(use gdn_prefill_fwd or gdn_prefill_fwd_ws)",
                    need, kStaticScratchBytes);
    if ((st = check_sm100()) != GDN_OK) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(GDN_ERR_CUDA, "gdn_prefill_fwd_noalloc: no current device");
    // once per device, with that device current: the device address of the static
    // scratch (the symbol itself is only a host-side stand-in); this first call
    // should come before any stream capture
    std::call_once(g_scratch_once[dev], [dev]() {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_prefill_scratch);
        g_scratch_ptr[dev] = p;
        g_scratch_status[dev] = (e == cudaSuccess && p != nullptr) ? GDN_OK : GDN_ERR_CUDA;
    });
    if (g_scratch_status[dev] != GDN_OK)
        return fail(GDN_ERR_CUDA, "gdn_prefill_fwd_noalloc: cudaGetSymbolAddress of the static scratch failed");
    return gdn_prefill_fwd_ws(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, mask, state_in, out,
                              state_out, B, T, Hqk, Hv, dk, dv, layout, scale, g_scratch_ptr[dev], kStaticScratchBytes,
                              stream);
}
