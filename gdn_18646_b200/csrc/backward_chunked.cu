// backward_chunked.cu -- the prefill's gradients computed chunk by chunk.
//
// The reference has no backward.  This is the chunked form of the same
// derivative as backward.cu (restated and pinned in oracle
// prefill_backward_chunked): only the state at every chunk start and its
// gradient at every chunk end are carried, never a per-token state.  Per chunk
// of C = 64 tokens, with S the state entering it, Sb the gradient of the state
// leaving it, G_t = prod_{i<=t} g_i (Lambda = log G), b = beta * mask,
// dO' = mask * dO, M = (K K^T) * [G_t/G_s, s < t], P = scale (Q K^T) * [G_t/G_s, s <= t]:
//
//   forward   r_t = G_t (K S)_t + sum_{s<t} M_ts d_s,  d_t = b_t (v_t - r_t),
//             i.e. D = A (b (V - diag(G) K S)) with A = (I + diag(b) M)^-1
//             S <- G_L S + K^T diag(G_L/G) D
//   reverse   X = diag(G_L/G) K Sb + P^T dO'
//             dd_s = X_s - sum_{u>s} M_us b_u dd_u, i.e. dd = A^T X
//             Sb <- G_L Sb + scale (diag(G) Q)^T dO' - (diag(G b) K)^T dd
//   gradients dv = b dd, dr = -b dd, db' = dd . (v - r)
//             dq = scale diag(G) dO' S^T + ((dO' D^T) * P) K
//             dk = diag(G_L/G) D Sb^T + ((dO' D^T) * P)^T Q + ((dr D^T) * M)^T K
//                  + diag(G) dr S^T + ((dr D^T) * M) K
//             g_t dg_t = G_L <S, Sb> + sum_{u>=t} G_u scale q_u.(S dO'_u)
//                  + sum_{u>t} G_u k_u.(S dr_u) + sum_{s<t} (G_L/G_s) k_s.(Sb d_s)
//                  + sum_{s<t<=u} P_us (dO'_u.d_s) + sum_{s<t<u} M_us (dr_u.d_s) + r_t.dr_t
//
// Four launches; every product on tcgen05 (kind::f16, fp32 accumulation in TMEM)
// with fp32 operands split into bf16 hi + lo (hi.hi + hi.lo + lo.hi, relative
// error ~2^-16; q, k, v exact in bf16):
//   cb_mats_kernel      per chunk, all chunks in parallel: the gate vectors, [Q; K] K^T,
//                       P, M and A = (I + diag(b) M)^-1 (16 x 16 diagonal blocks by
//                       substitution, the blocks below by products), written as the
//                       chunk's record: operand images in the shared-memory layout of the
//                       products (k, A, A^T, P^T, scale G q, (m dO)^T, v) and decay tables;
//   cb_chain_kernel     both chunk recurrences at once (one CTA per (b, h) and direction,
//                       one value column of the state per thread in registers): per chunk
//                       three products (K S or K Sb, then A or A^T, then the rank-64 state
//                       update), the record bulk-copied in and prefetched into L2 a chunk
//                       ahead; it stores the state at every chunk start (S) or end (Sb)
//                       and the chunk's d (dd) rows as bf16 hi/lo images, and dv = b dd;
//   cb_grads_tc_kernel  per chunk, persistent: the images bulk-loaded as MN-major
//                       operands of five products ([dO'; dd] S^T, [dO'; dd] D^T, [Q; K] K^T,
//                       [dd; D] Sb^T, and the decay-masked 64 x 64 matrices times k and q),
//                       the per-token scalars of g dg and db' from the same accumulators,
//                       then the gate chain rule into da, db;
//   the head sums of dA_log, ddt_bias (backward.cu's bwd_head_kernel).
#include <type_traits>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {

// the head sums (backward.cu): dA_log[h] = sum dlogg log g, ddt_bias[h] = sum da; a status
int launch_bwd_head_sums(const float* A_log, const void* a, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                         const float* dlogg, const float* da, float* dA_log, float* ddt_bias, int B, int T, int H,
                         cudaStream_t st);

namespace {

constexpr int kCC = 64;                 // chunk length

struct CbArgs {
    const uint16_t* q;                  // [B,H,T,DK] bf16
    const uint16_t* k;
    const uint16_t* v;                  // [B,H,T,DV] bf16
    const float* A_log;                 // [H]
    const void* a;                      // [B,H,T] gate_dtype
    const void* b;
    int gate_dtype;
    float dt_bias;
    const float* dt_bias_vec;           // [H] or null
    const float* mask;                  // [B,T] or null
    const float* state_in;              // [B,H,DK,DV] or null
    const void* dO;                     // [B,H,T,DV] do_dtype
    int do_dtype;
    const float* dS_final;              // [B,H,DK,DV] or null
    float* dq;                          // [B,H,T,DK]
    float* dk;
    float* dv;                          // [B,H,T,DV]
    float* da;                          // [B,H,T]
    float* db;
    float* dstate_in;                   // [B,H,DK,DV] or null
    // workspace, per chunk cid = bh * n + c
    float* gv;                          // [cid][3][64]: Lambda (in-chunk cumulative log g), b, m
    uint8_t* rec;                       // [cid]: the chain kernel's record (CRec)
    uint8_t* ckS;                       // [cid]: the state entering the chunk, S^T image (hi, lo)
    uint8_t* ckD;                       // [cid]: the chunk's d rows as a d^T image (hi, lo; rows v)
    uint8_t* ckSb;                      // [cid]: the gradient of the state leaving it, Sb^T image (hi, lo)
    uint8_t* ckDD;                      // [cid]: the chunk's dd rows as a dd^T image (hi, lo; rows v)
    float* dlogg;                       // [B,H,T]: g dg per token
    unsigned int* err;                  // device error word (bounded waits)
    int B, T, H, n;
    float scale;
};

__device__ __forceinline__ void unpack_bf16x8(const uint4 u, float (&x)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void split_store8(uint8_t* hi, uint8_t* lo, const float (&x)[8]) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) split2_bf16(x[2 * i], x[2 * i + 1], h[i], l[i]);
    *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Per-chunk record for the chain kernel, written by cb_mats_kernel: bf16 images
// in the shared-memory operand layout of the tcgen05 products (K-major, 128-byte
// swizzle, blocks of 64 columns x rows of 128 B), hi/lo pairs for fp32 values, so
// that the chain kernel moves a chunk's operands with bulk copies.  The forward
// role reads [KIMG .. FWD_END), the reverse role KIMG, TAB and [FWD_END .. BYTES).
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct CRec {
    static constexpr int KIMG = 0;                      // k, rows t, DK/64 blocks of 64 rows
    static constexpr int TAB = KIMG + DK * 128;         // tables [5][64] f32: G, G_L/G, b, G b, m
    static constexpr int AH = TAB + 2048;               // A, rows t, columns s (hi, lo)
    static constexpr int AL = AH + 8192;
    static constexpr int VR = AL + 8192;                // v as stored, bf16 [64][DV], rows past T zero
    static constexpr int FWD_END = VR + kCC * DV * 2;
    static constexpr int QGH = FWD_END;                 // scale G_t q_t, rows t (hi, lo)
    static constexpr int QGL = QGH + DK * 128;
    static constexpr int ATH = QGL + DK * 128;          // A^T, rows s, columns u
    static constexpr int ATL = ATH + 8192;
    static constexpr int PTH = ATL + 8192;              // P^T, rows t, columns u
    static constexpr int PTL = PTH + 8192;
    static constexpr int OH = PTL + 8192;               // (m dO)^T, rows v (128, zero past DV), columns u
    static constexpr int OL = OH + 16384;
    static constexpr int BYTES = OL + 16384;
    static constexpr int T_G = 0, T_CF = 64, T_B = 128, T_GB = 192, T_M = 256;   // table rows (floats)
};

// ---------------------------------------------------------------------------
// Per chunk (one CTA of 256 threads): the gate vectors (Lambda, b, m) and the
// chunk's record.  [Q; K] K^T runs on the tensor cores (bf16 q, k, fp32
// accumulate: TMEM lane r < 64 holds row r of Q K^T, lane 64 + t row t of K K^T);
// P = scale (Q K^T) * [G_t/G_s, s <= t]; A = (I + diag(b) M)^-1 with
// M = (K K^T) * [G_t/G_s, s < t]: the four 16 x 16 diagonal blocks by forward
// substitution (one column per thread), then the blocks below them by distance
// from the diagonal, A_ij = -A_ii sum_{j <= k < i} (diag(b) M)_ik A_kj.
// Padded tokens (past T) get log g = 0, b = m = 0 and zero k, q, v, dO.
// ---------------------------------------------------------------------------
// P overlays the [Q; K] image, which is copied into the record as soon as the
// product has read it: at DK = 128 the CTA then takes ~70 KB, three per SM.
template <int DK>
struct MatsSmem {
    static constexpr int QK_KB = 128 * 128;
    static constexpr int OFF_QK = 0;                               // [Q; K] image, 128 rows x DK
    static constexpr int OFF_P = OFF_QK;                           // P           [64][65] fp32, after the product
    static constexpr int QK_END = (DK / 64) * QK_KB > kCC * 65 * 4 ? (DK / 64) * QK_KB : kCC * 65 * 4;
    static constexpr int OFF_L = OFF_QK + QK_END;                  // diag(b) M   [64][65] fp32
    static constexpr int OFF_A = OFF_L + kCC * 65 * 4;             // A           [64][65]
    static constexpr int OFF_T = OFF_A + kCC * 65 * 4;             // block sums  [3][16][17]
    static constexpr int OFF_G = OFF_T + 3 * 16 * 17 * 4;          // Lambda, b, m, Lambda log2(e) [4][64]
    static constexpr int OFF_BAR = OFF_G + 4 * kCC * 4;
    static constexpr int BYTES = OFF_BAR + 16 + 1024;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256) cb_mats_kernel(const CbArgs a) {
    using L = MatsSmem<DK>;
    using R = CRec<DK, DV>;
    constexpr int CPK = DK / 8;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* Ls = reinterpret_cast<float*>(sm + L::OFF_L);
    float* As = reinterpret_cast<float*>(sm + L::OFF_A);
    float* Ps = reinterpret_cast<float*>(sm + L::OFF_P);
    float* Ts = reinterpret_cast<float*>(sm + L::OFF_T);
    float* lam = reinterpret_cast<float*>(sm + L::OFF_G);
    float* bms = lam + kCC;
    float* mks = lam + 2 * kCC;
    float* lam2 = lam + 3 * kCC;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int cid = blockIdx.x, bh = cid / a.n, c = cid - bh * a.n;
    const int h = bh % a.H, bi = bh / a.H;
    const int t0 = c * kCC, nt = min(kCC, a.T - t0);
    const int tid = threadIdx.x, warp = tid >> 5;
    const long tokbase = static_cast<long>(bh) * a.T + t0;
    uint8_t* rec = a.rec + static_cast<long>(cid) * R::BYTES;

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, 64);
        tmem_relinquish();
    }
    {
        constexpr int QN = 128 * CPK / 256;
        uint4 w[QN];
#pragma unroll
        for (int u = 0; u < QN; ++u) {
            const int it = tid + 256 * u, row = it / CPK, ch = it - row * CPK, t = row & (kCC - 1);
            w[u] = t < nt ? __ldg(reinterpret_cast<const uint4*>((row < kCC ? a.q : a.k) + (tokbase + t) * DK + ch * 8))
                          : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < QN; ++u) {
            const int it = tid + 256 * u, row = it / CPK, ch = it - row * CPK;
            *reinterpret_cast<uint4*>(sm + L::OFF_QK + (ch >> 3) * L::QK_KB + sw128_chunk(row, ch & 7)) = w[u];
        }
    }
    float* gv = a.gv + static_cast<long>(cid) * 3 * kCC;
    if (tid < kCC) {
        const int t = tid;
        float lg = 0.f, bm = 0.f, m = 0.f;
        if (t < nt) {
            const long i = tokbase + t;
            const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
            lg = -expf(a.A_log[h]) * softplus_f(load_gate(a.a, i, a.gate_dtype) + dtb);
            m = a.mask ? a.mask[static_cast<long>(bi) * a.T + t0 + t] : 1.f;
            bm = sigmoid_f(load_gate(a.b, i, a.gate_dtype)) * m;
        }
        lam[t] = lg;
        bms[t] = bm;
        mks[t] = m;
        gv[kCC + t] = bm;
        gv[2 * kCC + t] = m;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (tid == 0) {
        constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
        const uint32_t qk = smem_u32(sm + L::OFF_QK);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * L::QK_KB + (kk & 3) * 32;
            umma_bf16_ss(tmem, sdesc_sw128(qk + ko, 16, 1024), sdesc_sw128(qk + ko + kCC * 128, 16, 1024), id64,
                         kk > 0 ? 1u : 0u);
        }
        umma_commit(bar);
    }
    if (warp == 1) {
        // in-chunk cumulative log decay: lane L holds tokens 2L, 2L + 1; inclusive scan over lanes
        const int l = tid & 31;
        const float x0 = lam[2 * l], x1 = lam[2 * l + 1];
        float inc = x0 + x1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, inc, o);
            if (l >= o) inc += y;
        }
        const float c0 = inc - x1;
        lam[2 * l] = c0;
        lam[2 * l + 1] = inc;
        lam2[2 * l] = c0 * 1.4426950408889634f;
        lam2[2 * l + 1] = inc * 1.4426950408889634f;
    }
    // v rows and (m dO)^T as stored: independent of the product
    {
        constexpr int VN = kCC * DV / 8 / 256;
        uint4 w[VN];
#pragma unroll
        for (int u = 0; u < VN; ++u) {
            const int it = tid + 256 * u, t = it / (DV / 8), ch = it - t * (DV / 8);
            w[u] = t < nt ? __ldg(reinterpret_cast<const uint4*>(a.v + (tokbase + t) * DV + ch * 8))
                          : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < VN; ++u) {
            const int it = tid + 256 * u;
            *reinterpret_cast<uint4*>(rec + R::VR + it * 16) = w[u];
        }
    }
    __syncthreads();
    {
        // item (ch, row v): tokens 8 ch .. 8 ch + 7 of value column v; all loads issued first
        const bool bfo = a.do_dtype == GDN_DTYPE_BF16;
        float x[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int it = tid + 256 * u, ch = it >> 7, vr = it & 127;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int tk = ch * 8 + i;
                float d = 0.f;
                if (vr < DV && tk < nt) {
                    const long gi = (tokbase + tk) * DV + vr;
                    d = bfo ? bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(a.dO) + gi))
                            : __ldg(static_cast<const float*>(a.dO) + gi);
                }
                x[u][i] = d;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int it = tid + 256 * u, ch = it >> 7, vr = it & 127;
#pragma unroll
            for (int i = 0; i < 8; ++i) x[u][i] *= mks[ch * 8 + i];
            const uint32_t off = sw128_chunk(vr, ch);
            split_store8(rec + R::OH + off, rec + R::OL + off, x[u]);
        }
    }
    if (tid < kCC) gv[tid] = lam[tid];
    const bool ok = mbar_wait(bar, 0, a.err);
    tc_fence_after();
    // the k and scale G q images of the record, from the [Q; K] image the product has
    // finished reading (P overwrites it next)
    for (int it = tid; it < (DK / 64) * 512; it += 256) {
        const int b = it >> 9, t = (it >> 3) & 63, ch = it & 7;
        const uint4 kq = *reinterpret_cast<const uint4*>(sm + L::OFF_QK + b * L::QK_KB + sw128_chunk(kCC + t, ch));
        *reinterpret_cast<uint4*>(rec + R::KIMG + b * 8192 + sw128_chunk(t, ch)) = kq;
        const uint4 qq = *reinterpret_cast<const uint4*>(sm + L::OFF_QK + b * L::QK_KB + sw128_chunk(t, ch));
        float x[8];
        unpack_bf16x8(qq, x);
        const float gq = a.scale * expf(lam[t]);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] *= gq;
        split_store8(rec + R::QGH + b * 8192 + sw128_chunk(t, ch), rec + R::QGL + b * 8192 + sw128_chunk(t, ch), x);
    }
    __syncthreads();
    if (tid < 128) {
        // row r of the product: P row r (r < 64) or diag(b) M row r - 64
        const int r = tid, t = r & (kCC - 1);
        const float lt2 = lam2[t];
        const float bt = bms[t];
#pragma unroll 1
        for (int cb = 0; cb < kCC; cb += 32) {
            float x[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + cb, x);
            tmem_ld_wait();
            if (!ok) {
#pragma unroll
                for (int i = 0; i < 32; ++i) x[i] = 0.f;
            }
            float* dst = r < kCC ? Ps : Ls;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int s = cb + i;
                const float ex = ex2_approx(lt2 - lam2[s]);   // G_t / G_s
                dst[t * 65 + s] = r < kCC ? (s <= t ? a.scale * x[i] * ex : 0.f) : (s < t ? bt * x[i] * ex : 0.f);
            }
        }
    }
    __syncthreads();
    // diagonal blocks: thread (blk, col) solves column col of (I + L_bb)^-1
    if (tid < kCC) {
        const int blk = tid >> 4, col = tid & 15, o = blk * 16;
        float x[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            float acc = 0.f;
#pragma unroll
            for (int s = 0; s < t; ++s) acc = fmaf(Ls[(o + t) * 65 + o + s], x[s], acc);
            x[t] = t < col ? 0.f : (t == col ? 1.f : -acc);
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) As[(o + t) * 65 + o + col] = x[t];
    }
    for (int e = tid; e < kCC * kCC; e += 256) {      // blocks above the diagonal are zero
        const int r = e >> 6, s = e & 63;
        if ((s >> 4) > (r >> 4)) As[r * 65 + s] = 0.f;
    }
    __syncthreads();
    // below the diagonal, by distance dd from it: T = sum_k L_ik A_kj, then A_ij = -A_ii T
#pragma unroll 1
    for (int dd = 1; dd < 4; ++dd) {
        const int nb = 4 - dd;
        for (int e = tid; e < nb * 256; e += 256) {
            const int jb = e >> 8, rr = (e >> 4) & 15, cc = e & 15, ib = jb + dd;
            float acc = 0.f;
            for (int kb = jb; kb < ib; ++kb)
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    acc = fmaf(Ls[(ib * 16 + rr) * 65 + kb * 16 + q], As[(kb * 16 + q) * 65 + jb * 16 + cc], acc);
            Ts[(jb * 16 + rr) * 17 + cc] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nb * 256; e += 256) {
            const int jb = e >> 8, rr = (e >> 4) & 15, cc = e & 15, ib = jb + dd;
            float acc = 0.f;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                acc = fmaf(As[(ib * 16 + rr) * 65 + ib * 16 + q], Ts[(jb * 16 + q) * 17 + cc], acc);
            As[(ib * 16 + rr) * 65 + jb * 16 + cc] = -acc;
        }
        __syncthreads();
    }
    // the record: A, A^T, P^T (hi/lo), k and scale G q images, tables
    for (int it = tid; it < 3 * 512; it += 256) {
        const int img = it >> 9, row = (it >> 3) & 63, ch = it & 7;
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int cc = ch * 8 + i;
            x[i] = img == 0 ? As[row * 65 + cc] : (img == 1 ? As[cc * 65 + row] : Ps[cc * 65 + row]);
        }
        const uint32_t off = sw128_chunk(row, ch);
        const int hi = img == 0 ? R::AH : (img == 1 ? R::ATH : R::PTH);
        const int lo = img == 0 ? R::AL : (img == 1 ? R::ATL : R::PTL);
        split_store8(rec + hi + off, rec + lo + off, x);
    }
    if (tid < kCC) {
        const int t = tid;
        float* tab = reinterpret_cast<float*>(rec + R::TAB);
        const float G = expf(lam[t]);
        tab[R::T_G + t] = G;
        tab[R::T_CF + t] = expf(lam[kCC - 1] - lam[t]);
        tab[R::T_B + t] = bms[t];
        tab[R::T_GB + t] = G * bms[t];
        tab[R::T_M + t] = mks[t];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------
// The two chunk recurrences in one launch of 2 B H CTAs of 256 threads: CTA
// bh < B H runs the forward recurrence of (b, h), CTA B H + bh the reverse one
// (they are independent).  Threads v and 128 + v share TMEM lane v and value
// column v of the state (S or Sb, fp32; v >= DV holds zeros): each keeps half
// its rows in DK/2 registers and takes half the chunk's tokens in the row passes.
// Per chunk, three tcgen05 rounds with bf16 hi/lo operands, the record of the chunk in shared
// memory (bulk-copied once the previous chunk's last product has completed, and
// prefetched into L2 a chunk ahead):
//   forward  D1 = S^T K^T;  y_t = b_t (v_t - G_t D1_t)  -> D2 = y^T A^T = d^T
//            U = (d diag(G_L/G))^T K;  S <- G_L S + U
//   reverse  D1 = Sb^T K^T, Z = (m dO)^T P;  X_t = (G_L/G_t) D1_t + Z_t
//            D2 = X^T A = dd^T;  U = (-diag(G b) dd)^T K + (m dO)^T diag(scale G) Q
//            Sb <- G_L Sb + U
// storing S (Sb) at every chunk start (end) and the d (dd) rows.
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct ChainSmem {
    using R = CRec<DK, DV>;
    static constexpr int SB = (DK / 64) * 16384;             // state image (hi or lo): 128 rows x DK
    static constexpr int OFF_SH = 0, OFF_SL = SB;
    static constexpr int OFF_XH = 2 * SB, OFF_XL = OFF_XH + 16384;   // 128 rows x 64 tokens
    static constexpr int OFF_REC = OFF_XL + 16384;
    static constexpr int REV_BASE = R::TAB + 2048;           // reverse part of the record in shared memory
    static constexpr int REC_FWD = R::FWD_END, REC_REV = REV_BASE + R::BYTES - R::FWD_END;
    static constexpr int REC = REC_FWD > REC_REV ? REC_FWD : REC_REV;
    static constexpr int OFF_BAR = OFF_REC + REC;
    static constexpr int BYTES = OFF_BAR + 64 + 1024;
    static constexpr int rev(int rec_off) { return REV_BASE + rec_off - R::FWD_END; }
    static_assert(BYTES <= 232448, "shared memory");
};

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) cb_chain_kernel(const CbArgs a) {
    using R = CRec<DK, DV>;
    using L = ChainSmem<DK, DV>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* rs = sm + L::OFF_REC;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);   // [0] record landed, [1] products done
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
    int* dead = reinterpret_cast<int*>(bars + 3);
    const float* tab = reinterpret_cast<const float*>(rs + R::TAB);
    const int BH = a.B * a.H;
    const bool rev = static_cast<int>(blockIdx.x) >= BH;
    const int bh = rev ? blockIdx.x - BH : blockIdx.x;
    // thread (half, v): TMEM lane v (warps w and w + 4 share lanes 32 (w % 4) ..), state
    // columns d in [half DK/2, half DK/2 + DK/2) and tokens [32 half, 32 half + 32)
    const int tid = threadIdx.x, warp = tid >> 5, v = tid & 127, half = tid >> 7;
    constexpr int DH = DK / 2;
    const int d0 = half * DH, t0h = half * 32;
    const bool col_ok = v < DV;
    const uint32_t sbase = smem_u32(sm), rbase = sbase + L::OFF_REC;
    const uint32_t T_D1 = 0, T_Z = 64, T_D2 = 128, T_U = 256;

    auto rec_of = [&](int c) { return a.rec + (static_cast<long>(bh) * a.n + c) * R::BYTES; };
    auto issue = [&](int c) {                      // bulk-copy chunk c's record (thread 0)
        const uint8_t* g = rec_of(c);
        if (!rev) {
            mbar_arrive_expect_tx(&bars[0], R::FWD_END);
            bulk_load(rs, g, R::FWD_END, &bars[0]);
        } else {
            mbar_arrive_expect_tx(&bars[0], L::REV_BASE + R::BYTES - R::FWD_END);
            bulk_load(rs, g, L::REV_BASE, &bars[0]);
            bulk_load(rs + L::REV_BASE, g + R::FWD_END, R::BYTES - R::FWD_END, &bars[0]);
        }
    };
    auto prefetch = [&](int c) {
        const uint8_t* g = rec_of(c);
        if (!rev) {
            bulk_prefetch_l2(g, R::FWD_END);
        } else {
            bulk_prefetch_l2(g, L::REV_BASE);
            bulk_prefetch_l2(g + R::FWD_END, R::BYTES - R::FWD_END);
        }
    };

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        *dead = 0;
        fence_mbar_init();
        issue(rev ? a.n - 1 : 0);
    }
    if (warp == 0) tmem_alloc(tslot, 512);
    float S[DH];
    {
        const float* src = rev ? a.dS_final : a.state_in;
        const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
        for (int d = 0; d < DH; ++d) S[d] = (src && col_ok) ? src[s0 + static_cast<long>(d0 + d) * DV + v] : 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot, lane_t = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint32_t mph = 0;                              // parity of the next products-done phase
    bool ok = true;
    auto mma_wait = [&]() {
        if (!mbar_wait(&bars[1], mph, a.err)) ok = false;
        mph ^= 1u;
        tc_fence_after();
    };
    // columns 32 j .. 32 j + 31 of row v of a 64-column image, split into hi/lo
    auto put32 = [&](uint32_t off_h, uint32_t off_l, int j, const float (&x)[32]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = x[q * 8 + i];
            split_store8(sm + off_h + sw128_chunk(v, 4 * j + q), sm + off_l + sw128_chunk(v, 4 * j + q), y);
        }
    };

#pragma unroll 1
    for (int step = 0; step < a.n; ++step) {
        const int c = rev ? a.n - 1 - step : step;
        const long cid = static_cast<long>(bh) * a.n + c;
        // ---- the state entering (forward) or leaving (reverse) the chunk as a bf16 hi/lo
        //      image (rows v), which is also the checkpoint: bulk-stored for the gradient kernel;
        //      built while the chunk's record is still landing
        {
#pragma unroll
            for (int q = 0; q < DH / 8; ++q) {
                float y[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) y[i] = S[q * 8 + i];
                const int col = d0 + 8 * q;
                const uint32_t off = (col >> 6) * 16384 + sw128_chunk(v, (col & 63) >> 3);
                split_store8(sm + L::OFF_SH + off, sm + L::OFF_SL + off, y);
            }
        }
        if (!mbar_wait(&bars[0], step & 1, a.err)) ok = false;
        if (tid == 0 && step + 1 < a.n) prefetch(rev ? c - 1 : c + 1);
        fence_async_smem();
        __syncthreads();
        const float GL = tab[R::T_G + kCC - 1];
        if (tid == 0) {
            bulk_store((rev ? a.ckSb : a.ckS) + cid * 2 * L::SB, sm + L::OFF_SH, 2 * L::SB);
            bulk_commit();
            tc_fence_after();
            constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
            const uint32_t sh = sbase + L::OFF_SH, sl = sbase + L::OFF_SL, kim = rbase + R::KIMG;
#pragma unroll
            for (int p = 0; p < 2; ++p)
#pragma unroll
                for (int kk = 0; kk < DK / 16; ++kk)
                    umma_bf16_ss(tmem + T_D1, sdesc_sw128((p ? sl : sh) + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                                 sdesc_sw128(kim + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), id64,
                                 (p > 0 || kk > 0) ? 1u : 0u);
            if (rev) {
                const uint32_t oh = rbase + L::rev(R::OH), ol = rbase + L::rev(R::OL);
                const uint32_t ph_ = rbase + L::rev(R::PTH), pl = rbase + L::rev(R::PTL);
                const uint32_t pa[3] = {oh, oh, ol}, pb[3] = {ph_, pl, ph_};
#pragma unroll
                for (int p = 0; p < 3; ++p)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16_ss(tmem + T_Z, sdesc_sw128(pa[p] + kk * 32, 16, 1024),
                                     sdesc_sw128(pb[p] + kk * 32, 16, 1024), id64, (p > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&bars[1]);
        }
        mma_wait();
        // ---- y (forward) or X (reverse) -> the 64-column image
        {
            const int cb = t0h;
            float d1[32], z[32];
            tmem_ld32(lane_t + T_D1 + cb, d1);
            if (rev) tmem_ld32(lane_t + T_Z + cb, z);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int t = cb + i;
                if (!rev) {
                    const float vt = col_ok ? bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(
                                                  rs + R::VR + (t * DV + (col_ok ? v : 0)) * 2))
                                            : 0.f;
                    d1[i] = tab[R::T_B + t] * (vt - tab[R::T_G + t] * d1[i]);
                } else {
                    d1[i] = fmaf(tab[R::T_CF + t], d1[i], z[i]);
                }
            }
            put32(L::OFF_XH, L::OFF_XL, cb >> 5, d1);
        }
        if (tid == 0) bulk_wait_read0();           // the state image may now be overwritten (d / dd image)
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
            const uint32_t xh = sbase + L::OFF_XH, xl = sbase + L::OFF_XL;
            const uint32_t bh_ = rev ? rbase + L::rev(R::ATH) : rbase + R::AH;
            const uint32_t bl_ = rev ? rbase + L::rev(R::ATL) : rbase + R::AL;
            const uint32_t pa[3] = {xh, xh, xl}, pb[3] = {bh_, bl_, bh_};
#pragma unroll
            for (int p = 0; p < 3; ++p)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + T_D2, sdesc_sw128(pa[p] + kk * 32, 16, 1024),
                                 sdesc_sw128(pb[p] + kk * 32, 16, 1024), id64, (p > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&bars[1]);
        }
        mma_wait();
        // ---- d (forward) or dd (reverse): its image over the state image (bulk-stored for the
        //      gradient kernel), dv = b dd (reverse), then the scaled image for the state update
        {
            const int nt = min(kCC, a.T - c * kCC);
            float* dvo = a.dv + (static_cast<long>(bh) * a.T + c * kCC) * DV + v;
            {
                const int cb = t0h;
                float d2[32];
                tmem_ld32(lane_t + T_D2 + cb, d2);
                tmem_ld_wait();
                put32(L::OFF_SH, L::OFF_SH + 16384, cb >> 5, d2);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int t = cb + i;
                    if (rev && col_ok && t < nt) dvo[static_cast<long>(t) * DV] = tab[R::T_B + t] * d2[i];
                    d2[i] = rev ? -tab[R::T_GB + t] * d2[i] : tab[R::T_CF + t] * d2[i];
                }
                put32(L::OFF_XH, L::OFF_XL, cb >> 5, d2);
            }
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            bulk_store((rev ? a.ckDD : a.ckD) + cid * 32768, sm + L::OFF_SH, 32768);
            bulk_commit();
            tc_fence_after();
            constexpr uint32_t idU = idesc_bf16(128, DK, false, true);
            const uint32_t xh = sbase + L::OFF_XH, xl = sbase + L::OFF_XL, kim = rbase + R::KIMG;
#pragma unroll
            for (int p = 0; p < 2; ++p)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + T_U, sdesc_sw128((p ? xl : xh) + kk * 32, 16, 1024),
                                 sdesc_sw128(kim + kk * 2048, 8192, 1024), idU, (p > 0 || kk > 0) ? 1u : 0u);
            if (rev) {
                const uint32_t oh = rbase + L::rev(R::OH), ol = rbase + L::rev(R::OL);
                const uint32_t qh = rbase + L::rev(R::QGH), ql = rbase + L::rev(R::QGL);
                const uint32_t pa[3] = {oh, oh, ol}, pb[3] = {qh, ql, qh};
#pragma unroll
                for (int p = 0; p < 3; ++p)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16_ss(tmem + T_U, sdesc_sw128(pa[p] + kk * 32, 16, 1024),
                                     sdesc_sw128(pb[p] + kk * 2048, 8192, 1024), idU, 1u);
            }
            umma_commit(&bars[1]);
        }
        mma_wait();
        if (tid == 0 && step + 1 < a.n) issue(rev ? c - 1 : c + 1);   // the record is no longer read
        // ---- S <- G_L S + U
#pragma unroll
        for (int cb = 0; cb < DH; cb += 32) {
            float u[32];
            tmem_ld32(lane_t + T_U + d0 + cb, u);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) S[cb + i] = fmaf(GL, S[cb + i], u[i]);
        }
        if (!ok) *dead = 1;
        if (tid == 0) bulk_wait_read0();           // the state image may be rewritten
        tc_fence_before();
        __syncthreads();
        if (*dead) break;
    }
    if (tid == 0) bulk_wait_all0();
    if (rev && col_ok && a.dstate_in && *dead == 0) {
        const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
        for (int d = 0; d < DH; ++d) a.dstate_in[s0 + static_cast<long>(d0 + d) * DV + v] = S[d];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// Per chunk on the tensor cores (one CTA of 256 threads, 512 TMEM columns).
// Every product runs as tcgen05 kind::f16 with fp32 operands split into bf16
// hi + lo (hi.hi + hi.lo + lo.hi; q, k exact in bf16), relative error ~2^-16:
//   T1 = [dO'; dd] S^T      -> lanes 0-63 X_q = dO' S^T, lanes 64-127 X_dd = dd S^T
//   T3 = [dO'; dd] D^T      -> lanes 0-63 dO' D^T,       lanes 64-127 Y = dd D^T
//   T5 = [Q; K] K^T         -> lanes 0-63 Q K^T,         lanes 64-127 K K^T
//   T2 = [dd; D] Sb^T       -> lanes 64-127 X_e = D Sb^T
//   T4 = [F1; F2 + F2^T] K + [0; scale F1^T] Q  (k, q rows of [Q; K] as MN-major operands;
//        F1 = (dO' D^T) * [G_t/G_s, s <= t], F2 = -b (Y * [G_t/G_s, s < t]))
// so that, with TMEM lane = token row (lanes 0-63 the dq side, 64-127 the dk side),
//   dq_t = scale (G_t X_q + T4)_t,   dk_t = (G_L/G_t) X_e - G_t b_t X_dd + T4_{64+t},
// and the per-token scalars of g dg and db' are row dot products of the same
// accumulators: q_t.X_q, k_t.X_dd (= k_t.(S dd_t)), k_t.X_e, the rows of T3 and T5
// against the decay masks, and dd_t.v_t from the staging pass.  Operand images are
// K-major with the 128-byte swizzle, 64 bf16 columns per block:
//   [dO'; dd; D] 192 rows x DV (T1 and T3 read rows 0-127, T2 rows 64-127 and 128-191
//   is D as T3's B operand), S then Sb (DK rows x DV), [Q; K] (128 rows x DK), and
//   after T2 the T4 operands (128 rows x 64 tokens; DK rows x 64 tokens).
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct GtLayout {
    static constexpr int R_BYTES = 3 * 16384;              // [dO'^T | dd^T | d^T] (hi or lo): rows v, 64 t each
    static constexpr int S_BYTES = (DK / 64) * 16384;      // S^T image (hi or lo): rows v (128), DK columns
    static constexpr int QK_KB = 128 * 128;
    static constexpr int QK_BYTES = (DK / 64) * QK_KB;
    static constexpr int OFF_RH = 0, OFF_RL = R_BYTES, OFF_SH = 2 * R_BYTES, OFF_SL = OFF_SH + S_BYTES;
    static constexpr int AB_END = OFF_SL + S_BYTES;
    static constexpr int OFF_A1H = 0, OFF_A1L = 16384, OFF_A2H = 32768, OFF_A2L = 49152;   // after T2
    static constexpr int C_END = 65536;
    static constexpr int OFF_QK = AB_END > C_END ? AB_END : C_END;
    static constexpr int OFF_F = OFF_QK + QK_BYTES;                 // F1 (s <= t), F2 (s < t): packed rows
    static constexpr int OFF_MISC = OFF_F + 4096 * 4;
    static constexpr int MISC_FLOATS = 2048;
    static constexpr int OFF_BAR = OFF_MISC + MISC_FLOATS * 4;
    static constexpr int BYTES = OFF_BAR + 64 + 1024;      // + slack to align the dynamic base to 1024
    static constexpr uint32_t T_XS = 0, T_XE = DK, T_X4 = 2 * DK, T_DD = 3 * DK, T_QK = 3 * DK + 64;
    static_assert(BYTES <= 232448, "shared memory");
    static_assert(T_QK + 64 <= 512, "TMEM columns");
};

// The thread of the gradient kernel that issues its MMAs and bulk copies and waits for them: in
// warp 7, which has no row work, so that issuing never delays the row threads (warps 0-3).
constexpr int kIssuer = 255;

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) cb_grads_tc_kernel(const CbArgs a, int nchunks,
                                                             const __grid_constant__ CUtensorMap map_q,
                                                             const __grid_constant__ CUtensorMap map_k) {
    using L = GtLayout<DK, DV>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* misc = reinterpret_cast<float*>(sm + L::OFF_MISC);
    float* lam = misc;                             // Lambda [64]
    float* Gs = misc + 64;                         // G = e^Lambda
    float* bms = misc + 128;                       // b = beta * mask
    float* ms = misc + 192;                        // mask
    float* ddv = misc + 256;                       // dd_t . v_t
    float* s_a = misc + 320;                       // G_t scale q_t.(S dO'_t)
    float* s_c = misc + 384;                       // G_t k_t.(S dr_t)
    float* s_e = misc + 448;                       // (G_L/G_t) k_t.(Sb d_t)
    float* s_rdr = misc + 512;                     // r_t . dr_t
    float* s_dbm = misc + 576;                     // dd_t . (v_t - r_t)
    float* pairp = misc + 640;                     // [4 warps][64] pair-sum partials
    float* basep = misc + 896;                     // [8 warps] <S, Sb> partials
    int* dead = reinterpret_cast<int*>(misc + 904);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
    // bars: [0] T1/T3/T5 done, [1] T2 done, [2] T4 done, [3] the T image and [Q; K] landed,
    // [4] the S image landed, [5] the Sb image landed; each completes once per chunk
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 6);
    float* F1s = reinterpret_cast<float*>(sm + L::OFF_F);           // row t at t (t + 1) / 2, s <= t
    float* F2s = F1s + kCC * (kCC + 1) / 2;                         // row t at t (t - 1) / 2, s < t
    float* lam2 = misc + 912;                      // Lambda log2(e) [64]
    float* dotp = misc + 1024;                     // [2 halves][128 rows] row dot partials
    float* dep = misc + 1280;                      // [2][128] k . X_e partials
    float* krsp = misc + 1536;                     // [2][128] r . dd partials (the M Y part)
    float* pre32 = misc + 1792;                    // [128] per row: sum of its pair terms over s < 32
    float* dfac = misc + 1920;                     // d(da)/d(g dg) per token: -e^{A_log} sigmoid(a + dt_bias)
    float* dbfac = misc + 1984;                    // d(db)/d(db') per token: mask sigmoid'(b)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = smem_u32(sm);
    // the inputs of chunk cx -> L2 (issued one chunk ahead)
    auto prefetch = [&](int cx) {
        const int bx = cx / a.n, tx0 = (cx - bx * a.n) * kCC, ntx = min(kCC, a.T - tx0);
        const long tb = static_cast<long>(bx) * a.T + tx0;
        bulk_prefetch_l2(a.ckS + static_cast<long>(cx) * 2 * L::S_BYTES, 2 * L::S_BYTES);
        bulk_prefetch_l2(a.ckSb + static_cast<long>(cx) * 2 * L::S_BYTES, 2 * L::S_BYTES);
        bulk_prefetch_l2(a.ckD + static_cast<long>(cx) * 32768, 32768);
        bulk_prefetch_l2(a.ckDD + static_cast<long>(cx) * 32768, 32768);
        bulk_prefetch_l2(a.rec + static_cast<long>(cx) * CRec<DK, DV>::BYTES + CRec<DK, DV>::OH, 32768);
        bulk_prefetch_l2(a.q + tb * DK, ntx * DK * 2);
        bulk_prefetch_l2(a.k + tb * DK, ntx * DK * 2);
        bulk_prefetch_l2(a.v + tb * DV, ntx * DV * 2);
        bulk_prefetch_l2(a.gv + static_cast<long>(cx) * 3 * kCC, 3 * kCC * 4);
    };

    // chunk cx's S^T image -> the S region (issued once the previous chunk's T2 has read it)
    auto load_s = [&](int cx) {
        mbar_arrive_expect_tx(&bars[4], 2 * L::S_BYTES);
        bulk_load(sm + L::OFF_SH, a.ckS + static_cast<long>(cx) * 2 * L::S_BYTES, 2 * L::S_BYTES, &bars[4]);
    };
    // chunk cx's [dO'^T | dd^T | d^T] (hi, lo) -> the T image and its q, k rows (TMA, 128-byte
    // swizzle, rows past T zero) -> the [Q; K] image (issued once the previous chunk's T4 completed)
    auto load_t = [&](int cx) {
        const int bx = cx / a.n, tx0 = (cx - bx * a.n) * kCC;
        const uint8_t* rx = a.rec + static_cast<long>(cx) * CRec<DK, DV>::BYTES;
        const uint8_t* dd = a.ckDD + static_cast<long>(cx) * 32768;
        const uint8_t* d1 = a.ckD + static_cast<long>(cx) * 32768;
        mbar_arrive_expect_tx(&bars[3], 6 * 16384 + 2 * (DK / 64) * 8192);
#pragma unroll
        for (int cb = 0; cb < DK / 64; ++cb) {
            tma_load_3d(sm + L::OFF_QK + cb * L::QK_KB, &map_q, &bars[3], cb * 64, tx0, bx);
            tma_load_3d(sm + L::OFF_QK + cb * L::QK_KB + kCC * 128, &map_k, &bars[3], cb * 64, tx0, bx);
        }
        bulk_load(sm + L::OFF_RH, rx + CRec<DK, DV>::OH, 16384, &bars[3]);
        bulk_load(sm + L::OFF_RL, rx + CRec<DK, DV>::OL, 16384, &bars[3]);
        bulk_load(sm + L::OFF_RH + 16384, dd, 16384, &bars[3]);
        bulk_load(sm + L::OFF_RL + 16384, dd + 16384, 16384, &bars[3]);
        bulk_load(sm + L::OFF_RH + 32768, d1, 16384, &bars[3]);
        bulk_load(sm + L::OFF_RL + 32768, d1 + 16384, 16384, &bars[3]);
    };

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        mbar_init(&bars[3], 1);
        mbar_init(&bars[4], 1);
        mbar_init(&bars[5], 1);
        *dead = 0;
        fence_mbar_init();
        if (static_cast<int>(blockIdx.x) < nchunks) {
            load_s(blockIdx.x);
            load_t(blockIdx.x);
            if (static_cast<int>(blockIdx.x + gridDim.x) < nchunks) prefetch(blockIdx.x + gridDim.x);
        }
    }
    if (warp == 0) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    uint32_t ph = 0;                               // barrier parity of this CTA's current chunk
#pragma unroll 1
    for (int cid = blockIdx.x; cid < nchunks; cid += gridDim.x, ph ^= 1u) {
    const int bh = cid / a.n, c = cid - bh * a.n;
    const int h = bh % a.H;
    const int t0 = c * kCC, nt = min(kCC, a.T - t0);
    const long tokbase = static_cast<long>(bh) * a.T + t0;
    const uint8_t* ckS = a.ckS + static_cast<long>(cid) * 2 * L::S_BYTES;
    const uint8_t* ckSb = a.ckSb + static_cast<long>(cid) * 2 * L::S_BYTES;
    const uint8_t* rec = a.rec + static_cast<long>(cid) * CRec<DK, DV>::BYTES;
    const int next = cid + static_cast<int>(gridDim.x);   // this CTA's next chunk
    if (tid == kIssuer && next + static_cast<int>(gridDim.x) < nchunks) prefetch(next + gridDim.x);
    // ---- phase A: the images of this chunk (issued during the previous one) land on bars[3],
    //      bars[4]; T1, T3, T5 go to the tensor pipe before the chunk's gate loads
    const uint32_t rh = sbase + L::OFF_RH, rl = sbase + L::OFF_RL, sh = sbase + L::OFF_SH, sl = sbase + L::OFF_SL;
    if (tid == kIssuer) {
        if (!mbar_wait(&bars[4], ph, a.err) || !mbar_wait(&bars[3], ph, a.err)) *dead = 1;
        tc_fence_after();
        // Every operand here is MN-major (rows v of the images, 16 rows per K step): A = the
        // [dO'^T | dd^T] blocks (M = 128 tokens, next 64 at 16 KB), B = the S^T image (N = d)
        // or the d^T block (N = 64 tokens)
        constexpr uint32_t idN = idesc_bf16(128, DK, true, true);
        constexpr uint32_t id64 = idesc_bf16(128, 64, true, true);
        const uint32_t pa[3] = {rh, rh, rl}, pbs[3] = {sh, sl, sh}, pbd[3] = {rh, rl, rh};
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int kk = 0; kk < DV / 16; ++kk) {
                const uint32_t acc = (p > 0 || kk > 0) ? 1u : 0u;
                umma_bf16_ss(tmem + L::T_XS, sdesc_sw128(pa[p] + kk * 2048, 16384, 1024),
                             sdesc_sw128(pbs[p] + kk * 2048, 16384, 1024), idN, acc);
                umma_bf16_ss(tmem + L::T_DD, sdesc_sw128(pa[p] + kk * 2048, 16384, 1024),
                             sdesc_sw128(pbd[p] + 32768 + kk * 2048, 16384, 1024), id64, acc);
            }
        // [Q; K] K^T: both operands K-major
        constexpr uint32_t id64k = idesc_bf16(128, 64, false, false);
        const uint32_t qk = sbase + L::OFF_QK;
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * L::QK_KB + (kk & 3) * 32;
            umma_bf16_ss(tmem + L::T_QK, sdesc_sw128(qk + ko, 16, 1024), sdesc_sw128(qk + ko + kCC * 128, 16, 1024),
                         id64k, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[0]);
    }

    if (tid < kCC) {
        const float* gv = a.gv + static_cast<long>(cid) * 3 * kCC;
        // the gate chain-rule factors of the chunk's tokens, loaded with the gate vectors so
        // that the token sums at the end of the chunk read no global memory
        float xg = 0.f, xb = 0.f;
        if (tid < nt) {
            const long tok = tokbase + tid;
            xg = load_gate(a.a, tok, a.gate_dtype) + (a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias);
            xb = load_gate(a.b, tok, a.gate_dtype);
        }
        const float g0 = gv[tid], m0 = gv[2 * kCC + tid];
        lam[tid] = g0;
        lam2[tid] = g0 * 1.4426950408889634f;
        Gs[tid] = expf(g0);
        bms[tid] = gv[kCC + tid];
        ms[tid] = m0;
        dfac[tid] = -expf(a.A_log[h]) * (xg > 20.f ? 1.f : sigmoid_f(xg));
        const float sb = sigmoid_f(xb);
        dbfac[tid] = m0 * sb * (1.f - sb);
    }
    __syncthreads();

    // ---- phase B: dd . v while T1, T3, T5 run (the T image has landed), then the Sb^T image
    //      over the S image once T1 has read it, <S, Sb>, then T2
    if (!mbar_wait(&bars[3], ph, a.err)) *dead = 1;
    {
        // dd_t . v_t: four threads per token, 32 value columns each, dd from the image (hi + lo)
        const int t = tid & (kCC - 1), qv = tid >> 6;
        float pv = 0.f;
        if (t < nt && qv * 32 < DV) {
            const uint16_t* vr = a.v + (tokbase + t) * DV + qv * 32;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float v8[8];
                unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(vr) + j), v8);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int vv = qv * 32 + j * 8 + i;
                    const uint32_t o = 16384 + sw128_off(vv, t);
                    pv = fmaf(bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sm + L::OFF_RH + o)) +
                                  bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sm + L::OFF_RL + o)),
                              v8[i], pv);
                }
            }
        }
        pairp[qv * kCC + t] = pv;                   // pairp is free until the row work below
    }
    float sp = 0.f;
    {
        // <S, Sb> over the images: S (hi, lo) from memory (in L2; loaded while T1 runs), Sb
        // from shared memory once T1 has read the S image it replaces
        constexpr int NQ = 2 * L::S_BYTES / 2 / 16 / 256;     // uint4 of one image (hi or lo) per thread
        uint4 shv[NQ], slv[NQ];
#pragma unroll
        for (int u = 0; u < NQ; ++u) {
            const int q = tid + 256 * u;
            shv[u] = __ldg(reinterpret_cast<const uint4*>(ckS) + q);
            slv[u] = __ldg(reinterpret_cast<const uint4*>(ckS + L::S_BYTES) + q);
        }
        if (!mbar_wait(&bars[0], ph, a.err)) *dead = 1;
        tc_fence_after();
        if (tid == kIssuer) {
            mbar_arrive_expect_tx(&bars[5], 2 * L::S_BYTES);
            bulk_load(sm + L::OFF_SH, ckSb, 2 * L::S_BYTES, &bars[5]);
        }
        if (!mbar_wait(&bars[5], ph, a.err)) *dead = 1;
#pragma unroll
        for (int u = 0; u < NQ; ++u) {
            const int q = tid + 256 * u;
            float a8[8], b8[8], c8[8], d8[8];
            unpack_bf16x8(shv[u], a8);
            unpack_bf16x8(slv[u], b8);
            unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + L::OFF_SH + q * 16), c8);
            unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + L::OFF_SL + q * 16), d8);
#pragma unroll
            for (int i = 0; i < 8; ++i) sp = fmaf(a8[i] + b8[i], c8[i] + d8[i], sp);
        }
    }
    sp = warp_sum(sp);
    if (lane == 0) basep[warp] = sp;
    __syncthreads();
    if (tid < kCC) ddv[tid] = pairp[tid] + pairp[kCC + tid] + pairp[2 * kCC + tid] + pairp[3 * kCC + tid];
    fence_async_smem();
    __syncthreads();
    const bool dead_b = *dead != 0;
    if (tid == kIssuer && !dead_b) {
        tc_fence_after();
        constexpr uint32_t idN = idesc_bf16(128, DK, true, true);
        const uint32_t pa[3] = {rh, rh, rl}, pbs[3] = {sh, sl, sh};
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int kk = 0; kk < DV / 16; ++kk) {
                umma_bf16_ss(tmem + L::T_XE, sdesc_sw128(pa[p] + 16384 + kk * 2048, 16384, 1024),
                             sdesc_sw128(pbs[p] + kk * 2048, 16384, 1024), idN, (p > 0 || kk > 0) ? 1u : 0u);
            }
        umma_commit(&bars[1]);
    }
    const float scale = a.scale;
    const float lL = lam[kCC - 1], GL = Gs[kCC - 1];
    // row work on all 8 warps: thread (hf, r) = TMEM lane r (warps w and w + 4 share lanes
    // 32 (w % 4) ..), token t = r % 64, side = r / 64; half hf takes half the columns of the
    // row dot products and the tokens s in [32 hf, 32 hf + 32) of the decay-masked rows
    if (!dead_b) {
        const int hf = tid >> 7, r = tid & 127, t = r & (kCC - 1), side = r >> 6;
        const uint32_t lb = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
        // row r of an accumulator (columns [hf DK/2, hf DK/2 + DK/2)) against row r of [Q; K]
        auto row_dot = [&](uint32_t col0) {
            float acc = 0.f;
#pragma unroll 1
            for (int cb = hf * (DK / 2); cb < (hf + 1) * (DK / 2); cb += 32) {
                float x[32];
                tmem_ld32(lb + col0 + cb, x);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col = cb + 8 * j;
                    float y[8];
                    unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + L::OFF_QK + (col >> 6) * L::QK_KB +
                                                                  sw128_chunk(r, (col & 63) >> 3)),
                                  y);
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc = fmaf(x[8 * j + i], y[i], acc);
                }
            }
            return acc;
        };
        // q_t . X_q (side 0) or k_t . X_dd (side 1); k_t . X_e (side 1) comes last, so that
        // T2 runs in the tensor pipe during the decay-masked rows
        dotp[hf * 128 + r] = row_dot(L::T_XS);
        const float lt2 = lam2[t], bt = bms[t];
        float* Fs = side ? F2s + t * (t - 1) / 2 : F1s + t * (t + 1) / 2;
        float pre = 0.f, krs = 0.f;
        float cv[32];                               // this row's contribution to each token's pair sum
        {
            const int cb = hf * 32;
            float x[32], y[32];
            tmem_ld32(lb + L::T_DD + cb, x);        // dO' D^T row (side 0) or Y = dd D^T row (side 1)
            tmem_ld32(lb + L::T_QK + cb, y);        // Q K^T row or K K^T row
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int s = cb + i;
                const float ex = ex2_approx(lt2 - lam2[s]);   // G_t / G_s
                float f, e;
                bool in;
                if (side == 0) {
                    in = s <= t;
                    f = in ? x[i] * ex : 0.f;       // F1
                    e = scale * y[i] * f;           // P_ts (dO'_t . d_s)
                } else {
                    in = s < t;
                    const float my = in ? y[i] * ex * x[i] : 0.f;   // M_ts (dd_t . d_s)
                    krs += my;
                    f = in ? -bt * x[i] * ex : 0.f; // F2
                    e = -bt * my;                   // M_ts (dr_t . d_s)
                }
                if (in) Fs[s] = f;
                // pair sums: token s gets sum_{s' < s} e_{s'} from rows u >= s (side 0) or u > s
                // (side 1); the second half's prefix starts at zero, and the first half's row
                // totals (pre32) are added back per token after the reduction
                cv[i] = in ? pre : 0.f;
                pre += e;
            }
        }
        if (hf == 0) pre32[r] = pre;
        krsp[hf * 128 + r] = krs;
        // sum cv over the warp's 32 rows by a butterfly reduce-scatter: after the stage of lane
        // bit o a lane keeps the half of its values selected by that bit, so lane L ends with
        // the sum for token 32 hf + L
#pragma unroll
        for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; ++i) {
                const float send = up ? cv[i] : cv[i + n / 2];
                const float keep = up ? cv[i + n / 2] : cv[i];
                cv[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        pairp[(warp & 3) * kCC + hf * 32 + lane] = cv[0];
        if (side == 1) {
            if (!mbar_wait(&bars[1], ph, a.err)) *dead = 1;
            tc_fence_after();
            dep[hf * 128 + r] = row_dot(L::T_XE);
        }
    }
    __syncthreads();
    if (tid < 128 && !dead_b) {
        const int r = tid, t = r & (kCC - 1), side = r >> 6;
        const float Gt = Gs[t], bt = bms[t];
        const float dot = dotp[r] + dotp[128 + r];
        if (side == 0) {
            s_a[t] = Gt * scale * dot;
        } else {
            const float kr = Gt * dot + krsp[r] + krsp[128 + r];   // r_t . dd_t
            s_c[t] = -Gt * bt * dot;
            s_dbm[t] = ddv[t] - kr;
            s_rdr[t] = -bt * kr;
            s_e[t] = expf(lL - lam[t]) * (dep[r] + dep[128 + r]);
        }
    }

    // ---- phase C: the T4 operands over the freed images once T2 completed
    if (tid == kIssuer && !dead_b) {
        if (!mbar_wait(&bars[1], ph, a.err)) *dead = 1;
        else if (next < nchunks) load_s(next);     // T2 has read the S region
    }
    __syncthreads();
    const bool dead_c = *dead != 0;
    tc_fence_after();
    if (!dead_c) {
        // thread (half, row): row `row` of A1 and A2, column chunks 4 half .. 4 half + 3; the
        // token s of every element is a constant of the unrolled loops, so the transposed
        // reads (F2 row s, F1 row s at column t) take immediate offsets
        const int row = tid & 127, t = row & (kCC - 1);
        auto build = [&](auto half_c) {
            constexpr int H4 = decltype(half_c)::value * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int ch = H4 + q;
                float f1[8], f2[8];
                if (row < kCC) {
                    const float* fr = F1s + t * (t + 1) / 2;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int s = ch * 8 + i;
                        f1[i] = s <= t ? fr[s] : 0.f;
                        f2[i] = 0.f;
                    }
                } else {
                    const float* fr = F2s + t * (t - 1) / 2;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int s = ch * 8 + i;
                        const float lower = fr[s < t ? s : 0];                                  // F2[t][s], s < t
                        const float upper = F2s[s * (s - 1) / 2 + (t < s ? t : 0)];             // F2[s][t], s > t
                        f1[i] = s < t ? lower : (s > t ? upper : 0.f);
                        f2[i] = s >= t ? scale * F1s[s * (s + 1) / 2 + (t <= s ? t : 0)] : 0.f;   // F1[s][t]
                    }
                }
                const uint32_t off = sw128_chunk(row, ch);
                split_store8(sm + L::OFF_A1H + off, sm + L::OFF_A1L + off, f1);
                split_store8(sm + L::OFF_A2H + off, sm + L::OFF_A2L + off, f2);
            }
        };
        if (tid < 128) build(std::integral_constant<int, 0>());
        else build(std::integral_constant<int, 1>());
    }
    fence_async_smem();
    __syncthreads();
    if (tid == kIssuer && !dead_c) {
        tc_fence_after();
        constexpr uint32_t idN = idesc_bf16(128, DK, false, true);
        const uint32_t pa[4] = {sbase + L::OFF_A1H, sbase + L::OFF_A1L, sbase + L::OFF_A2H, sbase + L::OFF_A2L};
        // B = the k rows (8 KB into each 16 KB block of [Q; K]) or the q rows, MN-major (N = d)
        const uint32_t qk = sbase + L::OFF_QK;
        const uint32_t pb[4] = {qk + kCC * 128, qk + kCC * 128, qk, qk};
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_bf16_ss(tmem + L::T_X4, sdesc_sw128(pa[p] + kk * 32, 16, 1024),
                             sdesc_sw128(pb[p] + kk * 2048, L::QK_KB, 1024), idN, (p > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars[2]);
    }
    __syncthreads();
    if (tid < kCC && tid < nt && !dead_c) {
        const int t = tid;
        float base = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) base += basep[w];
        float sa = 0.f, scc = 0.f, se = 0.f;
#pragma unroll
        for (int u = 0; u < kCC; ++u) {            // masked sums, fully unrolled: all loads in flight
            sa += u >= t ? s_a[u] : 0.f;
            scc += u > t ? s_c[u] : 0.f;
            se += u < t ? s_e[u] : 0.f;
        }
        float pair = pairp[t] + pairp[kCC + t] + pairp[2 * kCC + t] + pairp[3 * kCC + t];
        if (t >= 32) {                             // the first half's row totals, rows u >= t / u > t
#pragma unroll
            for (int u = 32; u < kCC; ++u) pair += (u >= t ? pre32[u] : 0.f) + (u > t ? pre32[kCC + u] : 0.f);
        }
        const float dlogg = GL * base + sa + scc + se + pair + s_rdr[t];
        const long tok = tokbase + t;
        a.dlogg[tok] = dlogg;
        a.da[tok] = dlogg * dfac[t];
        a.db[tok] = s_dbm[t] * dbfac[t];
    }

    // ---- phase D: dq, dk (warps w and w + 4 share lanes 32 (w % 4) .. + 31, half the columns each)
    if (tid == kIssuer && !dead_c) {
        if (!mbar_wait(&bars[2], ph, a.err)) *dead = 1;
        else if (next < nchunks) load_t(next);     // T4 has read the T image, A1, A2 and [Q; K]
    }
    __syncthreads();
    tc_fence_after();
    if (*dead == 0) {
        const int wq = warp & 3, r = wq * 32 + lane, t = r & (kCC - 1), side = r >> 6;
        const uint32_t lb = tmem + (static_cast<uint32_t>(wq * 32) << 16);
        const float Gt = Gs[t], GLt = expf(lL - lam[t]), gb = Gt * bms[t];
        const int c0 = (warp >> 2) * (DK / 2);
#pragma unroll 1
        for (int cb = c0; cb < c0 + DK / 2; cb += 32) {
            float x1[32], x4[32], x2[32];
            tmem_ld32(lb + L::T_XS + cb, x1);
            tmem_ld32(lb + L::T_X4 + cb, x4);
            tmem_ld32(lb + L::T_XE + cb, x2);
            tmem_ld_wait();
            if (t < nt) {
                float* dst = (side ? a.dk : a.dq) + (tokbase + t) * DK + cb;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        o[j] = side ? fmaf(GLt, x2[i + j], fmaf(-gb, x1[i + j], x4[i + j]))
                                    : scale * fmaf(Gt, x1[i + j], x4[i + j]);
                    *reinterpret_cast<float4*>(dst + i) = make_float4(o[0], o[1], o[2], o[3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();                               // TMEM and shared memory free for the next chunk
    if (*dead) break;
    }
    if (warp == 0) tmem_dealloc(tmem, 512);
}


// Workspace of the chunked backward: gate vectors | records | S checkpoints | d rows |
// Sb checkpoints | dd rows | dlogg, each 1024-byte aligned.
struct CbWs {
    size_t gv, rec, ckS, ckD, ckSb, ckDD, dlogg, total;
};
size_t crec_bytes(int dk, int dv) {
    if (dk == 128) return dv == 128 ? CRec<128, 128>::BYTES : CRec<128, 64>::BYTES;
    return dv == 128 ? CRec<64, 128>::BYTES : CRec<64, 64>::BYTES;
}
CbWs cb_ws(size_t bh, int T, int dk, int dv) {
    const size_t n = (static_cast<size_t>(T) + kCC - 1) / kCC, nc = bh * n;
    auto al = [](size_t x) { return (x + 1023) / 1024 * 1024; };
    CbWs w;
    w.gv = 0;
    w.rec = w.gv + al(nc * 3 * kCC * 4);
    w.ckS = w.rec + al(nc * crec_bytes(dk, dv));
    w.ckD = w.ckS + al(nc * dk * 512);               // S^T image (hi, lo): 128 rows x dk bf16 each
    w.ckSb = w.ckD + al(nc * 32768);                 // d^T image (hi, lo): 128 rows x 64 bf16 each
    w.ckDD = w.ckSb + al(nc * dk * 512);
    w.dlogg = w.ckDD + al(nc * 32768);
    w.total = w.dlogg + al(bh * static_cast<size_t>(T) * 4) + 1024;
    return w;
}

template <int DK, int DV>
int launch_cb(const CbArgs& a, cudaStream_t st) {
    static int attr_ok = -1;                       // set once per process: the kernels' shared-memory limits
    if (attr_ok < 0)
        attr_ok = cudaFuncSetAttribute(cb_mats_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       MatsSmem<DK>::BYTES) == cudaSuccess &&
                          cudaFuncSetAttribute(cb_chain_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               ChainSmem<DK, DV>::BYTES) == cudaSuccess &&
                          cudaFuncSetAttribute(cb_grads_tc_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               GtLayout<DK, DV>::BYTES) == cudaSuccess
                      ? 1
                      : 0;
    if (!attr_ok) return fail(GDN_ERR_CUDA, "gdn_prefill_bwd (chunked): cannot configure the kernels' shared memory");
    const unsigned nchunks = static_cast<unsigned>(static_cast<long>(a.B) * a.H * a.n);
    cb_mats_kernel<DK, DV><<<nchunks, 256, MatsSmem<DK>::BYTES, st>>>(a);
    int s = launch_status("gdn_prefill_bwd (chunk matrices)");
    if (s != GDN_OK) return s;
    cb_chain_kernel<DK, DV><<<2 * a.B * a.H, 256, ChainSmem<DK, DV>::BYTES, st>>>(a);
    if ((s = launch_status("gdn_prefill_bwd (chunk recurrences)")) != GDN_OK) return s;
    int nsm = 148;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    }
    const int gridg = static_cast<int>(nchunks) < nsm ? static_cast<int>(nchunks) : nsm;
    // q, k as [B H][T][DK] bf16 for the TMA loads of the gradient kernel's [Q; K] image
    CUtensorMap mq, mk;
    {
        const uint64_t dims[3] = {static_cast<uint64_t>(DK), static_cast<uint64_t>(a.T),
                                  static_cast<uint64_t>(a.B) * a.H};
        const uint64_t strides[2] = {static_cast<uint64_t>(DK) * 2, static_cast<uint64_t>(a.T) * DK * 2};
        const uint32_t box[3] = {64, 64, 1};
        int ms;
        if ((ms = make_map_bf16(&mq, a.q, 3, dims, strides, box, true)) != GDN_OK) return ms;
        if ((ms = make_map_bf16(&mk, a.k, 3, dims, strides, box, true)) != GDN_OK) return ms;
    }
    cb_grads_tc_kernel<DK, DV><<<gridg, 256, GtLayout<DK, DV>::BYTES, st>>>(a, static_cast<int>(nchunks), mq, mk);
    return launch_status("gdn_prefill_bwd (chunk gradients)");
}

}  // namespace

size_t prefill_bwd_chunked_workspace(int B, int T, int H, int dk, int dv) {
    return cb_ws(static_cast<size_t>(B) * H, T, dk, dv).total;
}

// The chunked backward (the arguments of gdn_prefill_bwd, validated by it).
int prefill_bwd_chunked(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                        const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec, const float* mask,
                        const float* state_in, const void* dO, int do_dtype, const float* dS_final, float* dq, float* dk,
                        float* dv, float* da, float* db, float* dA_log, float* ddt_bias, float* dstate_in, int B, int T,
                        int H, int dkd, int dvd, float scale, void* workspace, cudaStream_t st) {
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dO) || !aligned16(dq) || !aligned16(dk) ||
        !aligned16(dv))
        return fail(GDN_ERR_ALIGN, "gdn_prefill_bwd (chunked): q, k, v, dO, dq, dk and dv must be 16-byte aligned");
    CbArgs ar;
    ar.q = static_cast<const uint16_t*>(q);
    ar.k = static_cast<const uint16_t*>(k);
    ar.v = static_cast<const uint16_t*>(v);
    ar.A_log = A_log;
    ar.a = a;
    ar.b = b_logits;
    ar.gate_dtype = gate_dtype;
    ar.dt_bias = dt_bias;
    ar.dt_bias_vec = dt_bias_vec;
    ar.mask = mask;
    ar.state_in = state_in;
    ar.dO = dO;
    ar.do_dtype = do_dtype;
    ar.dS_final = dS_final;
    ar.dq = dq;
    ar.dk = dk;
    ar.dv = dv;
    ar.da = da;
    ar.db = db;
    ar.dstate_in = dstate_in;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const CbWs wl = cb_ws(static_cast<size_t>(B) * H, T, dkd, dvd);
    ar.gv = reinterpret_cast<float*>(ws + wl.gv);
    ar.rec = ws + wl.rec;
    ar.ckS = ws + wl.ckS;
    ar.ckD = ws + wl.ckD;
    ar.ckSb = ws + wl.ckSb;
    ar.ckDD = ws + wl.ckDD;
    ar.dlogg = reinterpret_cast<float*>(ws + wl.dlogg);
    ar.err = device_error_word();
    ar.B = B;
    ar.T = T;
    ar.H = H;
    ar.n = (T + kCC - 1) / kCC;
    ar.scale = scale;
    int s;
    if (dkd == 128 && dvd == 128) s = launch_cb<128, 128>(ar, st);
    else if (dkd == 128 && dvd == 64) s = launch_cb<128, 64>(ar, st);
    else if (dkd == 64 && dvd == 128) s = launch_cb<64, 128>(ar, st);
    else s = launch_cb<64, 64>(ar, st);
    if (s != GDN_OK) return s;
    return launch_bwd_head_sums(A_log, a, gate_dtype, dt_bias, dt_bias_vec, ar.dlogg, da, dA_log, ddt_bias, B, T, H,
                                st);
}

}  // namespace gdn
