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
// Launches (all fp32 on CUDA cores):
//   cb_mats_kernel     per chunk: M, P, A = (I + diag(b) M)^-1 and the gate vectors (Lambda, b,
//                      m), all chunks in parallel, so that both substitutions become products:
//                      d = A (b (v - G K S)) and dd = A^T X;
//   cb_forward_kernel  per (b, h, 64 value columns): the forward chunk recurrence, storing S at
//                      every chunk start and the chunk's d rows;
//   cb_reverse_kernel  per (b, h, 64 value columns): the reverse chunk recurrence, storing Sb at
//                      every chunk end and the dd rows (the value columns are independent in both);
//   cb_grads_kernel    per chunk: every per-token gradient from S, Sb, D and dd, then the gate
//                      chain rule into da, db;
//   the head sums of dA_log, ddt_bias (the token-recurrent backward's bwd_head_kernel).
#include "common.cuh"

namespace gdn {

// the head sums (backward.cu): dA_log[h] = sum dlogg log g, ddt_bias[h] = sum da
void launch_bwd_head_sums(const float* A_log, const void* a, int gate_dtype, float dt_bias, const float* dt_bias_vec,
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
    float* mp;                          // [cid][3][64][64]: M, P, A
    float* ckS;                         // [cid][DK][DV]: the state entering the chunk
    float* ckD;                         // [cid][64][DV]: the chunk's d rows
    float* ckSb;                        // [cid][DK][DV]: the gradient of the state leaving the chunk
    float* ckDD;                        // [cid][64][DV]: the chunk's dd rows
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
__device__ __forceinline__ void load_f8(const float* p, float (&x)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Per chunk (one CTA of 128 threads): the gate vectors (Lambda, b, m), then
// [Q; K] K^T on the tensor cores (bf16 q, k, fp32 accumulate: TMEM lane r < 64
// holds row r of Q K^T, lane 64 + t row t of K K^T), P = scale (Q K^T) * [G_t/G_s,
// s <= t] and A = (I + diag(b) M)^-1 with M = (K K^T) * [G_t/G_s, s < t]:
// the four 16 x 16 diagonal blocks by forward substitution (one column per
// thread), then the blocks below them by distance from the diagonal,
// A_ij = -A_ii sum_{j <= k < i} (diag(b) M)_ik A_kj.  Writes A^T, P and A.
// Padded tokens (past T) get log g = 0, b = m = 0 and zero k, q.
// ---------------------------------------------------------------------------
template <int DK>
struct MatsSmem {
    static constexpr int QK_KB = 128 * 128;
    static constexpr int OFF_QK = 0;                               // [Q; K] image, 128 rows x DK
    static constexpr int OFF_L = OFF_QK + (DK / 64) * QK_KB;       // diag(b) M   [64][65] fp32
    static constexpr int OFF_A = OFF_L + kCC * 65 * 4;             // A           [64][65]
    static constexpr int OFF_T = OFF_A + kCC * 65 * 4;             // block sums  [3][16][17]
    static constexpr int OFF_G = OFF_T + 3 * 16 * 17 * 4;          // Lambda, b, m [3][64]
    static constexpr int OFF_BAR = OFF_G + 3 * kCC * 4;
    static constexpr int BYTES = OFF_BAR + 16 + 1024;
};

template <int DK>
__global__ void __launch_bounds__(128) cb_mats_kernel(const CbArgs a) {
    using L = MatsSmem<DK>;
    constexpr int CPK = DK / 8;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* Ls = reinterpret_cast<float*>(sm + L::OFF_L);
    float* As = reinterpret_cast<float*>(sm + L::OFF_A);
    float* Ts = reinterpret_cast<float*>(sm + L::OFF_T);
    float* lam = reinterpret_cast<float*>(sm + L::OFF_G);
    float* bms = lam + kCC;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int cid = blockIdx.x, bh = cid / a.n, c = cid - bh * a.n;
    const int h = bh % a.H, bi = bh / a.H;
    const int t0 = c * kCC, nt = min(kCC, a.T - t0);
    const int tid = threadIdx.x, warp = tid >> 5;
    const long tokbase = static_cast<long>(bh) * a.T + t0;

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, 64);
        tmem_relinquish();
    }
    for (int it = tid; it < 128 * CPK; it += 128) {
        const int row = it / CPK, ch = it - row * CPK, t = row & (kCC - 1);
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (t < nt) u = __ldg(reinterpret_cast<const uint4*>((row < kCC ? a.q : a.k) + (tokbase + t) * DK + ch * 8));
        *reinterpret_cast<uint4*>(sm + L::OFF_QK + (ch >> 3) * L::QK_KB + sw128_chunk(row, ch & 7)) = u;
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
        float s = 0.f;                                 // in-chunk cumulative log decay, in token order
        for (int t = 0; t < kCC; ++t) {
            s += lam[t];
            lam[t] = s;
        }
    }
    __syncthreads();
    if (tid < kCC) gv[tid] = lam[tid];
    const bool ok = mbar_wait(bar, 0, a.err);
    tc_fence_after();
    float* At = a.mp + static_cast<long>(cid) * 3 * kCC * kCC;
    float* P = At + kCC * kCC;
    float* A = P + kCC * kCC;
    {
        // row r of the product: P row r (r < 64) or diag(b) M row r - 64
        const int r = tid, t = r & (kCC - 1);
        const float lt = lam[t];
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
            if (r < kCC) {
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float o[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int s = cb + i + q;
                        o[q] = s <= t ? a.scale * x[i + q] * expf(lt - lam[s]) : 0.f;
                    }
                    *reinterpret_cast<float4*>(P + t * kCC + cb + i) = make_float4(o[0], o[1], o[2], o[3]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int s = cb + i;
                    Ls[t * 65 + s] = s < t ? bt * x[i] * expf(lt - lam[s]) : 0.f;
                }
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
    // blocks above the diagonal are zero
    for (int e = tid; e < kCC * kCC; e += 128) {
        const int r = e >> 6, s = e & 63;
        if ((s >> 4) > (r >> 4)) As[r * 65 + s] = 0.f;
    }
    __syncthreads();
    // below the diagonal, by distance dd from it: T = sum_k L_ik A_kj, then A_ij = -A_ii T
#pragma unroll 1
    for (int dd = 1; dd < 4; ++dd) {
        const int nb = 4 - dd;
        for (int e = tid; e < nb * 256; e += 128) {
            const int jb = e >> 8, rr = (e >> 4) & 15, cc = e & 15, ib = jb + dd;
            float acc = 0.f;
            for (int kb = jb; kb < ib; ++kb)
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    acc = fmaf(Ls[(ib * 16 + rr) * 65 + kb * 16 + q], As[(kb * 16 + q) * 65 + jb * 16 + cc], acc);
            Ts[(jb * 16 + rr) * 17 + cc] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nb * 256; e += 128) {
            const int jb = e >> 8, rr = (e >> 4) & 15, cc = e & 15, ib = jb + dd;
            float acc = 0.f;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                acc = fmaf(As[(ib * 16 + rr) * 65 + ib * 16 + q], Ts[(jb * 16 + q) * 17 + cc], acc);
            As[(ib * 16 + rr) * 65 + jb * 16 + cc] = -acc;
        }
        __syncthreads();
    }
    for (int e = tid; e < kCC * kCC / 4; e += 128) {
        const int r = e >> 4, s = (e & 15) * 4;
        *reinterpret_cast<float4*>(A + r * kCC + s) =
            make_float4(As[r * 65 + s], As[r * 65 + s + 1], As[r * 65 + s + 2], As[r * 65 + s + 3]);
        *reinterpret_cast<float4*>(At + r * kCC + s) =
            make_float4(As[s * 65 + r], As[(s + 1) * 65 + r], As[(s + 2) * 65 + r], As[(s + 3) * 65 + r]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------
// The chunk recurrences, grid (B*H, DV/64), 256 threads.  Thread (rg, col) keeps
// rows [32 rg, 32 rg + 32) of value column 64 blockIdx.y + col of the state in
// registers (rg < DK/32); for the per-token passes thread (g, col), g = tid / 64,
// takes token rows [16 g, 16 g + 16).  The next chunk's operands are loaded into
// registers while the current chunk computes and are stored to shared memory at
// its end, so no chunk waits on a global load.  k and q are held in fp32 and read
// as float4 broadcasts (one per four multiply-adds); the decay factors are tables.
// ---------------------------------------------------------------------------
template <int DK>
struct RecSmem {
    static constexpr int RG = DK / 32;
    static constexpr int KF = 0;                   // k [64][DK] fp32
    static constexpr int QF = KF + kCC * DK;       // q [64][DK] fp32 (reverse)
    static constexpr int M0 = QF + kCC * DK;       // A^T (forward) or P (reverse) [64][64]
    static constexpr int M1 = M0 + kCC * kCC;      // A (reverse)
    static constexpr int CB = M1 + kCC * kCC;      // v (forward) or dO (reverse), this CTA's 64 columns
    static constexpr int PART = CB + kCC * 64;     // [RG][64][64] partial row sums over state rows
    static constexpr int XB = PART + RG * kCC * 64;   // [64][64] y then d (forward), X then dd (reverse)
    static constexpr int GVR = XB + kCC * 64;      // the next chunk's gate vectors as stored (Lambda, b, m)
    static constexpr int TB = GVR + 3 * kCC;       // tables: G, G_L/G, b, m
    static constexpr int FLOATS = TB + 4 * kCC;
    static constexpr int BYTES = FLOATS * 4;
};

__device__ __forceinline__ void bf8_to_f32(const uint4 u, float* dst) {
    float x[8];
    unpack_bf16x8(u, x);
    *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

// The tables of the chunk whose gate vectors are in GVR.
__device__ __forceinline__ void rec_tables(float* sm_f, int gvr, int tb, int tid) {
    if (tid < kCC) {
        const float l = sm_f[gvr + tid], lL = sm_f[gvr + kCC - 1];
        sm_f[tb + tid] = expf(l);
        sm_f[tb + kCC + tid] = expf(lL - l);
        sm_f[tb + 2 * kCC + tid] = sm_f[gvr + kCC + tid];
        sm_f[tb + 3 * kCC + tid] = sm_f[gvr + 2 * kCC + tid];
    }
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) cb_forward_kernel(const CbArgs a) {
    using L = RecSmem<DK>;
    constexpr int RG = L::RG, NK = DK / 32;        // k pieces (8 bf16) per thread
    extern __shared__ float smf[];
    float* KF = smf + L::KF;
    float* At = smf + L::M0;
    float* Vb = smf + L::CB;
    float* part = smf + L::PART;
    float* XB = smf + L::XB;
    const float* Gt_ = smf + L::TB;
    const float* CF = smf + L::TB + kCC;
    const float* Bt = smf + L::TB + 2 * kCC;
    const int bh = blockIdx.x, tid = threadIdx.x, col = tid & 63, rg = tid >> 6;
    const int j = blockIdx.y * 64 + col;
    const bool rows_ok = rg < RG;

    uint4 pk[NK], pv[2];
    float4 pa[4], pg = make_float4(0.f, 0.f, 0.f, 0.f);
    auto load = [&](int c) {
        const int t0 = c * kCC, nt = min(kCC, a.T - t0);
        const long tb = static_cast<long>(bh) * a.T + t0, cid = static_cast<long>(bh) * a.n + c;
#pragma unroll
        for (int i = 0; i < NK; ++i) {
            const int p = tid + 256 * i, row = p / (DK / 8);
            pk[i] = row < nt ? __ldg(reinterpret_cast<const uint4*>(a.k + tb * DK) + p) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int p = tid + 256 * i, row = p >> 3;
            pv[i] = row < nt ? __ldg(reinterpret_cast<const uint4*>(a.v + (tb + row) * DV + blockIdx.y * 64) + (p & 7))
                             : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
            pa[i] = __ldg(reinterpret_cast<const float4*>(a.mp + (cid * 3 + 0) * kCC * kCC) + tid + 256 * i);
        if (tid < 48) pg = __ldg(reinterpret_cast<const float4*>(a.gv + cid * 3 * kCC) + tid);
    };
    auto store = [&]() {
#pragma unroll
        for (int i = 0; i < NK; ++i) bf8_to_f32(pk[i], KF + (tid + 256 * i) * 8);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int p = tid + 256 * i;
            bf8_to_f32(pv[i], Vb + (p >> 3) * 64 + (p & 7) * 8);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) reinterpret_cast<float4*>(At)[tid + 256 * i] = pa[i];
        if (tid < 48) reinterpret_cast<float4*>(smf + L::GVR)[tid] = pg;
        __syncthreads();
        rec_tables(smf, L::GVR, L::TB, tid);
        __syncthreads();
    };

    float S[32];
    const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
    for (int i = 0; i < 32; ++i)
        S[i] = (rows_ok && a.state_in) ? a.state_in[s0 + static_cast<long>(rg * 32 + i) * DV + j] : 0.f;
    load(0);
    store();
#pragma unroll 1
    for (int c = 0; c < a.n; ++c) {
        const long cid = static_cast<long>(bh) * a.n + c;
        if (c + 1 < a.n) load(c + 1);
        if (rows_ok) {
            float* ck = a.ckS + cid * DK * DV + static_cast<long>(rg * 32) * DV + j;
#pragma unroll
            for (int i = 0; i < 32; ++i) ck[static_cast<long>(i) * DV] = S[i];
            // (K S) partials over this thread's 32 rows, four tokens at a time
#pragma unroll 1
            for (int t = 0; t < kCC; t += 4) {
                float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
                for (int i = 0; i < 32; i += 4)
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 k4 = *reinterpret_cast<const float4*>(KF + (t + u) * DK + rg * 32 + i);
                        acc[u][0] = fmaf(k4.x, S[i], fmaf(k4.y, S[i + 1], acc[u][0]));
                        acc[u][1] = fmaf(k4.z, S[i + 2], fmaf(k4.w, S[i + 3], acc[u][1]));
                    }
#pragma unroll
                for (int u = 0; u < 4; ++u) part[(rg * kCC + t + u) * 64 + col] = acc[u][0] + acc[u][1];
            }
        }
        __syncthreads();
        // y = b (v - G K S), rows [16 rg, 16 rg + 16)
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int t = rg * 16 + r;
            float kS = 0.f;
#pragma unroll
            for (int g = 0; g < RG; ++g) kS += part[(g * kCC + t) * 64 + col];
            XB[t * 64 + col] = Bt[t] * (Vb[t * 64 + col] - Gt_[t] * kS);
        }
        __syncthreads();
        // d = A y: A^T rows give a thread's 16 rows as float4 broadcasts (A[t][s] = 0 for s > t)
        float acc[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll 2
        for (int s = 0; s < rg * 16 + 16; ++s) {
            const float ys = XB[s * 64 + col];
            const float4* ar = reinterpret_cast<const float4*>(At + s * kCC + rg * 16);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const float4 a4 = ar[q4];
                acc[4 * q4] = fmaf(a4.x, ys, acc[4 * q4]);
                acc[4 * q4 + 1] = fmaf(a4.y, ys, acc[4 * q4 + 1]);
                acc[4 * q4 + 2] = fmaf(a4.z, ys, acc[4 * q4 + 2]);
                acc[4 * q4 + 3] = fmaf(a4.w, ys, acc[4 * q4 + 3]);
            }
        }
        __syncthreads();
        {
            float* ckd = a.ckD + cid * kCC * DV + j;
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                XB[(rg * 16 + r) * 64 + col] = acc[r];
                ckd[static_cast<long>(rg * 16 + r) * DV] = acc[r];
            }
        }
        __syncthreads();
        // S <- G_L S + K^T diag(G_L/G) D
        if (rows_ok) {
            const float GL = Gt_[kCC - 1];
#pragma unroll
            for (int i = 0; i < 32; ++i) S[i] *= GL;
#pragma unroll 2
            for (int t = 0; t < kCC; ++t) {
                const float cf = CF[t] * XB[t * 64 + col];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(KF + t * DK + rg * 32 + i);
                    S[i] = fmaf(k4.x, cf, S[i]);
                    S[i + 1] = fmaf(k4.y, cf, S[i + 1]);
                    S[i + 2] = fmaf(k4.z, cf, S[i + 2]);
                    S[i + 3] = fmaf(k4.w, cf, S[i + 3]);
                }
            }
        }
        __syncthreads();
        if (c + 1 < a.n) store();
    }
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) cb_reverse_kernel(const CbArgs a) {
    using L = RecSmem<DK>;
    constexpr int RG = L::RG, NK = DK / 32;
    extern __shared__ float smf[];
    float* KF = smf + L::KF;
    float* QF = smf + L::QF;
    float* Pm = smf + L::M0;
    float* Am = smf + L::M1;
    float* Ob = smf + L::CB;
    float* part = smf + L::PART;
    float* XB = smf + L::XB;
    const float* Gt_ = smf + L::TB;
    const float* CF = smf + L::TB + kCC;
    const float* Bt = smf + L::TB + 2 * kCC;
    const float* Mt = smf + L::TB + 3 * kCC;
    const int bh = blockIdx.x, tid = threadIdx.x, col = tid & 63, rg = tid >> 6;
    const int j = blockIdx.y * 64 + col;
    const bool rows_ok = rg < RG;
    const bool do_bf = a.do_dtype == GDN_DTYPE_BF16;

    uint4 pk[NK], pq[NK];
    float4 pp[4], pa[4], po[4], pg = make_float4(0.f, 0.f, 0.f, 0.f);
    auto load = [&](int c) {
        const int t0 = c * kCC, nt = min(kCC, a.T - t0);
        const long tb = static_cast<long>(bh) * a.T + t0, cid = static_cast<long>(bh) * a.n + c;
#pragma unroll
        for (int i = 0; i < NK; ++i) {
            const int p = tid + 256 * i, row = p / (DK / 8);
            const bool in = row < nt;
            pk[i] = in ? __ldg(reinterpret_cast<const uint4*>(a.k + tb * DK) + p) : make_uint4(0u, 0u, 0u, 0u);
            pq[i] = in ? __ldg(reinterpret_cast<const uint4*>(a.q + tb * DK) + p) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            pp[i] = __ldg(reinterpret_cast<const float4*>(a.mp + (cid * 3 + 1) * kCC * kCC) + tid + 256 * i);
            pa[i] = __ldg(reinterpret_cast<const float4*>(a.mp + (cid * 3 + 2) * kCC * kCC) + tid + 256 * i);
        }
        if (do_bf) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int p = tid + 256 * i, row = p >> 3;
                const uint4 u = row < nt ? __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.dO) +
                                                                                (tb + row) * DV + blockIdx.y * 64) +
                                                 (p & 7))
                                         : make_uint4(0u, 0u, 0u, 0u);
                po[2 * i] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                                        __uint_as_float(u.w));
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int p = tid + 256 * i, row = p >> 4;
                po[i] = row < nt ? __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.dO) +
                                                                        (tb + row) * DV + blockIdx.y * 64) +
                                         (p & 15))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        if (tid < 48) pg = __ldg(reinterpret_cast<const float4*>(a.gv + cid * 3 * kCC) + tid);
    };
    auto store = [&]() {
#pragma unroll
        for (int i = 0; i < NK; ++i) {
            bf8_to_f32(pk[i], KF + (tid + 256 * i) * 8);
            bf8_to_f32(pq[i], QF + (tid + 256 * i) * 8);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            reinterpret_cast<float4*>(Pm)[tid + 256 * i] = pp[i];
            reinterpret_cast<float4*>(Am)[tid + 256 * i] = pa[i];
        }
        if (do_bf) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int p = tid + 256 * i;
                const float4 f = po[2 * i];
                bf8_to_f32(make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z),
                                      __float_as_uint(f.w)),
                           Ob + (p >> 3) * 64 + (p & 7) * 8);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int p = tid + 256 * i;
                *reinterpret_cast<float4*>(Ob + (p >> 4) * 64 + (p & 15) * 4) = po[i];
            }
        }
        if (tid < 48) reinterpret_cast<float4*>(smf + L::GVR)[tid] = pg;
        __syncthreads();
        rec_tables(smf, L::GVR, L::TB, tid);
        __syncthreads();
    };

    float Sb[32];
    const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
    for (int i = 0; i < 32; ++i)
        Sb[i] = (rows_ok && a.dS_final) ? a.dS_final[s0 + static_cast<long>(rg * 32 + i) * DV + j] : 0.f;
    load(a.n - 1);
    store();
#pragma unroll 1
    for (int c = a.n - 1; c >= 0; --c) {
        const long cid = static_cast<long>(bh) * a.n + c;
        if (c > 0) load(c - 1);
        if (rows_ok) {
            float* ck = a.ckSb + cid * DK * DV + static_cast<long>(rg * 32) * DV + j;
#pragma unroll
            for (int i = 0; i < 32; ++i) ck[static_cast<long>(i) * DV] = Sb[i];
#pragma unroll 1
            for (int t = 0; t < kCC; t += 4) {
                float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
                for (int i = 0; i < 32; i += 4)
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 k4 = *reinterpret_cast<const float4*>(KF + (t + u) * DK + rg * 32 + i);
                        acc[u][0] = fmaf(k4.x, Sb[i], fmaf(k4.y, Sb[i + 1], acc[u][0]));
                        acc[u][1] = fmaf(k4.z, Sb[i + 2], fmaf(k4.w, Sb[i + 3], acc[u][1]));
                    }
#pragma unroll
                for (int u = 0; u < 4; ++u) part[(rg * kCC + t + u) * 64 + col] = acc[u][0] + acc[u][1];
            }
        }
        __syncthreads();
        // X_t = (G_L/G_t)(K Sb)_t + sum_{u >= t} P_ut m_u dO_u, rows [16 rg, 16 rg + 16)
        float acc[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int t = rg * 16 + r;
            float kS = 0.f;
#pragma unroll
            for (int g = 0; g < RG; ++g) kS += part[(g * kCC + t) * 64 + col];
            acc[r] = CF[t] * kS;
        }
#pragma unroll 2
        for (int u = rg * 16; u < kCC; ++u) {
            const float d = Mt[u] * Ob[u * 64 + col];
            const float4* pr = reinterpret_cast<const float4*>(Pm + u * kCC + rg * 16);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const float4 p4 = pr[q4];
                acc[4 * q4] = fmaf(p4.x, d, acc[4 * q4]);
                acc[4 * q4 + 1] = fmaf(p4.y, d, acc[4 * q4 + 1]);
                acc[4 * q4 + 2] = fmaf(p4.z, d, acc[4 * q4 + 2]);
                acc[4 * q4 + 3] = fmaf(p4.w, d, acc[4 * q4 + 3]);
            }
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) XB[(rg * 16 + r) * 64 + col] = acc[r];
        __syncthreads();
        // dd_s = sum_{u >= s} A_us X_u
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll 2
        for (int u = rg * 16; u < kCC; ++u) {
            const float x = XB[u * 64 + col];
            const float4* ar = reinterpret_cast<const float4*>(Am + u * kCC + rg * 16);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const float4 a4 = ar[q4];
                acc[4 * q4] = fmaf(a4.x, x, acc[4 * q4]);
                acc[4 * q4 + 1] = fmaf(a4.y, x, acc[4 * q4 + 1]);
                acc[4 * q4 + 2] = fmaf(a4.z, x, acc[4 * q4 + 2]);
                acc[4 * q4 + 3] = fmaf(a4.w, x, acc[4 * q4 + 3]);
            }
        }
        __syncthreads();
        {
            float* ckdd = a.ckDD + cid * kCC * DV + j;
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                XB[(rg * 16 + r) * 64 + col] = acc[r];
                ckdd[static_cast<long>(rg * 16 + r) * DV] = acc[r];
            }
        }
        __syncthreads();
        // Sb <- G_L Sb + scale (diag(G) Q)^T dO' - (diag(G b) K)^T dd
        if (rows_ok) {
            const float GL = Gt_[kCC - 1];
#pragma unroll
            for (int i = 0; i < 32; ++i) Sb[i] *= GL;
#pragma unroll 2
            for (int t = 0; t < kCC; ++t) {
                const float G = Gt_[t];
                const float cq = a.scale * G * Mt[t] * Ob[t * 64 + col], ck_ = -G * Bt[t] * XB[t * 64 + col];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(QF + t * DK + rg * 32 + i);
                    const float4 k4 = *reinterpret_cast<const float4*>(KF + t * DK + rg * 32 + i);
                    Sb[i] = fmaf(q4.x, cq, fmaf(k4.x, ck_, Sb[i]));
                    Sb[i + 1] = fmaf(q4.y, cq, fmaf(k4.y, ck_, Sb[i + 1]));
                    Sb[i + 2] = fmaf(q4.z, cq, fmaf(k4.z, ck_, Sb[i + 2]));
                    Sb[i + 3] = fmaf(q4.w, cq, fmaf(k4.w, ck_, Sb[i + 3]));
                }
            }
        }
        __syncthreads();
        if (c > 0) store();
    }
    if (rows_ok && a.dstate_in) {
#pragma unroll
        for (int i = 0; i < 32; ++i) a.dstate_in[s0 + static_cast<long>(rg * 32 + i) * DV + j] = Sb[i];
    }
}

// ---------------------------------------------------------------------------
// Per chunk on the tensor cores (one CTA of 256 threads, 512 TMEM columns).
// Every product runs as tcgen05 kind::f16 with fp32 operands split into bf16
// hi + lo (hi.hi + hi.lo + lo.hi; q, k exact in bf16), relative error ~2^-16:
//   T1 = [dO'; dd] S^T      -> lanes 0-63 X_q = dO' S^T, lanes 64-127 X_dd = dd S^T
//   T3 = [dO'; dd] D^T      -> lanes 0-63 dO' D^T,       lanes 64-127 Y = dd D^T
//   T5 = [Q; K] K^T         -> lanes 0-63 Q K^T,         lanes 64-127 K K^T
//   T2 = [dd; D] Sb^T       -> lanes 64-127 X_e = D Sb^T
//   T4 = [F1; F2 + F2^T] K^T' + [0; scale F1^T] Q^T'  (K^T', Q^T' the k, q tiles
//        transposed; F1 = (dO' D^T) * [G_t/G_s, s <= t], F2 = -b (Y * [G_t/G_s, s < t]))
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
    static constexpr int R_KB = 192 * 128;                 // one 64-column block of the 192-row image
    static constexpr int R_BYTES = (DV / 64) * R_KB;
    static constexpr int S_KB = DK * 128;
    static constexpr int S_BYTES = (DV / 64) * S_KB;
    static constexpr int QK_KB = 128 * 128;
    static constexpr int QK_BYTES = (DK / 64) * QK_KB;
    static constexpr int OFF_RH = 0, OFF_RL = R_BYTES, OFF_SH = 2 * R_BYTES, OFF_SL = OFF_SH + S_BYTES;
    static constexpr int AB_END = OFF_SL + S_BYTES;
    static constexpr int OFF_A1H = 0, OFF_A1L = 16384, OFF_A2H = 32768, OFF_A2L = 49152;   // after T2
    static constexpr int OFF_KT = 65536, OFF_QT = OFF_KT + DK * 128;
    static constexpr int C_END = OFF_QT + DK * 128;
    static constexpr int OFF_QK = AB_END > C_END ? AB_END : C_END;
    static constexpr int QK_REGION = QK_BYTES > 32768 ? QK_BYTES : 32768;       // then F1, F2 fp32 [64][64]
    static constexpr int OFF_MISC = OFF_QK + QK_REGION;
    static constexpr int MISC_FLOATS = 912;
    static constexpr int OFF_BAR = OFF_MISC + MISC_FLOATS * 4;
    static constexpr int BYTES = OFF_BAR + 64 + 1024;      // + slack to align the dynamic base to 1024
    static constexpr uint32_t T_XS = 0, T_XE = DK, T_X4 = 2 * DK, T_DD = 3 * DK, T_QK = 3 * DK + 64;
    static_assert(BYTES <= 232448, "shared memory");
    static_assert(T_QK + 64 <= 512, "TMEM columns");
};

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) cb_grads_tc_kernel(const CbArgs a) {
    using L = GtLayout<DK, DV>;
    constexpr int CPR = DV / 8;                    // 8-value chunks per value row
    constexpr int CPK = DK / 8;                    // per key row
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
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
    float* F1s = reinterpret_cast<float*>(sm + L::OFF_QK);          // [64][64], row t rotated by t
    float* F2s = F1s + 4096;

    const int cid = blockIdx.x, bh = cid / a.n, c = cid - bh * a.n;
    const int h = bh % a.H;
    const int t0 = c * kCC, nt = min(kCC, a.T - t0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long tokbase = static_cast<long>(bh) * a.T + t0;
    const uint32_t sbase = smem_u32(sm);
    const float* ckS = a.ckS + static_cast<long>(cid) * DK * DV;
    const float* ckSb = a.ckSb + static_cast<long>(cid) * DK * DV;
    const float* ckD = a.ckD + static_cast<long>(cid) * kCC * DV;
    const float* ckDD = a.ckDD + static_cast<long>(cid) * kCC * DV;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        *dead = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, 512);
    if (tid < kCC) {
        const float* gv = a.gv + static_cast<long>(cid) * 3 * kCC;
        lam[tid] = gv[tid];
        Gs[tid] = expf(gv[tid]);
        bms[tid] = gv[kCC + tid];
        ms[tid] = gv[2 * kCC + tid];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    // ---- phase A: [dO'; dd; D] and S as bf16 hi/lo images, [Q; K]; dv = b dd; dd . v
    for (int it = tid; it < 192 * CPR; it += 256) {
        const int row = it / CPR, ch = it - row * CPR;
        float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float dvp = 0.f;
        if (row < kCC) {
            if (row < nt) {
                const long gi = (tokbase + row) * DV + ch * 8;
                if (a.do_dtype == GDN_DTYPE_BF16)
                    unpack_bf16x8(*reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.dO) + gi), x);
                else
                    load_f8(static_cast<const float*>(a.dO) + gi, x);
                const float m = ms[row];
#pragma unroll
                for (int i = 0; i < 8; ++i) x[i] *= m;
            }
        } else if (row < 2 * kCC) {
            const int t = row - kCC;
            load_f8(ckDD + t * DV + ch * 8, x);
            if (t < nt) {
                const float b = bms[t];
                float* dst = a.dv + (tokbase + t) * DV + ch * 8;
                *reinterpret_cast<float4*>(dst) = make_float4(b * x[0], b * x[1], b * x[2], b * x[3]);
                *reinterpret_cast<float4*>(dst + 4) = make_float4(b * x[4], b * x[5], b * x[6], b * x[7]);
                float vv[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(a.v + (tokbase + t) * DV + ch * 8), vv);
#pragma unroll
                for (int i = 0; i < 8; ++i) dvp = fmaf(x[i], vv[i], dvp);
            }
        } else {
            load_f8(ckD + (row - 2 * kCC) * DV + ch * 8, x);
        }
#pragma unroll
        for (int o = CPR / 2; o > 0; o >>= 1) dvp += __shfl_xor_sync(0xffffffffu, dvp, o);
        if (row >= kCC && row < 2 * kCC && ch == 0) ddv[row - kCC] = dvp;
        const uint32_t off = (ch >> 3) * L::R_KB + sw128_chunk(row, ch & 7);
        split_store8(sm + L::OFF_RH + off, sm + L::OFF_RL + off, x);
    }
    for (int it = tid; it < DK * CPR; it += 256) {
        const int d = it / CPR, ch = it - d * CPR;
        float x[8];
        load_f8(ckS + d * DV + ch * 8, x);
        const uint32_t off = (ch >> 3) * L::S_KB + sw128_chunk(d, ch & 7);
        split_store8(sm + L::OFF_SH + off, sm + L::OFF_SL + off, x);
    }
    for (int it = tid; it < 128 * CPK; it += 256) {
        const int row = it / CPK, ch = it - row * CPK, t = row & (kCC - 1);
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (t < nt) u = *reinterpret_cast<const uint4*>((row < kCC ? a.q : a.k) + (tokbase + t) * DK + ch * 8);
        *reinterpret_cast<uint4*>(sm + L::OFF_QK + (ch >> 3) * L::QK_KB + sw128_chunk(row, ch & 7)) = u;
    }
    fence_async_smem();
    __syncthreads();
    const uint32_t rh = sbase + L::OFF_RH, rl = sbase + L::OFF_RL, sh = sbase + L::OFF_SH, sl = sbase + L::OFF_SL;
    if (tid == 0) {
        tc_fence_after();
        constexpr uint32_t idN = idesc_bf16(128, DK, false, false);
        constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
        const uint32_t pa[3] = {rh, rh, rl}, pbs[3] = {sh, sl, sh}, pbd[3] = {rh, rl, rh};
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int kk = 0; kk < DV / 16; ++kk) {
                const uint32_t ko = (kk >> 2) * L::R_KB + (kk & 3) * 32, so = (kk >> 2) * L::S_KB + (kk & 3) * 32;
                const uint32_t acc = (p > 0 || kk > 0) ? 1u : 0u;
                umma_bf16_ss(tmem + L::T_XS, sdesc_sw128(pa[p] + ko, 16, 1024), sdesc_sw128(pbs[p] + so, 16, 1024),
                             idN, acc);
                umma_bf16_ss(tmem + L::T_DD, sdesc_sw128(pa[p] + ko, 16, 1024),
                             sdesc_sw128(pbd[p] + ko + 2 * kCC * 128, 16, 1024), id64, acc);
            }
        const uint32_t qk = sbase + L::OFF_QK;
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * L::QK_KB + (kk & 3) * 32;
            umma_bf16_ss(tmem + L::T_QK, sdesc_sw128(qk + ko, 16, 1024), sdesc_sw128(qk + ko + kCC * 128, 16, 1024),
                         id64, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[0]);
    }

    // ---- phase B: Sb over the S image once T1 has read it, <S, Sb>, then T2
    if (!mbar_wait(&bars[0], 0, a.err)) *dead = 1;
    tc_fence_after();
    float sp = 0.f;
    for (int it = tid; it < DK * CPR; it += 256) {
        const int d = it / CPR, ch = it - d * CPR;
        float x[8], s8[8];
        load_f8(ckSb + d * DV + ch * 8, x);
        load_f8(ckS + d * DV + ch * 8, s8);
#pragma unroll
        for (int i = 0; i < 8; ++i) sp = fmaf(s8[i], x[i], sp);
        const uint32_t off = (ch >> 3) * L::S_KB + sw128_chunk(d, ch & 7);
        split_store8(sm + L::OFF_SH + off, sm + L::OFF_SL + off, x);
    }
    sp = warp_sum(sp);
    if (lane == 0) basep[warp] = sp;
    fence_async_smem();
    __syncthreads();
    const bool dead_b = *dead != 0;
    if (tid == 0 && !dead_b) {
        tc_fence_after();
        constexpr uint32_t idN = idesc_bf16(128, DK, false, false);
        const uint32_t pa[3] = {rh, rh, rl}, pbs[3] = {sh, sl, sh};
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int kk = 0; kk < DV / 16; ++kk) {
                const uint32_t ko = (kk >> 2) * L::R_KB + (kk & 3) * 32, so = (kk >> 2) * L::S_KB + (kk & 3) * 32;
                umma_bf16_ss(tmem + L::T_XE, sdesc_sw128(pa[p] + ko + kCC * 128, 16, 1024),
                             sdesc_sw128(pbs[p] + so, 16, 1024), idN, (p > 0 || kk > 0) ? 1u : 0u);
            }
        umma_commit(&bars[1]);
    }
    const float scale = a.scale;
    const float lL = lam[kCC - 1], GL = Gs[kCC - 1];
    // row work on warps 0-3: thread r = TMEM lane r, token t = r % 64, side = r / 64
    if (tid < 128 && !dead_b) {
        const int r = tid, t = r & (kCC - 1), side = r >> 6;
        const uint32_t lb = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        // q_t . X_q (side 0) or k_t . X_dd (side 1): row r of T1 against row r of [Q; K]
        float dot = 0.f;
#pragma unroll 1
        for (int cb = 0; cb < DK; cb += 32) {
            float x[32];
            tmem_ld32(lb + L::T_XS + cb, x);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = cb + 8 * j;
                float y[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + L::OFF_QK + (col >> 6) * L::QK_KB +
                                                              sw128_chunk(r, (col & 63) >> 3)),
                              y);
#pragma unroll
                for (int i = 0; i < 8; ++i) dot = fmaf(x[8 * j + i], y[i], dot);
            }
        }
        named_bar(1, 128);                          // [Q; K] read by all: its bytes become F1, F2
        const float lt = lam[t], Gt = Gs[t], bt = bms[t];
        float* Fs = side ? F2s : F1s;
        float pre = 0.f, krs = 0.f;
#pragma unroll 1
        for (int cb = 0; cb < kCC; cb += 32) {
            float x[32], y[32];
            tmem_ld32(lb + L::T_DD + cb, x);        // dO' D^T row (side 0) or Y = dd D^T row (side 1)
            tmem_ld32(lb + L::T_QK + cb, y);        // Q K^T row or K K^T row
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int s = cb + i;
                const float ex = expf(lt - lam[s]);
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
                Fs[t * kCC + ((s + t) & (kCC - 1))] = f;
                // pair sums: token s gets sum_{s' < s} e_{s'} from rows u >= s (side 0) or u > s (side 1)
                const float v = warp_sum(in || (side == 0 && s == t) ? pre : 0.f);
                if (lane == 0) pairp[warp * kCC + s] = v;
                pre += e;
            }
        }
        if (side == 0) {
            s_a[t] = Gt * scale * dot;
        } else {
            const float kr = Gt * dot + krs;        // r_t . dd_t
            s_c[t] = -Gt * bt * dot;
            s_dbm[t] = ddv[t] - kr;
            s_rdr[t] = -bt * kr;
        }
    }

    // ---- phase C: the T4 operands over the freed images once T2 completed
    if (tid == 0 && !dead_b && !mbar_wait(&bars[1], 0, a.err)) *dead = 1;
    __syncthreads();
    const bool dead_c = *dead != 0;
    tc_fence_after();
    if (!dead_c) {
        for (int it = tid; it < 8 * 128; it += 256) {
            const int ch = it >> 7, row = it & 127, t = row & (kCC - 1);
            float f1[8], f2[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int s = ch * 8 + i;
                if (row < kCC) {
                    f1[i] = F1s[t * kCC + ((s + t) & (kCC - 1))];
                    f2[i] = 0.f;
                } else {
                    f1[i] = F2s[t * kCC + ((s + t) & (kCC - 1))] + F2s[s * kCC + ((t + s) & (kCC - 1))];
                    f2[i] = scale * F1s[s * kCC + ((t + s) & (kCC - 1))];
                }
            }
            const uint32_t off = sw128_chunk(row, ch);
            split_store8(sm + L::OFF_A1H + off, sm + L::OFF_A1L + off, f1);
            split_store8(sm + L::OFF_A2H + off, sm + L::OFF_A2L + off, f2);
        }
        for (int it = tid; it < 8 * DK; it += 256) {
            const int ch = it / DK, d = it - ch * DK;
            uint16_t kv[8], qv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int s = ch * 8 + i;
                kv[i] = s < nt ? a.k[(tokbase + s) * DK + d] : static_cast<uint16_t>(0);
                qv[i] = s < nt ? a.q[(tokbase + s) * DK + d] : static_cast<uint16_t>(0);
            }
            const uint32_t off = sw128_chunk(d, ch);
            *reinterpret_cast<uint4*>(sm + L::OFF_KT + off) =
                make_uint4(kv[0] | (uint32_t(kv[1]) << 16), kv[2] | (uint32_t(kv[3]) << 16),
                           kv[4] | (uint32_t(kv[5]) << 16), kv[6] | (uint32_t(kv[7]) << 16));
            *reinterpret_cast<uint4*>(sm + L::OFF_QT + off) =
                make_uint4(qv[0] | (uint32_t(qv[1]) << 16), qv[2] | (uint32_t(qv[3]) << 16),
                           qv[4] | (uint32_t(qv[5]) << 16), qv[6] | (uint32_t(qv[7]) << 16));
        }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0 && !dead_c) {
        tc_fence_after();
        constexpr uint32_t idN = idesc_bf16(128, DK, false, false);
        const uint32_t pa[4] = {sbase + L::OFF_A1H, sbase + L::OFF_A1L, sbase + L::OFF_A2H, sbase + L::OFF_A2L};
        const uint32_t pb[4] = {sbase + L::OFF_KT, sbase + L::OFF_KT, sbase + L::OFF_QT, sbase + L::OFF_QT};
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_bf16_ss(tmem + L::T_X4, sdesc_sw128(pa[p] + kk * 32, 16, 1024),
                             sdesc_sw128(pb[p] + kk * 32, 16, 1024), idN, (p > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars[2]);
    }
    // k_t . X_e on the dk side (k_t read from the transposed k tile)
    if (tid >= 64 && tid < 128 && !dead_c) {
        const int t = tid - kCC;
        const uint32_t lb = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        float dot = 0.f;
#pragma unroll 1
        for (int cb = 0; cb < DK; cb += 32) {
            float x[32];
            tmem_ld32(lb + L::T_XE + cb, x);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i)
                dot = fmaf(x[i], bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sm + L::OFF_KT +
                                                                                     sw128_off(cb + i, t))),
                           dot);
        }
        s_e[t] = expf(lL - lam[t]) * dot;
    }
    __syncthreads();
    if (tid < kCC && tid < nt && !dead_c) {
        const int t = tid;
        float base = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) base += basep[w];
        float sa = 0.f, scc = 0.f, se = 0.f;
        for (int u = t; u < kCC; ++u) sa += s_a[u];
        for (int u = t + 1; u < kCC; ++u) scc += s_c[u];
        for (int s = 0; s < t; ++s) se += s_e[s];
        const float pair = pairp[t] + pairp[kCC + t] + pairp[2 * kCC + t] + pairp[3 * kCC + t];
        const float dlogg = GL * base + sa + scc + se + pair + s_rdr[t];
        const long tok = tokbase + t;
        a.dlogg[tok] = dlogg;
        const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
        const float xg = load_gate(a.a, tok, a.gate_dtype) + dtb;
        a.da[tok] = dlogg * (-expf(a.A_log[h])) * (xg > 20.f ? 1.f : sigmoid_f(xg));
        const float sb = sigmoid_f(load_gate(a.b, tok, a.gate_dtype));
        a.db[tok] = s_dbm[t] * ms[t] * sb * (1.f - sb);
    }

    // ---- phase D: dq, dk (warps w and w + 4 share lanes 32 (w % 4) .. + 31, half the columns each)
    if (tid == 0 && !dead_c && !mbar_wait(&bars[2], 0, a.err)) *dead = 1;
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
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}


// Workspace of the chunked backward: gate vectors | M, P, A | S checkpoints | d rows |
// Sb checkpoints | dd rows | dlogg, each 256-byte aligned.
struct CbWs {
    size_t gv, mp, ckS, ckD, ckSb, ckDD, dlogg, total;
};
CbWs cb_ws(size_t bh, int T, int dk, int dv) {
    const size_t n = (static_cast<size_t>(T) + kCC - 1) / kCC, nc = bh * n;
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    CbWs w;
    w.gv = 0;
    w.mp = w.gv + al(nc * 3 * kCC * 4);
    w.ckS = w.mp + al(nc * 3 * kCC * kCC * 4);
    w.ckD = w.ckS + al(nc * dk * dv * 4);
    w.ckSb = w.ckD + al(nc * kCC * dv * 4);
    w.ckDD = w.ckSb + al(nc * dk * dv * 4);
    w.dlogg = w.ckDD + al(nc * kCC * dv * 4);
    w.total = w.dlogg + al(bh * static_cast<size_t>(T) * 4) + 1024;
    return w;
}

template <int DK, int DV>
int launch_cb(const CbArgs& a, cudaStream_t st) {
    static int attr_ok = -1;                       // set once per process: the kernels' shared-memory limits
    if (attr_ok < 0)
        attr_ok = cudaFuncSetAttribute(cb_mats_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       MatsSmem<DK>::BYTES) == cudaSuccess &&
                          cudaFuncSetAttribute(cb_forward_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               RecSmem<DK>::BYTES) == cudaSuccess &&
                          cudaFuncSetAttribute(cb_reverse_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               RecSmem<DK>::BYTES) == cudaSuccess &&
                          cudaFuncSetAttribute(cb_grads_tc_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               GtLayout<DK, DV>::BYTES) == cudaSuccess
                      ? 1
                      : 0;
    if (!attr_ok) return fail(GDN_ERR_CUDA, "gdn_prefill_bwd (chunked): cannot configure the kernels' shared memory");
    const unsigned nchunks = static_cast<unsigned>(static_cast<long>(a.B) * a.H * a.n);
    const dim3 rec(a.B * a.H, DV / 64);
    cb_mats_kernel<DK><<<nchunks, 128, MatsSmem<DK>::BYTES, st>>>(a);
    int s = launch_status("gdn_prefill_bwd (chunk matrices)");
    if (s != GDN_OK) return s;
    cb_forward_kernel<DK, DV><<<rec, 256, RecSmem<DK>::BYTES, st>>>(a);
    if ((s = launch_status("gdn_prefill_bwd (chunk forward)")) != GDN_OK) return s;
    cb_reverse_kernel<DK, DV><<<rec, 256, RecSmem<DK>::BYTES, st>>>(a);
    if ((s = launch_status("gdn_prefill_bwd (chunk reverse)")) != GDN_OK) return s;
    cb_grads_tc_kernel<DK, DV><<<nchunks, 256, GtLayout<DK, DV>::BYTES, st>>>(a);
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
    ar.mp = reinterpret_cast<float*>(ws + wl.mp);
    ar.ckS = reinterpret_cast<float*>(ws + wl.ckS);
    ar.ckD = reinterpret_cast<float*>(ws + wl.ckD);
    ar.ckSb = reinterpret_cast<float*>(ws + wl.ckSb);
    ar.ckDD = reinterpret_cast<float*>(ws + wl.ckDD);
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
    launch_bwd_head_sums(A_log, a, gate_dtype, dt_bias, dt_bias_vec, ar.dlogg, da, dA_log, ddt_bias, B, T, H, st);
    return launch_status("gdn_prefill_bwd (heads)");
}

}  // namespace gdn
