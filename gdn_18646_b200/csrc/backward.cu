// backward.cu -- gradients of the gated delta rule prefill (dq, dk, dv, da, db,
// dA_log, ddt_bias and the initial state), for training use.
//
// The reference has no backward.  This is the token-recurrent derivative (the
// same recurrence as the forward, per token: S' = g S_p, r = S'^T k,
// d = b'(v - r), S_n = S' + k d^T, o = m scale q^T S_n), in four launches:
//
//   bwd_states_kernel   the forward recurrence again, storing the state S_p
//                       before every token (fp32 [B,H,T,dk,dv]) and k . S_p per
//                       value column;
//   bwd_reverse_kernel  the reverse recurrence of dS (the gradient of S_n):
//                       dS += scale q (m dO)^T, dd = dS^T k, dv = b' dd,
//                       dS <- g (dS - b' k dd^T); per token it also reads S_p and
//                       leaves, per block of value columns, the row sums of
//                       S_p (m dO) and dS delta + g S_p dr and the scalars of
//                       db' and dg (dg = <S_p, dS + k dr^T>), so dS is never stored;
//   bwd_finish_kernel   per token, those partials summed over the column blocks:
//                       dq, dk, and the chain rule through g = exp(-exp(A_log)
//                       softplus(a + dt_bias)) and b' = sigmoid(b) m into da, db;
//   bwd_head_kernel     dA_log and ddt_bias, summed per head in token order.
//
// The recurrences keep 32 rows of a value column per thread, so their column
// reductions stay inside a warp; fp32 on CUDA cores throughout.  The traffic is
// the state workspace, written once and read once (2 x 4 dk dv bytes per token
// and head).  Restates oracle prefill_backward (pinned to finite differences).
#include "common.cuh"

namespace gdn {
namespace {

struct BwdArgs {
    const uint16_t* q;         // [B,H,T,DK] bf16
    const uint16_t* k;
    const uint16_t* v;         // [B,H,T,DV] bf16
    const float* A_log;        // [H]
    const void* a;             // [B,H,T] gate_dtype
    const void* b;
    int gate_dtype;
    float dt_bias;
    const float* dt_bias_vec;  // [H] or null
    const float* mask;         // [B,T] or null
    const float* state_in;     // [B,H,DK,DV] or null
    const void* dO;            // [B,H,T,DV] in do_dtype
    int do_dtype;
    const float* dS_final;     // [B,H,DK,DV] or null
    float* dq;                 // [B,H,T,DK] f32
    float* dk;
    float* dv;                 // [B,H,T,DV] f32
    float* da;                 // [B,H,T] f32
    float* db;
    float* dA_log;             // [H] f32
    float* ddt_bias;           // [H] f32
    float* dstate_in;          // [B,H,DK,DV] f32 or null
    float* states;             // workspace: S_p per token of the window [B*H][WT][DK][DV]
    float* rp;                 // workspace: [B*H][WT][DV], k . S_p per value column
    float* part;               // workspace: per token of the window and column block, row sums and scalars
    float* dlogg;              // workspace: [B,H,T]
    int B, T, H;
    float scale;
    // token window of a launch: tokens [t0, t1); the window buffers (states, rp, part) hold
    // WT tokens per sequence-head, indexed from t0
    int t0, t1, WT;
    const float* S0;           // states kernel: the state before token t0, S0 + bh * S0_stride; null = zeros
    long S0_stride;
    float* ckpt;               // checkpoint pass: the state before every token t % win == 0,
    int win, nwin;             //   ckpt[(bh * nwin + t / win) * DK * DV]; no per-token state stored
    const float* dS_in;        // reverse kernel: the gradient of the state after token t1 - 1 (null = 0)
    float* dS_out;             //   and, at the end, of the state before token t0 (null = not stored)
};

__device__ __forceinline__ float bf16_at(const uint16_t* p, long i) { return bf16_bits_to_f32(p[i]); }

// decay and masked write strength of token t of sequence-head bh
__device__ __forceinline__ void gate_of(const BwdArgs& a, int bh, int t, float& g, float& bm) {
    const int h = bh % a.H, bi = bh / a.H;
    const long i = static_cast<long>(bh) * a.T + t;
    const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
    g = expf(-expf(a.A_log[h]) * softplus_f(load_gate(a.a, i, a.gate_dtype) + dtb));
    const float m = a.mask ? a.mask[static_cast<long>(bi) * a.T + t] : 1.f;
    bm = sigmoid_f(load_gate(a.b, i, a.gate_dtype)) * m;
}

// The recurrences keep 32 state rows of one value column per thread: a column
// is spread over PARTS = dk/32 lanes of a warp (its dot products add the parts
// with log2(PARTS) shuffles) and a warp covers COLS = 32/PARTS columns, so one
// store instruction writes whole 32-byte sectors (PARTS rows x COLS columns).
// A CTA of 4 warps covers 4 * COLS adjacent columns and shares the staged
// tokens; config 1 (B*H = 64, dv = 128) runs 1024 warps.  (16 rows per thread
// doubled the warps but wrote half sectors, and ran 3x slower.)
template <int DK>
struct RecLayout {
    static constexpr int ROWS = 32;                // rows per thread
    static constexpr int PARTS = DK / ROWS;        // threads per column
    static constexpr int COLS = 32 / PARTS;        // columns per warp
    static constexpr int WARPS = 4;
    static constexpr int CTA_COLS = COLS * WARPS;  // columns per CTA
    static constexpr int THREADS = 32 * WARPS;
};

// Tokens a recurrence stages in shared memory at once (one global round trip
// per block instead of one per token).
constexpr int kTB = 32;

template <int PARTS_, int COLS_>
__device__ __forceinline__ float sum_parts(float x) {
#pragma unroll
    for (int o = COLS_; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Forward recurrence, storing S_p (the state before each token) and rp = k . S_p
// per value column.  Grid (B*H, DV/CTA_COLS).
template <int DK, int DV>
__global__ void __launch_bounds__(128) bwd_states_kernel(const BwdArgs a) {
    using L = RecLayout<DK>;
    const int bh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int jl = lane % L::COLS;
    const int jc = warp * L::COLS + jl;                // column within the CTA
    const int j = blockIdx.y * L::CTA_COLS + jc;
    const int i0 = (lane / L::COLS) * L::ROWS;        // first row of this thread
    __shared__ float ks[kTB][DK];
    __shared__ float vs[kTB][L::CTA_COLS];
    __shared__ float gs[kTB], bs[kTB];
    float S[L::ROWS];
    const long s0 = static_cast<long>(bh) * a.S0_stride;
#pragma unroll
    for (int i = 0; i < L::ROWS; ++i) S[i] = a.S0 ? a.S0[s0 + static_cast<long>(i0 + i) * DV + j] : 0.f;
    for (int tb = a.t0; tb < a.t1; tb += kTB) {
        const int nt = min(kTB, a.t1 - tb);
        const long tok0 = static_cast<long>(bh) * a.T + tb;
        const long loc0 = static_cast<long>(bh) * a.WT + (tb - a.t0);      // window-local token index
        __syncthreads();
        for (int e = tid; e < nt * DK; e += L::THREADS) ks[e / DK][e % DK] = bf16_at(a.k, tok0 * DK + e);
        for (int e = tid; e < nt * L::CTA_COLS; e += L::THREADS)
            vs[e / L::CTA_COLS][e % L::CTA_COLS] =
                bf16_at(a.v, (tok0 + e / L::CTA_COLS) * DV + blockIdx.y * L::CTA_COLS + e % L::CTA_COLS);
        if (tid < nt) gate_of(a, bh, tb + tid, gs[tid], bs[tid]);
        __syncthreads();
        for (int u = 0; u < nt; ++u) {
            const long loc = loc0 + u;
            if (a.ckpt) {
                if ((tb + u) % a.win == 0) {
                    float* out = a.ckpt + ((static_cast<long>(bh) * a.nwin + (tb + u) / a.win) * DK + i0) * DV + j;
#pragma unroll
                    for (int i = 0; i < L::ROWS; ++i) out[static_cast<long>(i) * DV] = S[i];
                }
            } else {
                float* out = a.states + (loc * DK + i0) * DV + j;
#pragma unroll
                for (int i = 0; i < L::ROWS; ++i) out[static_cast<long>(i) * DV] = S[i];
            }
            const float* kk = ks[u] + i0;
            const float g = gs[u], bm = bs[u];
            float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
            for (int i = 0; i < L::ROWS; i += 4) {
                r0 = fmaf(kk[i], S[i], r0);
                r1 = fmaf(kk[i + 1], S[i + 1], r1);
                r2 = fmaf(kk[i + 2], S[i + 2], r2);
                r3 = fmaf(kk[i + 3], S[i + 3], r3);
            }
            const float rp = sum_parts<L::PARTS, L::COLS>((r0 + r1) + (r2 + r3));
            if (i0 == 0 && !a.ckpt) a.rp[loc * DV + j] = rp;
            const float d = bm * (vs[u][jc] - g * rp);
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) S[i] = fmaf(kk[i], d, g * S[i]);
        }
    }
}

// Partial sums a reverse CTA leaves per token: X_i = S_p[i,:].(m dO), Y_i = dS[i,:].delta
// + g S_p[i,:].dr over its columns, then p_db = dd.(v - r), p_ddo = delta.(m dO),
// p_rdr = dr.rp, p_sds = <S_p, dS>.
template <int DK>
struct PartLayout {
    static constexpr int STRIDE = 2 * DK + 4;
};

// Sum 32 per-row values over the COLS lanes of a warp that share rows (lanes
// p*COLS + jl, jl < COLS): a butterfly reduce-scatter, after which lane jl holds
// the sums of rows (32/COLS) * jl + t, t < 32/COLS, in v[t].
template <int COLS>
__device__ __forceinline__ void rows_reduce_scatter(float (&v)[32], int jl) {
    int n = 32;
#pragma unroll
    for (int m = COLS / 2; m >= 1; m >>= 1) {
        n >>= 1;
        const bool upper = (jl & m) != 0;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            if (t < n) {
                const float send = upper ? v[t] : v[t + n];
                const float keep = upper ? v[t + n] : v[t];
                v[t] = keep + __shfl_xor_sync(0xffffffffu, send, m);
            }
        }
    }
}

constexpr int kRevTB = 16;   // tokens the reverse recurrence stages at once

// Reverse recurrence of dS (the gradient of S_n) with every token's dq/dk/gate
// work folded in, so no per-token dS is stored.  Per token: dS += scale q (m dO)^T,
// dd = dS^T k, dv = b' dd; with S_p from the forward pass, this CTA's partial row
// sums X, Y and scalars go to the workspace (summed over column blocks by
// bwd_finish_kernel); then dS <- g (dS - b' k dd^T).  Grid (B*H, DV/CTA_COLS).
template <int DK, int DV>
__global__ void __launch_bounds__(128) bwd_reverse_kernel(const BwdArgs a) {
    using L = RecLayout<DK>;
    constexpr int NCB = DV / L::CTA_COLS, PST = PartLayout<DK>::STRIDE, RPL = L::ROWS / L::COLS;
    const int bh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int jl = lane % L::COLS;
    const int jc = warp * L::COLS + jl;
    const int j = blockIdx.y * L::CTA_COLS + jc;
    const int i0 = (lane / L::COLS) * L::ROWS;
    const int bi = bh / a.H;
    __shared__ float ks[kRevTB][DK], qs[kRevTB][DK];
    __shared__ float mdo[kRevTB][L::CTA_COLS], vv[kRevTB][L::CTA_COLS], rps[kRevTB][L::CTA_COLS];
    __shared__ float gs[kRevTB], bs[kRevTB];
    __shared__ float xr[2][L::WARPS][DK], yr[2][L::WARPS][DK];
    __shared__ float scr[2][L::WARPS][4];
    float dS[L::ROWS];
    const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
    for (int i = 0; i < L::ROWS; ++i) dS[i] = a.dS_in ? a.dS_in[s0 + static_cast<long>(i0 + i) * DV + j] : 0.f;
    // S_p of the token processed next, loaded one token ahead (the loads are the
    // long-latency part of a step); window-local token indices
    float SpN[L::ROWS];
    const long loc_first = static_cast<long>(bh) * a.WT;
    {
        const float* sp = a.states + ((loc_first + (a.t1 - 1 - a.t0)) * DK + i0) * DV + j;
#pragma unroll
        for (int i = 0; i < L::ROWS; ++i) SpN[i] = sp[static_cast<long>(i) * DV];
    }
    for (int tend = a.t1; tend > a.t0; tend -= kRevTB) {
        const int tb = max(a.t0, tend - kRevTB), nt = tend - tb;
        const long tok0 = static_cast<long>(bh) * a.T + tb;
        const long loc0 = loc_first + (tb - a.t0);
        __syncthreads();
        for (int e = tid; e < nt * DK; e += L::THREADS) {
            ks[e / DK][e % DK] = bf16_at(a.k, tok0 * DK + e);
            qs[e / DK][e % DK] = bf16_at(a.q, tok0 * DK + e);
        }
        for (int e = tid; e < nt * L::CTA_COLS; e += L::THREADS) {
            const int u = e / L::CTA_COLS, c = e % L::CTA_COLS;
            const long idx = (tok0 + u) * DV + blockIdx.y * L::CTA_COLS + c;
            const float m = a.mask ? a.mask[static_cast<long>(bi) * a.T + tb + u] : 1.f;
            mdo[u][c] = m * (a.do_dtype == GDN_DTYPE_BF16 ? bf16_at(static_cast<const uint16_t*>(a.dO), idx)
                                                          : static_cast<const float*>(a.dO)[idx]);
            vv[u][c] = bf16_at(a.v, idx);
            rps[u][c] = a.rp[(loc0 + u) * DV + blockIdx.y * L::CTA_COLS + c];
        }
        if (tid < nt) gate_of(a, bh, tb + tid, gs[tid], bs[tid]);
        __syncthreads();
        for (int u = nt - 1; u >= 0; --u) {
            const long tok = tok0 + u;
            const long loc = loc0 + u;
            const float* kk = ks[u] + i0;
            const float* qq = qs[u] + i0;
            const float dos = mdo[u][jc];
            const float sdo = a.scale * dos;
            const float g = gs[u], bm = bs[u];
            // S_p of these rows (forward pass), loaded during the previous step; start the next
            float Sp[L::ROWS];
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) Sp[i] = SpN[i];
            if (loc > loc_first) {
                const float* sp = a.states + ((loc - 1) * DK + i0) * DV + j;
#pragma unroll
                for (int i = 0; i < L::ROWS; ++i) SpN[i] = sp[static_cast<long>(i) * DV];
            }
            float e0 = 0.f, e1 = 0.f, e2 = 0.f, e3 = 0.f;
#pragma unroll
            for (int i = 0; i < L::ROWS; i += 4) {
                dS[i] = fmaf(qq[i], sdo, dS[i]);
                dS[i + 1] = fmaf(qq[i + 1], sdo, dS[i + 1]);
                dS[i + 2] = fmaf(qq[i + 2], sdo, dS[i + 2]);
                dS[i + 3] = fmaf(qq[i + 3], sdo, dS[i + 3]);
                e0 = fmaf(kk[i], dS[i], e0);
                e1 = fmaf(kk[i + 1], dS[i + 1], e1);
                e2 = fmaf(kk[i + 2], dS[i + 2], e2);
                e3 = fmaf(kk[i + 3], dS[i + 3], e3);
            }
            const float ddj = sum_parts<L::PARTS, L::COLS>((e0 + e1) + (e2 + e3));
            if (i0 == 0) a.dv[tok * DV + j] = bm * ddj;
            const float rp = rps[u][jc], vj = vv[u][jc];
            const float r = g * rp, dlt = bm * (vj - r), dr = -bm * ddj, gdr = g * dr;
            // products for the row sums (dq, dk) and <S_p, dS>
            float X[32], Y[32];
            float sds = 0.f;
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) {
                X[i] = Sp[i] * dos;
                Y[i] = fmaf(dS[i], dlt, Sp[i] * gdr);
                sds = fmaf(Sp[i], dS[i], sds);
            }
            float c0 = 0.f, c1 = 0.f, c2 = 0.f;        // column scalars, once per column
            if (i0 == 0) {
                c0 = ddj * (vj - r);
                c1 = dlt * dos;
                c2 = dr * rp;
            }
            rows_reduce_scatter<L::COLS>(X, jl);
            rows_reduce_scatter<L::COLS>(Y, jl);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sds += __shfl_xor_sync(0xffffffffu, sds, o);
            // the column scalars live on lanes 0 .. COLS-1 (zero elsewhere): their sum
            // reaches lane 0, the only reader, in log2(COLS) steps
#pragma unroll
            for (int o = L::COLS / 2; o > 0; o >>= 1) {
                c0 += __shfl_xor_sync(0xffffffffu, c0, o);
                c1 += __shfl_xor_sync(0xffffffffu, c1, o);
                c2 += __shfl_xor_sync(0xffffffffu, c2, o);
            }
            const int pb = u & 1;
#pragma unroll
            for (int t = 0; t < RPL; ++t) {
                xr[pb][warp][i0 + RPL * jl + t] = X[t];
                yr[pb][warp][i0 + RPL * jl + t] = Y[t];
            }
            if (lane == 0) {
                scr[pb][warp][0] = c0;
                scr[pb][warp][1] = c1;
                scr[pb][warp][2] = c2;
                scr[pb][warp][3] = sds;
            }
            __syncthreads();
            float* pp = a.part + (loc * NCB + blockIdx.y) * PST;
            for (int i = tid; i < DK; i += L::THREADS) {
                float xs = 0.f, ys = 0.f;
#pragma unroll
                for (int w = 0; w < L::WARPS; ++w) {
                    xs += xr[pb][w][i];
                    ys += yr[pb][w][i];
                }
                pp[i] = xs;
                pp[DK + i] = ys;
            }
            if (tid < 4) {
                float t4 = 0.f;
#pragma unroll
                for (int w = 0; w < L::WARPS; ++w) t4 += scr[pb][w][tid];
                pp[2 * DK + tid] = t4;
            }
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) dS[i] = g * fmaf(kk[i], dr, dS[i]);
        }
    }
    if (a.dS_out) {
#pragma unroll
        for (int i = 0; i < L::ROWS; ++i) a.dS_out[s0 + static_cast<long>(i0 + i) * DV + j] = dS[i];
    }
}

// Per token: the column blocks' partials summed into dq, dk, da, db (and dlog g for the
// head sums).  One CTA of 128 threads per token.
template <int DK, int DV>
__global__ void __launch_bounds__(128) bwd_finish_kernel(const BwdArgs a) {
    constexpr int NCB = DV / RecLayout<DK>::CTA_COLS, PST = PartLayout<DK>::STRIDE;
    const int nw = a.t1 - a.t0;                   // one CTA per token of the window
    const int bh = static_cast<int>(blockIdx.x / nw), t = a.t0 + static_cast<int>(blockIdx.x % nw);
    const long tok = static_cast<long>(bh) * a.T + t;
    const int bi = bh / a.H, h = bh % a.H;
    const int tid = threadIdx.x;
    const float* pp = a.part + (static_cast<long>(bh) * a.WT + (t - a.t0)) * NCB * PST;
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb)
#pragma unroll
        for (int q = 0; q < 4; ++q) sc[q] += pp[cb * PST + 2 * DK + q];
    float g, bm;
    gate_of(a, bh, t, g, bm);
    for (int i = tid; i < DK; i += 128) {
        float X = 0.f, Y = 0.f;
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
            X += pp[cb * PST + i];
            Y += pp[cb * PST + DK + i];
        }
        a.dq[tok * DK + i] = a.scale * fmaf(g, X, bf16_at(a.k, tok * DK + i) * sc[1]);
        a.dk[tok * DK + i] = Y;
    }
    if (tid == 0) {
        const float m = a.mask ? a.mask[static_cast<long>(bi) * a.T + t] : 1.f;
        const float dg = sc[3] + sc[2];                // <S_p, dS + k dr^T> = <S_p, dS> + dr . rp
        const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
        const float x = load_gate(a.a, tok, a.gate_dtype) + dtb;
        const float dlogg = dg * g;
        a.dlogg[tok] = dlogg;
        a.da[tok] = dlogg * (-expf(a.A_log[h])) * (x > 20.f ? 1.f : sigmoid_f(x));
        const float sb = sigmoid_f(load_gate(a.b, tok, a.gate_dtype));
        a.db[tok] = sc[0] * m * sb * (1.f - sb);
    }
}

// dA_log[h] = sum dlogg * log g, ddt_bias[h] = sum da over (b, t), in order.  One CTA per head.
// A cluster of kHeadSplit CTAs per head, each summing every kHeadSplit-th token
// block of the head's B*T tokens; rank 0 adds the CTAs' sums in rank order (the
// peers' shared memory, read after a cluster barrier), so the result does not
// depend on scheduling.
constexpr int kHeadSplit = 8;
__global__ void __launch_bounds__(256) bwd_head_kernel(const BwdArgs a) {
    const int h = blockIdx.x / kHeadSplit, rank = blockIdx.x % kHeadSplit, tid = threadIdx.x;
    __shared__ float r0[256], r1[256];
    const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
    const float Aneg = -expf(a.A_log[h]);
    float s0 = 0.f, s1 = 0.f;
    for (int bi = 0; bi < a.B; ++bi) {
        const long base = (static_cast<long>(bi) * a.H + h) * a.T;
        for (int t = rank * 256 + tid; t < a.T; t += 256 * kHeadSplit) {
            const float logg = Aneg * softplus_f(load_gate(a.a, base + t, a.gate_dtype) + dtb);
            s0 = fmaf(a.dlogg[base + t], logg, s0);
            s1 += a.da[base + t];
        }
    }
    r0[tid] = s0;
    r1[tid] = s1;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (tid < s) {
            r0[tid] += r0[tid + s];
            r1[tid] += r1[tid + s];
        }
        __syncthreads();
    }
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (rank == 0 && tid == 0) {
        float t0 = 0.f, t1 = 0.f;
        for (int q = 0; q < kHeadSplit; ++q) {
            uint32_t p0, p1;
            float v0, v1;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(p0) : "r"(smem_u32(&r0[0])), "r"(q));
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(p1) : "r"(smem_u32(&r1[0])), "r"(q));
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v0) : "r"(p0) : "memory");
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v1) : "r"(p1) : "memory");
            t0 += v0;
            t1 += v1;
        }
        a.dA_log[h] = t0;
        a.ddt_bias[h] = t1;
    }
    // no CTA leaves (and releases its shared memory) before rank 0 has read it
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

int launch_head(const BwdArgs& a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.H * kHeadSplit);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kHeadSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, bwd_head_kernel, a);
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_prefill_bwd (heads): launch failed: %s", cudaGetErrorString(e));
    return launch_status("gdn_prefill_bwd (heads)");
}

// The backward runs window by window, last window first, so that only one window's
// per-token states are in the workspace at a time: a checkpoint pass of the forward
// recurrence over the whole sequence stores the state at every window start, then
// per window the states kernel recomputes the window's per-token states from its
// checkpoint, the reverse kernel carries dS through the window (in and out of the
// carry buffer) and the finish kernel completes its tokens.  One window covering
// the sequence needs no checkpoint pass.
template <int DK, int DV>
int launch_bwd(BwdArgs a, int W, float* ckpt, float* carry, cudaStream_t st) {
    const dim3 rec(a.B * a.H, DV / RecLayout<DK>::CTA_COLS);
    const int nwin = (a.T + W - 1) / W;
    const float* state_in = a.state_in;
    int s;
    a.WT = W;
    a.win = W;
    a.nwin = nwin;
    if (nwin > 1) {
        a.t0 = 0;
        a.t1 = a.T;
        a.S0 = state_in;
        a.S0_stride = static_cast<long>(DK) * DV;
        a.ckpt = ckpt;
        bwd_states_kernel<DK, DV><<<rec, RecLayout<DK>::THREADS, 0, st>>>(a);
        if ((s = launch_status("gdn_prefill_bwd (checkpoints)")) != GDN_OK) return s;
    }
    a.ckpt = nullptr;
    for (int w = nwin - 1; w >= 0; --w) {
        a.t0 = w * W;
        a.t1 = a.t0 + W < a.T ? a.t0 + W : a.T;
        a.S0 = nwin > 1 ? ckpt + static_cast<long>(w) * DK * DV : state_in;
        a.S0_stride = static_cast<long>(nwin > 1 ? nwin : 1) * DK * DV;
        bwd_states_kernel<DK, DV><<<rec, RecLayout<DK>::THREADS, 0, st>>>(a);
        if ((s = launch_status("gdn_prefill_bwd (states)")) != GDN_OK) return s;
        a.dS_in = w == nwin - 1 ? a.dS_final : carry;
        a.dS_out = w == 0 ? a.dstate_in : carry;
        bwd_reverse_kernel<DK, DV><<<rec, RecLayout<DK>::THREADS, 0, st>>>(a);
        if ((s = launch_status("gdn_prefill_bwd (reverse)")) != GDN_OK) return s;
        bwd_finish_kernel<DK, DV><<<static_cast<unsigned>(static_cast<long>(a.B) * a.H * (a.t1 - a.t0)), 128, 0, st>>>(a);
        if ((s = launch_status("gdn_prefill_bwd (finish)")) != GDN_OK) return s;
    }
    return launch_head(a, st);
}

}  // namespace
}  // namespace gdn

namespace gdn {

// The head sums for the chunked backward (backward_chunked.cu), which leaves dlogg and da in
// the same layouts.
int launch_bwd_head_sums(const float* A_log, const void* a, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                         const float* dlogg, const float* da, float* dA_log, float* ddt_bias, int B, int T, int H,
                         cudaStream_t st) {
    BwdArgs ar{};
    ar.A_log = A_log;
    ar.a = a;
    ar.gate_dtype = gate_dtype;
    ar.dt_bias = dt_bias;
    ar.dt_bias_vec = dt_bias_vec;
    ar.dlogg = const_cast<float*>(dlogg);
    ar.da = const_cast<float*>(da);
    ar.dA_log = dA_log;
    ar.ddt_bias = ddt_bias;
    ar.B = B;
    ar.T = T;
    ar.H = H;
    return launch_head(ar, st);
}

size_t prefill_bwd_chunked_workspace(int B, int T, int H, int dk, int dv);
int prefill_bwd_chunked(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                        const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec, const float* mask,
                        const float* state_in, const void* dO, int do_dtype, const float* dS_final, float* dq, float* dk,
                        float* dv, float* da, float* db, float* dA_log, float* ddt_bias, float* dstate_in, int B, int T,
                        int H, int dkd, int dvd, float scale, void* workspace, cudaStream_t st);

namespace {
thread_local int t_bwd_window = 0;   // gdn_prefill_bwd_set_window: the calling thread's window (0 = automatic)

// Window length in tokens: the calling thread's setting, else max(256, sqrt T) rounded up to
// 32 tokens (the checkpoints and one window's states together, B H dk dv 4 (T / W + W) bytes,
// are then near their minimum without many short windows); never more than T.
thread_local int t_bwd_algo = GDN_BWD_AUTO;   // gdn_prefill_bwd_set_algorithm: the calling thread's choice

bool bwd_chunked() { return t_bwd_algo != GDN_BWD_TOKEN; }   // the default is the chunked backward

int bwd_window(int T) {
    int w = t_bwd_window;
    if (w <= 0) {
        const int r = (static_cast<int>(sqrtf(static_cast<float>(T))) + 31) / 32 * 32;
        w = r > 256 ? r : 256;
    }
    return w < T ? w : T;
}

// Workspace: checkpoints [bh][nwin][dk][dv] (several windows only) | window states [bh][W][dk][dv] |
// rp [bh][W][dv] | partials [bh][W][column blocks][2 dk + 4] | dlogg [bh][T] | dS carry [bh][dk][dv]
struct BwdWs {
    size_t ckpt, states, rp, part, dlogg, carry, total;
};
BwdWs bwd_ws(size_t bh, int T, int dk, int dv, int W) {
    const int cta_cols = dk == 128 ? RecLayout<128>::CTA_COLS : RecLayout<64>::CTA_COLS;
    const size_t ncb = static_cast<size_t>(dv / cta_cols);
    const size_t nwin = (static_cast<size_t>(T) + W - 1) / W;
    const size_t sd = static_cast<size_t>(dk) * dv * 4;
    BwdWs w;
    w.ckpt = 0;
    w.states = w.ckpt + (nwin > 1 ? bh * nwin * sd : 0);
    w.rp = w.states + bh * W * sd;
    w.part = w.rp + bh * W * dv * 4;
    w.dlogg = w.part + bh * W * ncb * (2 * dk + 4) * 4;
    w.carry = w.dlogg + (bh * T * 4 + 255) / 256 * 256;
    w.total = w.carry + bh * sd + 1024;
    return w;
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_bwd_set_window(int tokens) {
    if (tokens < 0) return gdn::fail(GDN_ERR_ARG, "gdn_prefill_bwd_set_window: tokens must be >= 0 (got %d)", tokens);
    gdn::t_bwd_window = tokens;
    return GDN_OK;
}

extern "C" int gdn_prefill_bwd_set_algorithm(int algorithm) {
    if (algorithm != GDN_BWD_AUTO && algorithm != GDN_BWD_TOKEN && algorithm != GDN_BWD_CHUNKED)
        return gdn::fail(GDN_ERR_ARG, "gdn_prefill_bwd_set_algorithm: unknown algorithm %d", algorithm);
    gdn::t_bwd_algo = algorithm;
    return GDN_OK;
}

extern "C" size_t gdn_prefill_bwd_workspace_bytes(int B, int T, int H, int dk, int dv) {
    if (B <= 0 || T <= 0 || H <= 0 || !(dk == 64 || dk == 128) || !(dv == 64 || dv == 128)) return 0;
    if (gdn::bwd_chunked()) return gdn::prefill_bwd_chunked_workspace(B, T, H, dk, dv);
    return gdn::bwd_ws(static_cast<size_t>(B) * H, T, dk, dv, gdn::bwd_window(T)).total;
}

extern "C" int gdn_prefill_bwd(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                               const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                               const float* mask, const float* state_in, const void* dO, int do_dtype,
                               const float* dS_final, float* dq, float* dk, float* dv, float* da, float* db,
                               float* dA_log, float* ddt_bias, float* dstate_in, int B, int T, int H, int dkd,
                               int dvd, float scale, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace gdn;
    if (!q || !k || !v || !A_log || !a || !b_logits || !dO || !dq || !dk || !dv || !da || !db || !dA_log || !ddt_bias)
        return fail(GDN_ERR_NULL, "gdn_prefill_bwd: q, k, v, A_log, a, b_logits, dO and every gradient but dstate_in "
                                  "are required");
    if (B <= 0 || T <= 0 || H <= 0)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_bwd: need B, T, H > 0 (got %d, %d, %d)", B, T, H);
    if (!(dkd == 64 || dkd == 128) || !(dvd == 64 || dvd == 128))
        return fail(GDN_ERR_UNSUPPORTED, "gdn_prefill_bwd: dk, dv must be 64 or 128 (got %d, %d)", dkd, dvd);
    if ((gate_dtype != GDN_DTYPE_BF16 && gate_dtype != GDN_DTYPE_F32) ||
        (do_dtype != GDN_DTYPE_BF16 && do_dtype != GDN_DTYPE_F32))
        return fail(GDN_ERR_DTYPE, "gdn_prefill_bwd: gate_dtype and do_dtype must be GDN_DTYPE_BF16 or GDN_DTYPE_F32");
    if (static_cast<long>(B) * H * T > 0x7fffffffL)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_bwd: B*H*T exceeds the launch limit");
    const size_t need = gdn_prefill_bwd_workspace_bytes(B, T, H, dkd, dvd);
    if (!workspace || workspace_bytes < need)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_bwd: workspace of %zu B required, %zu B given", need,
                    workspace ? workspace_bytes : static_cast<size_t>(0));
    if (!aligned16(workspace)) return fail(GDN_ERR_ALIGN, "gdn_prefill_bwd: workspace must be 16-byte aligned");
    int st = check_sm100();
    if (st != GDN_OK) return st;
    if (bwd_chunked())
        return prefill_bwd_chunked(q, k, v, A_log, a, b_logits, gate_dtype, dt_bias, dt_bias_vec, mask, state_in, dO,
                                   do_dtype, dS_final, dq, dk, dv, da, db, dA_log, ddt_bias, dstate_in, B, T, H, dkd,
                                   dvd, scale == 0.f ? 1.f / sqrtf(static_cast<float>(dkd)) : scale, workspace,
                                   static_cast<cudaStream_t>(stream));
    BwdArgs ar;
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
    ar.dA_log = dA_log;
    ar.ddt_bias = ddt_bias;
    ar.dstate_in = dstate_in;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int W = bwd_window(T);
    const BwdWs wl = bwd_ws(static_cast<size_t>(B) * H, T, dkd, dvd, W);
    float* ckpt = reinterpret_cast<float*>(ws + wl.ckpt);
    float* carry = reinterpret_cast<float*>(ws + wl.carry);
    ar.states = reinterpret_cast<float*>(ws + wl.states);
    ar.rp = reinterpret_cast<float*>(ws + wl.rp);
    ar.part = reinterpret_cast<float*>(ws + wl.part);
    ar.dlogg = reinterpret_cast<float*>(ws + wl.dlogg);
    ar.B = B;
    ar.T = T;
    ar.H = H;
    ar.scale = scale == 0.f ? 1.f / sqrtf(static_cast<float>(dkd)) : scale;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dkd == 128 && dvd == 128) return launch_bwd<128, 128>(ar, W, ckpt, carry, s);
    if (dkd == 128 && dvd == 64) return launch_bwd<128, 64>(ar, W, ckpt, carry, s);
    if (dkd == 64 && dvd == 128) return launch_bwd<64, 128>(ar, W, ckpt, carry, s);
    return launch_bwd<64, 64>(ar, W, ckpt, carry, s);
}
