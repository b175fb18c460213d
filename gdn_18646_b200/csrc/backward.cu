// backward.cu -- gradients of the gated delta rule prefill (dq, dk, dv, da, db,
// dA_log, ddt_bias and the initial state), for training use.
//
// The reference has no backward.  This is the token-recurrent derivative (the
// same recurrence as the forward, per token: S' = g S_p, r = S'^T k,
// d = b'(v - r), S_n = S' + k d^T, o = m scale q^T S_n), computed by three
// kernels over a workspace that holds every token's state:
//
//   bwd_states_kernel  the forward recurrence again, storing the state S_p
//                      before every token (fp32 [B,H,T,dk,dv]);
//   bwd_dstate_kernel  the reverse recurrence of dS (the gradient of S_n):
//                      dS += scale q (m dO)^T, dd = dS^T k, dS <- g (dS - b' k dd^T),
//                      storing dS for every token, dv = b' dd and dd itself;
//   bwd_token_kernel   every token independently, from S_p and dS: dq, dk, the
//                      gate gradients (dg = <S_p, dS + k dr^T>, db') and their
//                      chain rule through g = exp(-exp(A_log) softplus(a + dt_bias))
//                      and b' = sigmoid(b) m;
//   bwd_head_kernel    dA_log and ddt_bias, summed per head in token order.
//
// The two recurrences keep (half) a value column of the state per thread (64
// registers), so their reductions stay inside a warp; a warp writes state rows
// as 64- or 128-byte segments.  All arithmetic is
// fp32 on CUDA cores; the kernels are bound by the workspace traffic
// (2 x 4 dk dv bytes per token and head, written once and read once).
// Restates oracle prefill_backward (pinned to finite differences).
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
    float* states;             // workspace: S_p per token [B,H,T,DK,DV]
    float* dstates;            // workspace: dS per token
    float* dd;                 // workspace: [B,H,T,DV]
    float* rp;                 // workspace: [B,H,T,DV], k . S_p per value column
    float* dlogg;              // workspace: [B,H,T]
    int B, T, H;
    float scale;
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
    const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
    for (int i = 0; i < L::ROWS; ++i)
        S[i] = a.state_in ? a.state_in[s0 + static_cast<long>(i0 + i) * DV + j] : 0.f;
    for (int tb = 0; tb < a.T; tb += kTB) {
        const int nt = min(kTB, a.T - tb);
        const long tok0 = static_cast<long>(bh) * a.T + tb;
        __syncthreads();
        for (int e = tid; e < nt * DK; e += L::THREADS) ks[e / DK][e % DK] = bf16_at(a.k, tok0 * DK + e);
        for (int e = tid; e < nt * L::CTA_COLS; e += L::THREADS)
            vs[e / L::CTA_COLS][e % L::CTA_COLS] =
                bf16_at(a.v, (tok0 + e / L::CTA_COLS) * DV + blockIdx.y * L::CTA_COLS + e % L::CTA_COLS);
        if (tid < nt) gate_of(a, bh, tb + tid, gs[tid], bs[tid]);
        __syncthreads();
        for (int u = 0; u < nt; ++u) {
            const long tok = tok0 + u;
            float* out = a.states + (tok * DK + i0) * DV + j;
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) out[static_cast<long>(i) * DV] = S[i];
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
            if (i0 == 0) a.rp[tok * DV + j] = rp;
            const float d = bm * (vs[u][jc] - g * rp);
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) S[i] = fmaf(kk[i], d, g * S[i]);
        }
    }
}

// Reverse recurrence of dS, storing dS (gradient of S_n) per token, dv and dd.  Grid (B*H, DV/CTA_COLS).
template <int DK, int DV>
__global__ void __launch_bounds__(128) bwd_dstate_kernel(const BwdArgs a) {
    using L = RecLayout<DK>;
    const int bh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int jl = lane % L::COLS;
    const int jc = warp * L::COLS + jl;
    const int j = blockIdx.y * L::CTA_COLS + jc;
    const int i0 = (lane / L::COLS) * L::ROWS;
    const int bi = bh / a.H;
    __shared__ float ks[kTB][DK], qs[kTB][DK];
    __shared__ float dos[kTB][L::CTA_COLS];
    __shared__ float gs[kTB], bs[kTB];
    float dS[L::ROWS];
    const long s0 = static_cast<long>(bh) * DK * DV;
#pragma unroll
    for (int i = 0; i < L::ROWS; ++i)
        dS[i] = a.dS_final ? a.dS_final[s0 + static_cast<long>(i0 + i) * DV + j] : 0.f;
    for (int tend = a.T; tend > 0; tend -= kTB) {
        const int tb = max(0, tend - kTB), nt = tend - tb;
        const long tok0 = static_cast<long>(bh) * a.T + tb;
        __syncthreads();
        for (int e = tid; e < nt * DK; e += L::THREADS) {
            ks[e / DK][e % DK] = bf16_at(a.k, tok0 * DK + e);
            qs[e / DK][e % DK] = bf16_at(a.q, tok0 * DK + e);
        }
        for (int e = tid; e < nt * L::CTA_COLS; e += L::THREADS) {
            const int u = e / L::CTA_COLS;
            const long idx = (tok0 + u) * DV + blockIdx.y * L::CTA_COLS + e % L::CTA_COLS;
            const float m = a.mask ? a.mask[static_cast<long>(bi) * a.T + tb + u] : 1.f;
            dos[u][e % L::CTA_COLS] =
                a.scale * m * (a.do_dtype == GDN_DTYPE_BF16 ? bf16_at(static_cast<const uint16_t*>(a.dO), idx)
                                                             : static_cast<const float*>(a.dO)[idx]);
        }
        if (tid < nt) gate_of(a, bh, tb + tid, gs[tid], bs[tid]);
        __syncthreads();
        for (int u = nt - 1; u >= 0; --u) {
            const long tok = tok0 + u;
            const float* kk = ks[u] + i0;
            const float* qq = qs[u] + i0;
            const float sdo = dos[u][jc];
            const float g = gs[u], bm = bs[u];
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
            float* out = a.dstates + (tok * DK + i0) * DV + j;
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) out[static_cast<long>(i) * DV] = dS[i];
            const float ddj = sum_parts<L::PARTS, L::COLS>((e0 + e1) + (e2 + e3));
            if (i0 == 0) {
                a.dd[tok * DV + j] = ddj;
                a.dv[tok * DV + j] = bm * ddj;
            }
            const float dr = -bm * ddj;
#pragma unroll
            for (int i = 0; i < L::ROWS; ++i) dS[i] = g * fmaf(kk[i], dr, dS[i]);
        }
    }
    if (a.dstate_in) {
#pragma unroll
        for (int i = 0; i < L::ROWS; ++i) a.dstate_in[s0 + static_cast<long>(i0 + i) * DV + j] = dS[i];
    }
}

// Per token: dq, dk, da, db (and dlog g for the head sums), one pass over S_p and dS.
// One CTA of 4 warps per token; every warp holds all DV columns (DV/32 per lane), so
// the per-column vectors (r = g k.S_p from the forward pass, delta, dr, m dO) and
// their sums are formed in registers, and each warp reduces its rows' products
// (dq_i, dk_i) across its lanes while S_p and dS are read once, row by row.
template <int DK, int DV>
__global__ void __launch_bounds__(128) bwd_token_kernel(const BwdArgs a) {
    constexpr int NW = 4, CPL = DV / 32;             // warps, columns per lane
    const long tok = blockIdx.x;                  // bh * T + t
    const int bh = static_cast<int>(tok / a.T), t = static_cast<int>(tok - static_cast<long>(bh) * a.T);
    const int bi = bh / a.H, h = bh % a.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float red[NW];
    float g, bm;
    gate_of(a, bh, t, g, bm);
    const float m = a.mask ? a.mask[static_cast<long>(bi) * a.T + t] : 1.f;
    // ---- per-column vectors of this lane's columns j = lane * CPL + c
    float dlt[CPL], drs[CPL], dos[CPL];
    float p_db = 0.f, p_ddo = 0.f, p_rdr = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int j = lane * CPL + c;
        const float vj = bf16_at(a.v, tok * DV + j);
        const float rp = a.rp[tok * DV + j];
        const float ddj = a.dd[tok * DV + j];
        const float r = g * rp;
        dlt[c] = bm * (vj - r);
        drs[c] = -bm * ddj;
        dos[c] = m * (a.do_dtype == GDN_DTYPE_BF16 ? bf16_at(static_cast<const uint16_t*>(a.dO), tok * DV + j)
                                                   : static_cast<const float*>(a.dO)[tok * DV + j]);
        p_db = fmaf(ddj, vj - r, p_db);
        p_ddo = fmaf(dlt[c], dos[c], p_ddo);
        p_rdr = fmaf(drs[c], rp, p_rdr);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        p_db += __shfl_xor_sync(0xffffffffu, p_db, o);
        p_ddo += __shfl_xor_sync(0xffffffffu, p_ddo, o);
        p_rdr += __shfl_xor_sync(0xffffffffu, p_rdr, o);
    }
    // ---- rows i = warp, warp + NW, ...: dq_i = scale (g S_p[i,:].dO' + k_i (delta.dO')),
    //      dk_i = dS[i,:].delta + g S_p[i,:].dr; <S_p, dS> accumulated for dg
    const float* Sp = a.states + tok * DK * DV;
    const float* dS = a.dstates + tok * DK * DV;
    float p_sds = 0.f;
    for (int i = warp; i < DK; i += NW) {
        float s[CPL], ds[CPL];
        if constexpr (CPL == 4) {
            const float4 x = *reinterpret_cast<const float4*>(Sp + i * DV + lane * 4);
            const float4 y = *reinterpret_cast<const float4*>(dS + i * DV + lane * 4);
            s[0] = x.x; s[1] = x.y; s[2] = x.z; s[3] = x.w;
            ds[0] = y.x; ds[1] = y.y; ds[2] = y.z; ds[3] = y.w;
        } else {
            const float2 x = *reinterpret_cast<const float2*>(Sp + i * DV + lane * 2);
            const float2 y = *reinterpret_cast<const float2*>(dS + i * DV + lane * 2);
            s[0] = x.x; s[1] = x.y;
            ds[0] = y.x; ds[1] = y.y;
        }
        float sdo = 0.f, sdr = 0.f, dsd = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            sdo = fmaf(s[c], dos[c], sdo);
            sdr = fmaf(s[c], drs[c], sdr);
            dsd = fmaf(ds[c], dlt[c], dsd);
            p_sds = fmaf(s[c], ds[c], p_sds);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sdo += __shfl_xor_sync(0xffffffffu, sdo, o);
            sdr += __shfl_xor_sync(0xffffffffu, sdr, o);
            dsd += __shfl_xor_sync(0xffffffffu, dsd, o);
        }
        if (lane == 0) {
            const float ki = bf16_at(a.k, tok * DK + i);
            a.dq[tok * DK + i] = a.scale * fmaf(g, sdo, ki * p_ddo);
            a.dk[tok * DK + i] = fmaf(g, sdr, dsd);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p_sds += __shfl_xor_sync(0xffffffffu, p_sds, o);
    if (lane == 0) red[warp] = p_sds;
    __syncthreads();
    if (tid == 0) {
        float dg = p_rdr;                             // <S_p, dS + k dr^T> = <S_p, dS> + dr . rp
#pragma unroll
        for (int w = 0; w < NW; ++w) dg += red[w];
        const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
        const float x = load_gate(a.a, tok, a.gate_dtype) + dtb;
        const float dlogg = dg * g;
        a.dlogg[tok] = dlogg;
        a.da[tok] = dlogg * (-expf(a.A_log[h])) * (x > 20.f ? 1.f : sigmoid_f(x));
        const float sb = sigmoid_f(load_gate(a.b, tok, a.gate_dtype));
        a.db[tok] = p_db * m * sb * (1.f - sb);
    }
}

// dA_log[h] = sum dlogg * log g, ddt_bias[h] = sum da over (b, t), in order.  One CTA per head.
__global__ void __launch_bounds__(256) bwd_head_kernel(const BwdArgs a) {
    const int h = blockIdx.x, tid = threadIdx.x;
    __shared__ float r0[256], r1[256];
    const float dtb = a.dt_bias_vec ? a.dt_bias_vec[h] : a.dt_bias;
    const float Aneg = -expf(a.A_log[h]);
    float s0 = 0.f, s1 = 0.f;
    for (int bi = 0; bi < a.B; ++bi) {
        const long base = (static_cast<long>(bi) * a.H + h) * a.T;
        for (int t = tid; t < a.T; t += 256) {
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
    if (tid == 0) {
        a.dA_log[h] = r0[0];
        a.ddt_bias[h] = r1[0];
    }
}

template <int DK, int DV>
int launch_bwd(const BwdArgs& a, cudaStream_t st) {
    const dim3 rec(a.B * a.H, DV / RecLayout<DK>::CTA_COLS);
    bwd_states_kernel<DK, DV><<<rec, RecLayout<DK>::THREADS, 0, st>>>(a);
    int s = launch_status("gdn_prefill_bwd (states)");
    if (s != GDN_OK) return s;
    bwd_dstate_kernel<DK, DV><<<rec, RecLayout<DK>::THREADS, 0, st>>>(a);
    if ((s = launch_status("gdn_prefill_bwd (dstate)")) != GDN_OK) return s;
    bwd_token_kernel<DK, DV><<<static_cast<unsigned>(static_cast<long>(a.B) * a.H * a.T), 128, 0, st>>>(a);
    if ((s = launch_status("gdn_prefill_bwd (tokens)")) != GDN_OK) return s;
    bwd_head_kernel<<<a.H, 256, 0, st>>>(a);
    return launch_status("gdn_prefill_bwd (heads)");
}

}  // namespace
}  // namespace gdn

extern "C" size_t gdn_prefill_bwd_workspace_bytes(int B, int T, int H, int dk, int dv) {
    if (B <= 0 || T <= 0 || H <= 0 || !(dk == 64 || dk == 128) || !(dv == 64 || dv == 128)) return 0;
    const size_t tok = static_cast<size_t>(B) * H * T;
    return 2 * tok * dk * dv * 4 + 2 * tok * dv * 4 + tok * 4 + 1024;
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
    const size_t tok = static_cast<size_t>(B) * H * T;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    ar.states = reinterpret_cast<float*>(ws);
    ar.dstates = reinterpret_cast<float*>(ws + tok * dkd * dvd * 4);
    ar.dd = reinterpret_cast<float*>(ws + 2 * tok * dkd * dvd * 4);
    ar.rp = reinterpret_cast<float*>(ws + 2 * tok * dkd * dvd * 4 + tok * dvd * 4);
    ar.dlogg = reinterpret_cast<float*>(ws + 2 * tok * dkd * dvd * 4 + 2 * tok * dvd * 4);
    ar.B = B;
    ar.T = T;
    ar.H = H;
    ar.scale = scale == 0.f ? 1.f / sqrtf(static_cast<float>(dkd)) : scale;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dkd == 128 && dvd == 128) return launch_bwd<128, 128>(ar, s);
    if (dkd == 128 && dvd == 64) return launch_bwd<128, 64>(ar, s);
    if (dkd == 64 && dvd == 128) return launch_bwd<64, 128>(ar, s);
    return launch_bwd<64, 64>(ar, s);
}
