// prefill.cu -- chunked gated-delta-rule prefill on tcgen05 tensor cores.
//
// Math: reference/prefill_ref.py:11-132 (chunk C = 64, WY / UT form).  Replaces
// the reference's gdn_prefill_v2_kernel (kernels/prefill_chunked.cu:41-417),
// which runs fp32 CUDA-core loops and hard-codes H=16, K=128, V=256.
//
// One CTA per (batch, value head, 128-wide value tile).  Per 64-token chunk,
// with Lambda the in-chunk cumulative log decay, beta' = beta * mask and
//   N[t,s] = -beta'_t (k_t . k_s) exp(Lambda_t - Lambda_s)   (t > s)
//   A'     = (I - N)^-1 diag(beta')                          (prefill_ref.py:96-101)
// the chunk update is computed in the "R form"
//   R   = V - diag(e^Lambda) K S                 (K S on tensor cores)
//   dV  = A' R                                   (= U - W S of prefill_ref.py:103-118)
//   O   = diag(m) [ scale diag(e^Lambda) Q S + P dV ],
//         P[t,s] = scale (q_t . k_s) exp(Lambda_t - Lambda_s), s <= t    (:120-122)
//   S  <- e^{Lambda_last} S + K^T diag(e^{Lambda_last - Lambda}) dV       (:124-126)
// Every product is one tcgen05.mma.kind::f16 chain with M = 128 rows in TMEM:
// the state is kept TRANSPOSED (S^T, value index = TMEM lane) so the value
// tile is the M dimension of every product:
//   QKK = [Q;K] K^T                      M=128 (64 q rows + 64 k rows), N=64
//   SQK = S^T [Q;K]^T  (S_hi, + S_lo K)  M=128, N=128  -> (QS)^T | (KS)^T
//   DV  = R^T A'^T     (3 split terms)   M=128, N=64   -> dV^T
//   ST += dV'^T K      (2 split terms)   M=128, N=dk   (K operand MN-major)
//   PDV = dV^T P^T                       M=128, N=64
// fp32 intermediates that feed the state path (S, R, A', dV') are split into
// bf16 hi + lo pairs, so those products carry ~16 mantissa bits; q/k/v are
// exact bf16 inputs.  The output path (Q S_hi, P dV) uses single bf16.
// The 64x64 unit-lower-triangular inverse runs on CUDA cores in fp32
// (16x16 diagonal blocks by forward substitution in registers, then the
// off-diagonal blocks), the decay ratios are exp(Lambda_t - Lambda_s), never
// gamma_t / gamma_s.  q/k/v chunks arrive by TMA (128B swizzle), double
// buffered; the fp32 state lives in TMEM for the whole sequence.
#include <mutex>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {
namespace {

constexpr int kC = 64;          // chunk length
constexpr int kThreads = 128;   // 4 warps; warp w owns TMEM lanes 32w..32w+31
constexpr int kTmemCols = 512;

// TMEM column map (fp32 accumulators, 128 lanes)
constexpr uint32_t COL_QKK = 0;    // 64 cols: lanes 0-63 Q K^T, lanes 64-127 K K^T
constexpr uint32_t COL_SQK = 64;   // 128 cols: [0,64) (Q S)^T, [64,128) (K S)^T
constexpr uint32_t COL_DV = 192;   // 64 cols: dV^T
constexpr uint32_t COL_PDV = 256;  // 64 cols: (P dV)^T
constexpr uint32_t COL_ST = 320;   // dk cols: S^T (fp32 state)

template <int DK>
struct PrefillSmem {
    static constexpr int CB = DK / 64;                    // 64-wide column blocks of q/k
    static constexpr int QK_BYTES = CB * 16384;           // [Q;K]: per block 128 rows x 128 B
    static constexpr int V_BYTES = 2 * 8192;              // V: 2 blocks of 64 rows x 128 B
    static constexpr int SR_BYTES = (2 * CB * 16384 > 49152) ? 2 * CB * 16384 : 49152;
    // offsets (bytes from the 1024-aligned base)
    static constexpr int OFF_QK0 = 0;
    static constexpr int OFF_QK1 = OFF_QK0 + QK_BYTES;
    static constexpr int OFF_V0 = OFF_QK1 + QK_BYTES;
    static constexpr int OFF_V1 = OFF_V0 + V_BYTES;
    static constexpr int OFF_SR = OFF_V1 + V_BYTES;       // S_hi | S_lo, later R / dV' / dVb
    static constexpr int S_LO = CB * 16384;               // within SR
    static constexpr int R_HI = 0, R_LO = 16384, DVB = 32768;  // within SR
    static constexpr int OFF_P = OFF_SR + SR_BYTES;       // P [t][s] bf16, 8 KB
    static constexpr int OFF_AH = OFF_P + 8192;           // A' hi [t][s]
    static constexpr int OFF_AL = OFF_AH + 8192;          // A' lo
    static constexpr int NLD = 65;                        // fp32 row stride of N / A
    static constexpr int OFF_N = OFF_AL + 8192;           // N fp32 [64][65]
    static constexpr int OFF_A = OFF_N + 64 * NLD * 4;    // A fp32 [64][65]
    static constexpr int OFF_X = OFF_A + 64 * NLD * 4;    // X fp32 [16][48]
    static constexpr int OFF_G = OFF_X + 16 * 48 * 4;     // gates: 5 x 64 fp32 + 2 totals
    static constexpr int OFF_BAR = OFF_G + 6 * 64 * 4;    // 3 mbarriers + tmem base + flag
    static constexpr int BYTES = OFF_BAR + 64;
    static constexpr int ALLOC = BYTES + 1024;            // slack for 1024-B alignment
    static_assert(ALLOC <= 232448, "prefill shared memory exceeds 227 KB");
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
    uint16_t* out;
    unsigned int* err;
    int B, T, Hqk, Hv, dv, ntiles, layout;
    float scale;
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

// Write 64 fp32 values as one 128-byte row (64 bf16) of a 128B-swizzled
// K-major tile, split into hi and lo tiles.
__device__ __forceinline__ void store_row_split(uint8_t* hi_tile, uint8_t* lo_tile, int row,
                                                const float (&v)[64]) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            uint16_t h0, l0, h1, l1;
            split_bf16(v[8 * ch + 2 * p], h0, l0);
            split_bf16(v[8 * ch + 2 * p + 1], h1, l1);
            h[p] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
            l[p] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
        }
        const uint32_t off = sw128_chunk(row, ch);
        *reinterpret_cast<uint4*>(hi_tile + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(lo_tile + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}
__device__ __forceinline__ void store_row_bf16(uint8_t* tile, int row, const float (&v)[64]) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
        const uint32_t off = sw128_chunk(row, ch);
        *reinterpret_cast<uint4*>(tile + off) =
            make_uint4(pack_bf16x2(v[8 * ch], v[8 * ch + 1]), pack_bf16x2(v[8 * ch + 2], v[8 * ch + 3]),
                       pack_bf16x2(v[8 * ch + 4], v[8 * ch + 5]), pack_bf16x2(v[8 * ch + 6], v[8 * ch + 7]));
    }
}

template <int DK>
__global__ void __launch_bounds__(kThreads, 1)
prefill_chunk_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const PrefillArgs args) {
    using L = PrefillSmem<DK>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    float* g_lam = reinterpret_cast<float*>(sm + L::OFF_G);   // Lambda_t
    float* g_elam = g_lam + 64;                               // exp(Lambda_t)
    float* g_edec = g_lam + 128;                              // exp(Lambda_last - Lambda_t)
    float* g_bm = g_lam + 192;                                // beta_t * mask_t
    float* g_mk = g_lam + 256;                                // mask_t (0 for padding)
    float* g_tot = g_lam + 320;                               // per-warp scan totals
    uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);   // [2]
    uint64_t* bar_mma = bar_tma + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_tma + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* Nsm = reinterpret_cast<float*>(sm + L::OFF_N);
    float* Asm = reinterpret_cast<float*>(sm + L::OFF_A);
    float* Xsm = reinterpret_cast<float*>(sm + L::OFF_X);

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
    const int nvb = (dv_valid + 63) / 64;          // 64-wide V column blocks in this tile
    const uint32_t tma_bytes = static_cast<uint32_t>((2 * L::CB + nvb) * 8192);

    if (tid == 0) {
        mbar_init(&bar_tma[0], 1);
        mbar_init(&bar_tma[1], 1);
        mbar_init(bar_mma, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    auto taddr = [&](uint32_t col) { return tmem + lane_base + col; };

    // ---- initial state -> TMEM (S^T: lane j = value column, column d = key index)
    const long s_base = static_cast<long>(bh) * DK * args.dv + v0;
    {
        const int j = tid;
#pragma unroll
        for (int blk = 0; blk < DK / 32; ++blk) {
            float vals[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int d = blk * 32 + i;
                vals[i] = (args.state_in && j < dv_valid) ? args.state_in[s_base + static_cast<long>(d) * args.dv + j] : 0.f;
            }
            tmem_st32(taddr(COL_ST + 32 * blk), vals);
        }
        tmem_st_wait();
    }

    auto issue_tma = [&](int c, int buf) {
        uint8_t* qk = sm + (buf ? L::OFF_QK1 : L::OFF_QK0);
        uint8_t* vv = sm + (buf ? L::OFF_V1 : L::OFF_V0);
        mbar_arrive_expect_tx(&bar_tma[buf], tma_bytes);
#pragma unroll
        for (int cb = 0; cb < L::CB; ++cb) {
            tma_load_4d(qk + cb * 16384, &map_q, &bar_tma[buf], cb * 64, c * kC, hq, bidx);
            tma_load_4d(qk + cb * 16384 + 8192, &map_k, &bar_tma[buf], cb * 64, c * kC, hq, bidx);
        }
        for (int vb = 0; vb < nvb; ++vb)
            tma_load_4d(vv + vb * 8192, &map_v, &bar_tma[buf], v0 + vb * 64, c * kC, h, bidx);
    };
    if (tid == 0) issue_tma(0, 0);

    uint32_t tma_phase[2] = {0u, 0u};
    uint32_t mma_phase = 0u;
    const float A_neg = -expf(args.A_log[h]);
    const float dtb = args.dt_bias_vec ? args.dt_bias_vec[h] : args.dt_bias;
    const float scale = args.scale;
    const long gate_base = static_cast<long>(bh) * T;

    auto wait_mma = [&]() {
        if (!mbar_wait(bar_mma, mma_phase, args.err)) *abort_flag = 1;
        mma_phase ^= 1u;
        tc_fence_after();
    };

    for (int c = 0; c < nchunks; ++c) {
        const int buf = c & 1;
        uint8_t* qk_s = sm + (buf ? L::OFF_QK1 : L::OFF_QK0);
        uint8_t* v_s = sm + (buf ? L::OFF_V1 : L::OFF_V0);
        uint8_t* sr = sm + L::OFF_SR;
        if (tid == 0 && c + 1 < nchunks) issue_tma(c + 1, buf ^ 1);

        // ---- (1) gates: log decay, beta * mask, in-chunk cumulative sum (prefill_ref.py:49-64,79-91)
        float lg = 0.f;
        if (tid < kC) {
            const int tok = c * kC + tid;
            float bm = 0.f, mk = 0.f;
            if (tok < T) {
                const float av = load_gate(args.a, gate_base + tok, args.gate_dtype);
                const float bv = load_gate(args.b, gate_base + tok, args.gate_dtype);
                mk = args.mask ? args.mask[static_cast<long>(bidx) * T + tok] : 1.f;
                lg = A_neg * softplus_f(av + dtb);
                bm = sigmoid_f(bv) * mk;
            }
            g_bm[tid] = bm;
            g_mk[tid] = mk;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, lg, o);
                if (lane >= o) lg += y;
            }
            if (lane == 31) g_tot[warp] = lg;
        }
        __syncthreads();
        const float lam_last = g_tot[0] + g_tot[1];
        if (tid < kC) {
            const float lam = lg + (warp == 1 ? g_tot[0] : 0.f);
            g_lam[tid] = lam;
            g_elam[tid] = expf(lam);
            g_edec[tid] = expf(lam_last - lam);
        }
        const float gamma_c = expf(lam_last);

        // ---- (2) state S^T -> smem (bf16 hi/lo, K-major rows) and S^T *= gamma_c in TMEM
        {
            const int j = tid;
#pragma unroll
            for (int blk = 0; blk < DK / 32; ++blk) {
                float vals[32];
                tmem_ld32(taddr(COL_ST + 32 * blk), vals);
                tmem_ld_wait();
                const int cb = blk >> 1;
#pragma unroll
                for (int ch4 = 0; ch4 < 4; ++ch4) {
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        uint16_t h0, l0, h1, l1;
                        split_bf16(vals[8 * ch4 + 2 * p], h0, l0);
                        split_bf16(vals[8 * ch4 + 2 * p + 1], h1, l1);
                        hw[p] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
                        lw[p] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
                    }
                    const uint32_t off = cb * 16384 + sw128_chunk(j, (blk & 1) * 4 + ch4);
                    *reinterpret_cast<uint4*>(sr + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(sr + L::S_LO + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) vals[i] *= gamma_c;
                tmem_st32(taddr(COL_ST + 32 * blk), vals);
            }
            tmem_st_wait();
        }
        if (!mbar_wait(&bar_tma[buf], tma_phase[buf], args.err)) *abort_flag = 1;
        tma_phase[buf] ^= 1u;
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (*abort_flag) break;

        // ---- (3) MMA: QKK = [Q;K] K^T ; SQK = S_hi^T [Q;K]^T ; SQK[:,64:] += S_lo^T K^T
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sqk = smem_u32(qk_s);
            const uint32_t ssr = smem_u32(sr);
            constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
            constexpr uint32_t id128 = idesc_bf16(128, 128, false, false);
#pragma unroll
            for (int kk = 0; kk < DK / 16; ++kk) {
                const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tmem + COL_QKK, sdesc_sw128(sqk + o, 16, 1024), sdesc_sw128(sqk + o + 8192, 16, 1024),
                             id64, kk > 0);
            }
#pragma unroll
            for (int kk = 0; kk < DK / 16; ++kk) {
                const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tmem + COL_SQK, sdesc_sw128(ssr + o, 16, 1024), sdesc_sw128(sqk + o, 16, 1024),
                             id128, kk > 0);
            }
#pragma unroll
            for (int kk = 0; kk < DK / 16; ++kk) {
                const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tmem + COL_SQK + 64, sdesc_sw128(ssr + L::S_LO + o, 16, 1024),
                             sdesc_sw128(sqk + o + 8192, 16, 1024), id64, 1u);
            }
            umma_commit(bar_mma);
        }
        wait_mma();

        // ---- (4) epilogue: P (warps 0-1), N (warps 2-3), R = V - e^Lambda (K S) (all)
        {
            float row[64];
            tmem_ld64(taddr(COL_QKK), row);
            if (tid < kC) {
                const int t = tid;
                const float lt = g_lam[t];
#pragma unroll
                for (int s = 0; s < 64; ++s) row[s] = (s <= t) ? scale * row[s] * expf(lt - g_lam[s]) : 0.f;
                store_row_bf16(sm + L::OFF_P, t, row);
            } else {
                const int t = tid - kC;
                const float lt = g_lam[t];
                const float bt = -g_bm[t];
#pragma unroll
                for (int s = 0; s < 64; ++s) Nsm[t * L::NLD + s] = (s < t) ? bt * row[s] * expf(lt - g_lam[s]) : 0.f;
            }
            tmem_ld64(taddr(COL_SQK + 64), row);   // (K S)^T[j][t]
            const int j = tid;
            if (j < dv_valid) {
                const uint8_t* vb = v_s + (j >> 6) * 8192;
                const uint32_t jj = j & 63;
#pragma unroll
                for (int t = 0; t < 64; ++t) {
                    const float vt = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(vb + sw128_off(t, jj)));
                    row[t] = vt - g_elam[t] * row[t];
                }
            } else {
#pragma unroll
                for (int t = 0; t < 64; ++t) row[t] = 0.f;
            }
            store_row_split(sr + L::R_HI, sr + L::R_LO, j, row);
        }
        __syncthreads();
        if (*abort_flag) break;

        // ---- (5) A = (I - N)^-1: 16x16 diagonal blocks by forward substitution (warp w -> block w)
        {
            const int r = lane >> 1, hf = lane & 1;
            const int row0 = 16 * warp;
            float n[16], x[8];
#pragma unroll
            for (int s = 0; s < 16; ++s) n[s] = Nsm[(row0 + r) * L::NLD + row0 + s];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) x[cc] = (8 * hf + cc == r) ? 1.f : 0.f;
#pragma unroll
            for (int i = 0; i < 15; ++i) {
                float bi[8];
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) bi[cc] = __shfl_sync(0xffffffffu, x[cc], 2 * i + hf);
                if (r > i) {
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) x[cc] += n[i] * bi[cc];
                }
            }
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) Asm[(row0 + r) * L::NLD + row0 + 8 * hf + cc] = x[cc];
        }
        __syncthreads();
        // off-diagonal blocks, row block by row block: A_ij = D_i sum_{k=j}^{i-1} N_ik A_kj
        for (int ib = 1; ib < 4; ++ib) {
            const int ncol = 16 * ib;
            for (int e = tid; e < 16 * ncol; e += kThreads) {
                const int rr = e / ncol, cc = e % ncol;
                const float* nrow = Nsm + (16 * ib + rr) * L::NLD;
                float acc = 0.f;
                for (int s = cc; s < ncol; ++s) acc += nrow[s] * Asm[s * L::NLD + cc];
                Xsm[rr * 48 + cc] = acc;
            }
            __syncthreads();
            for (int e = tid; e < 16 * ncol; e += kThreads) {
                const int rr = e / ncol, cc = e % ncol;
                const float* drow = Asm + (16 * ib + rr) * L::NLD + 16 * ib;
                float acc = 0.f;
                for (int u = 0; u <= rr; ++u) acc += drow[u] * Xsm[u * 48 + cc];
                Asm[(16 * ib + rr) * L::NLD + cc] = acc;
            }
            __syncthreads();
        }
        // A' = A diag(beta') -> split bf16 rows [t][s] (B operand of dV^T = R^T A'^T)
        {
            const int t = tid >> 1, hf = tid & 1;
            const float* arow = Asm + t * L::NLD;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const int s0 = 32 * hf + 8 * ch + 2 * p;
                    const float a0 = (s0 <= t) ? arow[s0] * g_bm[s0] : 0.f;
                    const float a1 = (s0 + 1 <= t) ? arow[s0 + 1] * g_bm[s0 + 1] : 0.f;
                    uint16_t h0, l0, h1, l1;
                    split_bf16(a0, h0, l0);
                    split_bf16(a1, h1, l1);
                    hw[p] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
                    lw[p] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
                }
                const uint32_t off = sw128_chunk(t, 4 * hf + ch);
                *reinterpret_cast<uint4*>(sm + L::OFF_AH + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(sm + L::OFF_AL + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();

        // ---- (6) MMA: DV = R_hi A'_hi + R_lo A'_hi + R_hi A'_lo   (dV^T, M=128 N=64 K=64)
        if (tid == 0) {
            tc_fence_after();
            const uint32_t ssr = smem_u32(sr);
            const uint32_t sah = smem_u32(sm + L::OFF_AH), sal = smem_u32(sm + L::OFF_AL);
            constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                const uint32_t ra = ssr + (p == 1 ? L::R_LO : L::R_HI);
                const uint32_t rb = (p == 2) ? sal : sah;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + COL_DV, sdesc_sw128(ra + kk * 32, 16, 1024), sdesc_sw128(rb + kk * 32, 16, 1024),
                                 id64, (p > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(bar_mma);
        }
        wait_mma();

        // ---- (7) dV' = dV * exp(Lambda_last - Lambda) (split) and dV (bf16) -> smem rows [j][t]
        {
            float row[64];
            tmem_ld64(taddr(COL_DV), row);
            store_row_bf16(sr + L::DVB, tid, row);
#pragma unroll
            for (int t = 0; t < 64; ++t) row[t] *= g_edec[t];
            store_row_split(sr + L::R_HI, sr + L::R_LO, tid, row);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (*abort_flag) break;

        // ---- (8) MMA: ST += dV'_hi K + dV'_lo K (K as MN-major B) ; PDV = dV^T P^T
        if (tid == 0) {
            tc_fence_after();
            const uint32_t ssr = smem_u32(sr);
            const uint32_t sk = smem_u32(qk_s) + 8192;
            constexpr uint32_t idst = idesc_bf16(128, DK, false, true);
            constexpr uint32_t id64 = idesc_bf16(128, 64, false, false);
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const uint32_t ra = ssr + (p ? L::R_LO : L::R_HI);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + COL_ST, sdesc_sw128(ra + kk * 32, 16, 1024),
                                 sdesc_sw128(sk + kk * 2048, 16384, 1024), idst, 1u);
            }
            const uint32_t sp = smem_u32(sm + L::OFF_P);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_bf16_ss(tmem + COL_PDV, sdesc_sw128(ssr + L::DVB + kk * 32, 16, 1024),
                             sdesc_sw128(sp + kk * 32, 16, 1024), id64, kk > 0);
            umma_commit(bar_mma);
        }
        wait_mma();

        // ---- (9) output o[t, j] = mask_t (scale e^Lambda_t (Q S)[t,j] + (P dV)[t,j])
        {
            float qs[64], pd[64];
            tmem_ld64(taddr(COL_SQK), qs);
            tmem_ld64(taddr(COL_PDV), pd);
            const int j = tid;
            if (j < dv_valid) {
                const int tmax = min(kC, T - c * kC);
                const long tok0 = static_cast<long>(c) * kC;
                const long ostep = (args.layout == GDN_LAYOUT_BHTD) ? args.dv : static_cast<long>(args.Hv) * args.dv;
                uint16_t* obase = args.out + ((args.layout == GDN_LAYOUT_BHTD)
                                                  ? (static_cast<long>(bh) * T + tok0) * args.dv
                                                  : ((static_cast<long>(bidx) * T + tok0) * args.Hv + h) * args.dv) +
                                  v0 + j;
#pragma unroll
                for (int t = 0; t < kC; ++t) {
                    if (t < tmax) obase[t * ostep] = f32_to_bf16_bits(g_mk[t] * (scale * g_elam[t] * qs[t] + pd[t]));
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        if (*abort_flag) break;
    }

    // ---- final state S^T (TMEM) -> state_out [dk][dv]
    if (!*abort_flag && args.state_out) {
        const int j = tid;
#pragma unroll
        for (int blk = 0; blk < DK / 32; ++blk) {
            float vals[32];
            tmem_ld32(taddr(COL_ST + 32 * blk), vals);
            tmem_ld_wait();
            if (j < dv_valid) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    args.state_out[s_base + static_cast<long>(blk * 32 + i) * args.dv + j] = vals[i];
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
int launch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const PrefillArgs& args,
                   int grid, cudaStream_t st) {
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
    prefill_chunk_kernel<DK><<<grid, kThreads, L::ALLOC, st>>>(mq, mk, mv, args);
    return launch_status("gdn_prefill_fwd");
}

// q/k/v map: dims (D, T, H, B) innermost first, box (64, 64, 1, 1), 128B swizzle.
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

    CUtensorMap mq, mk, mv;
    if ((st = make_act_map(&mq, q, dk, T, Hqk, B, layout)) != GDN_OK) return st;
    if ((st = make_act_map(&mk, k, dk, T, Hqk, B, layout)) != GDN_OK) return st;
    if ((st = make_act_map(&mv, v, dv, T, Hv, B, layout)) != GDN_OK) return st;

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
    args.out = static_cast<uint16_t*>(out);
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
    if (dk == 128) return launch_prefill<128>(mq, mk, mv, args, grid, s);
    return launch_prefill<64>(mq, mk, mv, args, grid, s);
}
