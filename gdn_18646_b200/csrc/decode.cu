// decode.cu -- single-token gated delta rule step (the recurrence of
// reference/decode_ref.py:11-61; replaces kernels/decode.cu of the reference).
//
// One CTA per (batch, value head).  The fp32 state S[dk][dv] of the head is
// streamed exactly once in and once out with 16-byte accesses:
//   thread (cg, rg) owns 4 consecutive value columns 4cg..4cg+3 and the rows
//   i = r*RG + rg, r < RPT, held in registers as float4.
// Both reductions over the key dimension (k.S and q.S) are taken from the
// OLD state in a single pass, using
//   o_j = scale * (g * (q.S)_j + delta_j * (q.k)),   delta_j = beta*(v_j - g*(k.S)_j),
// so the update S' = g*S + k delta^T is written straight from registers.
// Every element is read before any is written by the same thread, so
// state_out may alias state_in (in-place update).
//
// With a gate (y != null) the CTA also applies the layer's gated output norm to
// its head's o row, which is exactly one norm group: y = (o * rsqrt(mean(o^2) +
// eps)) * gamma * silu(z), bf16 (the gated RMSNorm of rmsnorm.cu on the same
// row), so the output projection reads y without a norm launch in between.
#include "common.cuh"

namespace gdn {
namespace {

// SPLIT CTAs (a cluster) share a head, each owning DV/SPLIT value columns: for
// small batches, where one CTA per head leaves most SMs idle, the head's state
// streams through twice the SMs.  Every reduction over the key dimension stays
// inside a CTA; only the gated norm's sum of squares crosses the pair (DSMEM).
template <int DK, int DV, int SPLIT = 1>
struct DecodeCfg {
    static constexpr int DVC = DV / SPLIT;                              // value columns per CTA
    static constexpr int CG = DVC / 4;                                  // column groups (float4 each)
    static constexpr int RPT = DK * DVC >= 65536 ? 16 : (DK / 4 < 32 ? DK / 4 : 32);  // rows per thread
    static constexpr int RG = DK / RPT;                                 // row groups
    static constexpr int NT = CG * RG;                                  // threads per CTA
    static_assert(RPT <= 32 && NT <= 1024, "state slice too large for registers");
};

template <int DK, int DV, int SPLIT>
__global__ void __launch_bounds__(DecodeCfg<DK, DV, SPLIT>::NT)
decode_step_kernel(const uint16_t* q, const uint16_t* k, const uint16_t* v, const void* a, const void* b,
                   int gate_dtype, const float* __restrict__ A_log,
                   const float* __restrict__ dt_bias, const float* state_in, float* state_out,
                   float* __restrict__ out, int Hqk, int Hv, float scale, int l2qk, const uint16_t* z,
                   const uint16_t* __restrict__ gamma, float eps, uint16_t* __restrict__ y) {
    using C = DecodeCfg<DK, DV, SPLIT>;
    constexpr int kNormWarps = (C::CG + 31) / 32;      // warps holding the row's rg == 0 threads
    __shared__ float q_s[DK];
    __shared__ float k_s[DK];
    __shared__ float red_a[C::RG][C::DVC];
    __shared__ float red_b[C::RG][C::DVC];
    __shared__ float qk_s;
    __shared__ float inv_s[2];
    __shared__ float nrm_s[kNormWarps];
    __shared__ float nrm_peer;                 // SPLIT == 2: the other CTA's sum of squares

    pdl_launch_dependents();                   // the next kernel may launch (it waits for this one)
    pdl_wait_prior();                          // inputs and state come from earlier kernels
    const int tid = threadIdx.x;
    const int rank = SPLIT > 1 ? static_cast<int>(blockIdx.x % SPLIT) : 0;   // cluster rank = column half
    const int cg = tid % C::CG + rank * C::CG;  // this thread's float4 column group within the head
    const int rg = tid / C::CG;
    const int bh = blockIdx.x / SPLIT;         // b * Hv + h
    const int h = bh % Hv;
    const int bidx = bh / Hv;
    const int hq = h / (Hv / Hqk);
    const long qk_off = (static_cast<long>(bidx) * Hqk + hq) * DK;
    const long s_off = static_cast<long>(bh) * DK * DV;

    // issue the state loads first: they dominate the step
    float4 s[C::RPT];
#pragma unroll
    for (int r = 0; r < C::RPT; ++r)
        s[r] = ld_stream_f4(state_in + s_off + static_cast<long>(r * C::RG + rg) * DV + 4 * cg);

    // q, k, v, a, b are outputs of the kernel just before this one, which may still
    // run until pdl_wait_prior() above: read them through L2 (ld.global.cg), never
    // through the non-coherent read-only path
    for (int i = tid; i < DK; i += C::NT) {
        q_s[i] = bf16_bits_to_f32(__ldcg(q + qk_off + i));
        k_s[i] = bf16_bits_to_f32(__ldcg(k + qk_off + i));
    }
    // gates (reference/decode_ref.py:36-38)
    const float av = gate_dtype == GDN_DTYPE_BF16 ? bf16_bits_to_f32(__ldcg(static_cast<const uint16_t*>(a) + bh))
                                                  : __ldcg(static_cast<const float*>(a) + bh);
    const float bv = gate_dtype == GDN_DTYPE_BF16 ? bf16_bits_to_f32(__ldcg(static_cast<const uint16_t*>(b) + bh))
                                                  : __ldcg(static_cast<const float*>(b) + bh);
    const float dtb = dt_bias ? dt_bias[h] : 0.f;
    const float g = expf(-expf(A_log[h]) * softplus_f(av + dtb));
    const float beta = sigmoid_f(bv);
    const uint2 vraw = __ldcg(reinterpret_cast<const uint2*>(v + static_cast<long>(bh) * DV + 4 * cg));
    // the gated norm's z and gamma, fetched with the other inputs so their latency hides
    // behind the state loads
    uint2 zw = make_uint2(0u, 0u), gw = make_uint2(0u, 0u);
    if (y && rg == 0) {
        zw = __ldcg(reinterpret_cast<const uint2*>(z + static_cast<long>(bh) * DV + 4 * cg));
        gw = *reinterpret_cast<const uint2*>(gamma + 4 * cg);
    }
    __syncthreads();
    if (l2qk) {
        // q, k L2-normalised per head (fp32, eps 1e-6) and rounded to bf16, as the
        // layer's projection epilogue does (reference/fused_proj_conv_silu_ref.py:64-66
        // composition); warp 0 takes q, warp 1 k
        if (tid < 64) {
            const float* src = tid < 32 ? q_s : k_s;
            float ss = 0.f;
            for (int i = tid & 31; i < DK; i += 32) ss = fmaf(src[i], src[i], ss);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if ((tid & 31) == 0) inv_s[tid >> 5] = 1.f / sqrtf(ss + 1e-6f);
        }
        __syncthreads();
        for (int i = tid; i < DK; i += C::NT) {
            q_s[i] = bf16_bits_to_f32(f32_to_bf16_bits(q_s[i] * inv_s[0]));
            k_s[i] = bf16_bits_to_f32(f32_to_bf16_bits(k_s[i] * inv_s[1]));
        }
        __syncthreads();
    }

    if (tid < 32) {
        float acc = 0.f;
        for (int i = tid; i < DK; i += 32) acc += q_s[i] * k_s[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (tid == 0) qk_s = acc;
    }

    float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < C::RPT; ++r) {
        const int i = r * C::RG + rg;
        const float ki = k_s[i], qi = q_s[i];
        pa[0] += ki * s[r].x; pa[1] += ki * s[r].y; pa[2] += ki * s[r].z; pa[3] += ki * s[r].w;
        pb[0] += qi * s[r].x; pb[1] += qi * s[r].y; pb[2] += qi * s[r].z; pb[3] += qi * s[r].w;
    }
    const int cl = 4 * (cg - rank * C::CG);             // column within this CTA's slice
    *reinterpret_cast<float4*>(&red_a[rg][cl]) = make_float4(pa[0], pa[1], pa[2], pa[3]);
    *reinterpret_cast<float4*>(&red_b[rg][cl]) = make_float4(pb[0], pb[1], pb[2], pb[3]);
    __syncthreads();

    float ka[4] = {0.f, 0.f, 0.f, 0.f}, qa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int x = 0; x < C::RG; ++x) {
        const float4 ra = *reinterpret_cast<const float4*>(&red_a[x][cl]);
        const float4 rb = *reinterpret_cast<const float4*>(&red_b[x][cl]);
        ka[0] += ra.x; ka[1] += ra.y; ka[2] += ra.z; ka[3] += ra.w;
        qa[0] += rb.x; qa[1] += rb.y; qa[2] += rb.z; qa[3] += rb.w;
    }
    const float vj[4] = {bf16_bits_to_f32(vraw.x & 0xffffu), bf16_bits_to_f32(vraw.x >> 16),
                         bf16_bits_to_f32(vraw.y & 0xffffu), bf16_bits_to_f32(vraw.y >> 16)};
    const float qk = qk_s;
    float delta[4], oj[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        delta[c] = beta * (vj[c] - g * ka[c]);             // decode_ref.py:49-52
        oj[c] = scale * (g * qa[c] + delta[c] * qk);       // decode_ref.py:56
    }
    if (rg == 0 && out)
        *reinterpret_cast<float4*>(out + static_cast<long>(bh) * DV + 4 * cg) =
            make_float4(oj[0], oj[1], oj[2], oj[3]);

#pragma unroll
    for (int r = 0; r < C::RPT; ++r) {
        const int i = r * C::RG + rg;
        const float ki = k_s[i];
        float4 n;
        n.x = g * s[r].x + ki * delta[0];                  // decode_ref.py:46,53
        n.y = g * s[r].y + ki * delta[1];
        n.z = g * s[r].z + ki * delta[2];
        n.w = g * s[r].w + ki * delta[3];
        st_stream_f4(state_out + s_off + static_cast<long>(i) * DV + 4 * cg, n);
    }

    if (y) {
        // gated output norm of this head's row (the rg == 0 threads hold it, 4 columns each)
        float ss = 0.f;
        if (rg == 0) {
#pragma unroll
            for (int c = 0; c < 4; ++c) ss = fmaf(oj[c], oj[c], ss);
        }
        if (tid < 32 * kNormWarps) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if ((tid & 31) == 0) nrm_s[tid >> 5] = ss;
        }
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kNormWarps; ++w) tot += nrm_s[w];
        if constexpr (SPLIT == 2) {
            // the pair's other half of the row: write this CTA's sum into the peer's
            // shared memory, then a cluster barrier (release / acquire) for both
            if (tid == 0) {
                uint32_t ra;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(&nrm_peer)), "r"(rank ^ 1));
                asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(tot) : "memory");
            }
            asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
            asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
            tot = rank == 0 ? tot + nrm_peer : nrm_peer + tot;   // the same order in both CTAs
        }
        if (rg == 0) {
            const float r = rsqrtf(tot / static_cast<float>(DV) + eps);
            const float gf[4] = {bf16_bits_to_f32(gw.x & 0xffffu), bf16_bits_to_f32(gw.x >> 16),
                                 bf16_bits_to_f32(gw.y & 0xffffu), bf16_bits_to_f32(gw.y >> 16)};
            const float zf[4] = {bf16_bits_to_f32(zw.x & 0xffffu), bf16_bits_to_f32(zw.x >> 16),
                                 bf16_bits_to_f32(zw.y & 0xffffu), bf16_bits_to_f32(zw.y >> 16)};
            float yo[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) yo[c] = (oj[c] * r) * gf[c] * silu_fast(zf[c]);
            *reinterpret_cast<uint2*>(y + static_cast<long>(bh) * DV + 4 * cg) =
                make_uint2(pack_bf16x2(yo[0], yo[1]), pack_bf16x2(yo[2], yo[3]));
        }
    }
}

template <int DK, int DV, int SPLIT>
cudaError_t launch_decode_split(const void* q, const void* k, const void* v, const void* a, const void* b,
                                int gate_dtype, const float* A_log, const float* dt_bias, const float* s_in,
                                float* s_out, float* out, int B, int Hqk, int Hv, float scale, int l2qk,
                                const void* z, const void* gamma, float eps, void* y, cudaStream_t st) {
    using C = DecodeCfg<DK, DV, SPLIT>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(B * Hv * SPLIT);
    cfg.blockDim = dim3(C::NT);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (SPLIT > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = SPLIT;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (launch_overlap()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, decode_step_kernel<DK, DV, SPLIT>, static_cast<const uint16_t*>(q),
                       static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v), a, b, gate_dtype, A_log,
                       dt_bias, s_in, s_out, out, Hqk, Hv, scale, l2qk, static_cast<const uint16_t*>(z),
                       static_cast<const uint16_t*>(gamma), eps, static_cast<uint16_t*>(y));
}

// One CTA per head, or a pair of CTAs per head: for few heads (dv >= 128) so that
// the state streams through twice the SMs, and always at dv = 256, where one CTA
// would need 1024 threads of at most 64 registers and spill.
template <int DK, int DV>
cudaError_t launch_decode(const void* q, const void* k, const void* v, const void* a, const void* b,
                          int gate_dtype, const float* A_log, const float* dt_bias, const float* s_in,
                          float* s_out, float* out, int B, int Hqk, int Hv, float scale, int l2qk, const void* z,
                          const void* gamma, float eps, void* y, cudaStream_t st) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if constexpr (DV >= 128) {
        if (DV == 256 || 2L * B * Hv <= sms)
            return launch_decode_split<DK, DV, 2>(q, k, v, a, b, gate_dtype, A_log, dt_bias, s_in, s_out, out, B, Hqk,
                                                  Hv, scale, l2qk, z, gamma, eps, y, st);
    }
    if constexpr (DV < 256)
        return launch_decode_split<DK, DV, 1>(q, k, v, a, b, gate_dtype, A_log, dt_bias, s_in, s_out, out, B, Hqk,
                                              Hv, scale, l2qk, z, gamma, eps, y, st);
    return cudaErrorInvalidValue;                      // unreachable: dv = 256 always splits
}

}  // namespace
}  // namespace gdn

namespace {
int decode_common(const char* name, const void* q, const void* k, const void* v, const void* a, const void* b,
                  int gate_dtype, const float* A_log, const float* dt_bias, const float* state_in, float* state_out,
                  float* out, const void* z, const void* gamma, float eps, void* y, int B, int Hqk, int Hv, int dk,
                  int dv, float scale, int flags, void* stream) {
    using namespace gdn;
    if (flags & ~GDN_DECODE_L2NORM_QK) return fail(GDN_ERR_DTYPE, "%s: unknown flags 0x%x", name, flags);
    const int l2qk = (flags & GDN_DECODE_L2NORM_QK) ? 1 : 0;
    if (!q || !k || !v || !a || !b || !A_log || !state_in || !state_out || (!out && !y))
        return fail(GDN_ERR_NULL, "%s: q, k, v, a, b, A_log, state_in, state_out and an output are required", name);
    if (y && (!z || !gamma)) return fail(GDN_ERR_NULL, "%s: the gated norm needs z and norm_gamma", name);
    if (B <= 0 || Hqk <= 0 || Hv <= 0 || Hv % Hqk != 0)
        return fail(GDN_ERR_SHAPE, "%s: bad B=%d Hqk=%d Hv=%d (need B,H > 0 and Hv %% Hqk == 0)", name, B, Hqk, Hv);
    if (static_cast<long>(B) * Hv > 0x7fffffffL) return fail(GDN_ERR_SHAPE, "%s: B*Hv too large", name);
    if (gate_dtype != GDN_DTYPE_BF16 && gate_dtype != GDN_DTYPE_F32)
        return fail(GDN_ERR_DTYPE, "%s: gate_dtype must be GDN_DTYPE_BF16 or GDN_DTYPE_F32", name);
    const bool ok_dims = (dk == 64 || dk == 128 || dk == 256) && (dv == 64 || dv == 128 || dv == 256);
    if (!ok_dims)
        return fail(GDN_ERR_UNSUPPORTED, "%s: dk=%d dv=%d not supported (each must be 64, 128 or 256)", name, dk, dv);
    if (!aligned16(state_in) || !aligned16(state_out) || (out && !aligned16(out)) || !aligned16(q) || !aligned16(k) ||
        (reinterpret_cast<uintptr_t>(v) & 7u))
        return fail(GDN_ERR_ALIGN, "%s: state/out/q/k must be 16-byte aligned and v 8-byte aligned", name);
    if (y && ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(gamma)) & 7u))
        return fail(GDN_ERR_ALIGN, "%s: z, norm_gamma and y must be 8-byte aligned", name);
    int st = check_sm100();
    if (st != GDN_OK) return st;
    if (scale == 0.f) scale = 1.f / sqrtf(static_cast<float>(dk));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define GDN_DEC(DKV, DVV)                                                                          \
    if (dk == DKV && dv == DVV) {                                                                  \
        const cudaError_t e = launch_decode<DKV, DVV>(q, k, v, a, b, gate_dtype, A_log, dt_bias,   \
                                                      state_in, state_out, out, B, Hqk, Hv, scale,  \
                                                      l2qk, z, gamma, eps, y, s);                   \
        if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s: launch failed: %s", name, cudaGetErrorString(e)); \
        return launch_status(name);                                                                \
    }
    GDN_DEC(64, 64)
    GDN_DEC(64, 128)
    GDN_DEC(64, 256)
    GDN_DEC(128, 64)
    GDN_DEC(128, 128)
    GDN_DEC(128, 256)
    GDN_DEC(256, 64)
    GDN_DEC(256, 128)
    GDN_DEC(256, 256)
#undef GDN_DEC
    return fail(GDN_ERR_UNSUPPORTED, "%s: unreachable dims", name);
}
}  // namespace

extern "C" int gdn_decode_step_ex(const void* q, const void* k, const void* v, const void* a,
                                  const void* b, int gate_dtype, const float* A_log,
                                  const float* dt_bias, const float* state_in, float* state_out,
                                  float* out, int B, int Hqk, int Hv, int dk, int dv, float scale,
                                  int flags, void* stream) {
    if (!out) return gdn::fail(GDN_ERR_NULL, "gdn_decode_step: out is required");
    return decode_common("gdn_decode_step", q, k, v, a, b, gate_dtype, A_log, dt_bias, state_in, state_out, out,
                         nullptr, nullptr, 0.f, nullptr, B, Hqk, Hv, dk, dv, scale, flags, stream);
}

extern "C" int gdn_decode_step_gated(const void* q, const void* k, const void* v, const void* a, const void* b,
                                     int gate_dtype, const float* A_log, const float* dt_bias,
                                     const float* state_in, float* state_out, float* out, const void* z,
                                     const void* norm_gamma, float eps, void* y, int B, int Hqk, int Hv, int dk,
                                     int dv, float scale, int flags, void* stream) {
    if (!y) return gdn::fail(GDN_ERR_NULL, "gdn_decode_step_gated: y is required");
    return decode_common("gdn_decode_step_gated", q, k, v, a, b, gate_dtype, A_log, dt_bias, state_in, state_out,
                         out, z, norm_gamma, eps, y, B, Hqk, Hv, dk, dv, scale, flags, stream);
}

extern "C" int gdn_decode_step(const void* q, const void* k, const void* v, const void* a,
                               const void* b, int gate_dtype, const float* A_log,
                               const float* dt_bias, const float* state_in, float* state_out,
                               float* out, int B, int Hqk, int Hv, int dk, int dv, float scale,
                               void* stream) {
    return gdn_decode_step_ex(q, k, v, a, b, gate_dtype, A_log, dt_bias, state_in, state_out, out, B, Hqk, Hv, dk,
                              dv, scale, 0, stream);
}
