// rmsnorm.cu -- RMSNorm and the gated output RMSNorm, bf16 in/out, fp32 math.
//
// RMSNorm restates reference/rmsnorm_ref.py:24-28 (y = (x * rsqrt(mean(x^2)+eps)) * gamma,
// one bf16 rounding at the end) and replaces kernels/rmsnorm.cu (D=2048-only,
// scalar loads).  One warp per row; every lane moves 16-byte chunks (8 bf16),
// CPT chunks per lane held in registers between the reduction and the store,
// so each row is read once and written once.  gamma is read through L1.
#include "common.cuh"

namespace gdn {
namespace {

constexpr int kRowsPerBlock = 8;  // 8 warps per CTA, one row each

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(u[i] << 16);
        f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
}

// GATED = false: y = rmsnorm(x)*gamma.  GATED = true: y = rmsnorm(x)*gamma*silu(z);
// XF32: x is fp32 (else bf16).
template <int CPT, bool GATED, bool XF32>
__global__ void __launch_bounds__(32 * kRowsPerBlock)
rmsnorm_kernel(const void* __restrict__ xv, const uint16_t* __restrict__ z,
               const uint16_t* __restrict__ gamma, uint16_t* __restrict__ y, int R, int D, float eps) {
    pdl_launch_dependents();                   // the next kernel may launch (it waits for this one)
    pdl_wait_prior();                          // x and z come from earlier kernels
    // (x and z are read through L2 with ld.global.cg: under programmatic dependent launch
    // the kernel that writes them may still have been running when this one started)
    const int lane = threadIdx.x & 31;
    const long row = static_cast<long>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
    if (row >= R) return;
    const int nchunk = D >> 3;
    // bf16 rows stay packed in registers (4 words per chunk); fp32 rows as 8 floats
    uint4 xw[XF32 ? 1 : CPT];
    float xf[XF32 ? CPT : 1][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        const int ch = lane + 32 * c;
        if (ch < nchunk) {
            float f[8];
            if constexpr (XF32) {
                const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(xv) + row * D) + 2 * ch;
                const float4 u0 = __ldcg(p), u1 = __ldcg(p + 1);
                f[0] = u0.x; f[1] = u0.y; f[2] = u0.z; f[3] = u0.w;
                f[4] = u1.x; f[5] = u1.y; f[6] = u1.z; f[7] = u1.w;
#pragma unroll
                for (int i = 0; i < 8; ++i) xf[c][i] = f[i];
            } else {
                xw[c] = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xv) + row * D) + ch);
                unpack8(xw[c], f);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        const int ch = lane + 32 * c;
        if (ch < nchunk) {
            float f[8];
            if constexpr (XF32) {
#pragma unroll
                for (int i = 0; i < 8; ++i) f[i] = xf[c][i];
            } else {
                unpack8(xw[c], f);
            }
            float gf[8];
            unpack8(__ldg(reinterpret_cast<const uint4*>(gamma) + ch), gf);
            float o[8];
            if constexpr (GATED) {
                float zf[8];
                unpack8(__ldcg(reinterpret_cast<const uint4*>(z + row * D) + ch), zf);
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = (f[i] * r) * gf[i] * silu_fast(zf[i]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = (f[i] * r) * gf[i];
            }
            __stcs(reinterpret_cast<uint4*>(y + row * D) + ch, pack8(o));
        }
    }
}

// Rows of at most 16 chunks (D <= 128, e.g. the gated norm over one head's dv):
// a warp normalises 32/LPR rows, LPR lanes per row, one 16-byte chunk per lane,
// so no lane idles.  One warp per row group and no loop: a lane issues its x and z
// loads at once and holds few registers, so an SM keeps its full complement of
// warps (and their loads) in flight.  Same arithmetic and summation tree as
// rmsnorm_kernel (whose idle lanes add zeros).
template <int LPR, bool GATED, bool XF32>
__global__ void __launch_bounds__(32 * kRowsPerBlock)
rmsnorm_small_kernel(const void* __restrict__ xv, const uint16_t* __restrict__ z,
                     const uint16_t* __restrict__ gamma, uint16_t* __restrict__ y, int R, int D, float eps) {
    pdl_launch_dependents();
    pdl_wait_prior();
    constexpr int RPW = 32 / LPR;                  // rows per warp
    const int lane = threadIdx.x & 31, sub = lane / LPR, ch = lane % LPR;
    const long row = (static_cast<long>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5)) * RPW + sub;
    const bool on = ch < (D >> 3) && row < R;
    float f[8], zf[8];
    float ss = 0.f;
    if (on) {
        if constexpr (XF32) {
            const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(xv) + row * D) + 2 * ch;
            const float4 u0 = __ldcg(p), u1 = __ldcg(p + 1);
            f[0] = u0.x; f[1] = u0.y; f[2] = u0.z; f[3] = u0.w;
            f[4] = u1.x; f[5] = u1.y; f[6] = u1.z; f[7] = u1.w;
        } else {
            unpack8(__ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xv) + row * D) + ch), f);
        }
        if constexpr (GATED) unpack8(__ldcg(reinterpret_cast<const uint4*>(z + row * D) + ch), zf);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(D) + eps);
    if (on) {
        float gf[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(gamma) + ch), gf);
        float o[8];
        if constexpr (GATED) {
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (f[i] * r) * gf[i] * silu_fast(zf[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (f[i] * r) * gf[i];
        }
        __stcs(reinterpret_cast<uint4*>(y + row * D) + ch, pack8(o));
    }
}

template <bool GATED, bool XF32>
int launch_rmsnorm(const void* x, const void* z, const void* gamma, void* y, int R, int D, float eps,
                   cudaStream_t st, const char* name) {
    const int chunks_per_lane = (D / 8 + 31) / 32;
    const dim3 grid((R + kRowsPerBlock - 1) / kRowsPerBlock);
    const dim3 block(32 * kRowsPerBlock);
    auto* zz = static_cast<const uint16_t*>(z);
    auto* gg = static_cast<const uint16_t*>(gamma);
    auto* yy = static_cast<uint16_t*>(y);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = launch_overlap() ? 1 : 0;
    if (D <= 128) {                                 // small rows: several per warp, grid-stride
        const int lpr = D <= 64 ? 8 : 16;
        const long groups = (static_cast<long>(R) * lpr + 32 * kRowsPerBlock - 1) / (32 * kRowsPerBlock);
        if (groups > 0x7fffffffL) return fail(GDN_ERR_SHAPE, "%s: R=%d too large", name, R);
        cfg.gridDim = dim3(static_cast<unsigned>(groups));
        const cudaError_t e = lpr == 8 ? cudaLaunchKernelEx(&cfg, rmsnorm_small_kernel<8, GATED, XF32>, x, zz, gg, yy, R, D, eps)
                                       : cudaLaunchKernelEx(&cfg, rmsnorm_small_kernel<16, GATED, XF32>, x, zz, gg, yy, R, D, eps);
        if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s: launch failed: %s", name, cudaGetErrorString(e));
        return launch_status(name);
    }
#define GDN_RMS(N)                                                                           \
    if (chunks_per_lane <= N) {                                                              \
        const cudaError_t e = cudaLaunchKernelEx(&cfg, rmsnorm_kernel<N, GATED, XF32>, x, zz, gg, yy, R, D, eps); \
        if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s: launch failed: %s", name, cudaGetErrorString(e)); \
        return launch_status(name);                                                          \
    }
    GDN_RMS(1)
    GDN_RMS(2)
    GDN_RMS(4)
    GDN_RMS(8)
    GDN_RMS(16)
    if constexpr (!XF32) { GDN_RMS(32) }
#undef GDN_RMS
    return fail(GDN_ERR_UNSUPPORTED, "%s: D=%d too large", name, D);
}

int check_norm_args(const char* name, const void* x, const void* gamma, const void* y, int R, int D) {
    if (!x || !gamma || !y) return fail(GDN_ERR_NULL, "%s: x, gamma and y are required", name);
    if (R < 0 || D <= 0 || D % 8 != 0 || D > 8192)
        return fail(GDN_ERR_SHAPE, "%s: need R >= 0 and 0 < D <= 8192 with D %% 8 == 0 (got R=%d D=%d)", name, R, D);
    if (!aligned16(x) || !aligned16(gamma) || !aligned16(y))
        return fail(GDN_ERR_ALIGN, "%s: x, gamma and y must be 16-byte aligned", name);
    return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_rmsnorm_fwd(const void* x, const void* gamma, void* y, int R, int D, float eps,
                               void* stream) {
    using namespace gdn;
    int st = check_norm_args("gdn_rmsnorm_fwd", x, gamma, y, R, D);
    if (st != GDN_OK) return st;
    if ((st = check_sm100()) != GDN_OK) return st;
    if (R == 0) return GDN_OK;
    return launch_rmsnorm<false, false>(x, nullptr, gamma, y, R, D, eps, static_cast<cudaStream_t>(stream),
                                        "gdn_rmsnorm_fwd");
}

extern "C" int gdn_gated_rmsnorm_fwd(const void* x, int x_dtype, const void* z, const void* gamma, void* y,
                                     int R, int D, float eps, void* stream) {
    using namespace gdn;
    int st = check_norm_args("gdn_gated_rmsnorm_fwd", x, gamma, y, R, D);
    if (st != GDN_OK) return st;
    if (!z) return fail(GDN_ERR_NULL, "gdn_gated_rmsnorm_fwd: z is required");
    if (!aligned16(z)) return fail(GDN_ERR_ALIGN, "gdn_gated_rmsnorm_fwd: z must be 16-byte aligned");
    if (x_dtype != GDN_DTYPE_BF16 && x_dtype != GDN_DTYPE_F32)
        return fail(GDN_ERR_DTYPE, "gdn_gated_rmsnorm_fwd: x_dtype must be GDN_DTYPE_BF16 or GDN_DTYPE_F32");
    if ((st = check_sm100()) != GDN_OK) return st;
    if (R == 0) return GDN_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (x_dtype == GDN_DTYPE_F32)
        return launch_rmsnorm<true, true>(x, z, gamma, y, R, D, eps, s, "gdn_gated_rmsnorm_fwd");
    return launch_rmsnorm<true, false>(x, z, gamma, y, R, D, eps, s, "gdn_gated_rmsnorm_fwd");
}
