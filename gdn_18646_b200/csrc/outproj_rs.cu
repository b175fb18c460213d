// outproj_rs.cu -- head-sharded output projection fused with its reduce-scatter.
//
// With the value heads split over `world` GPUs (one process each), rank r holds
// the gated-normed outputs of its heads, x_r [M, K] (M = B*T tokens, K = its
// heads x dv), and the matching columns of the output projection, W_r [N, K].
// The layer output is y = sum_r x_r W_r^T [M, N]; each rank keeps the rows
// [rank * M/world, (rank + 1) * M/world) of it.  Instead of all-gathering o
// (M x 4096 bf16 at config 3's width) and running the whole projection on every
// rank, each rank computes its partial product and sends every 128 x 256 tile
// straight into the receive buffer of the rank that owns those rows, over
// NVLink peer memory, while its next tiles are still being multiplied; a
// local reduction then adds the `world` partials (gdn_outproj_reduce).  Half
// the bytes of the all-gather cross NVLink (N = hidden = 2048 bf16 per token
// instead of 4096), and the transfer is hidden under the GEMM.
//
// The GEMM is the projection kernel's: D[c, t] = sum_k W[c, k] x[t, k] with 128
// output channels on the TMEM lanes (tcgen05.mma M = 128) and 256 tokens on the
// columns (N = 256), persistent and warp-specialised (TMA producer, one MMA
// thread, 4 epilogue warps, 3-stage ring, two TMEM accumulators).  The epilogue
// rounds a tile to bf16, stages it in shared memory and copies it out row by
// row with 16-byte stores to the owner's buffer (peer or local: the kernel
// only sees device pointers).  No TMA touches peer memory and nothing waits on
// another GPU: the caller orders the reduction after every rank's launch.
#include <mutex>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {
namespace {

constexpr int RM = 128;               // output channels per tile (MMA M)
constexpr int RN = 256;               // tokens per tile (MMA N)
constexpr int RK = 64;                // K per stage (one 128-byte swizzle atom of bf16)
constexpr int RSTAGES = 3;
constexpr int RA_BYTES = RM * RK * 2;  // 16 KB
constexpr int RB_BYTES = RN * RK * 2;  // 32 KB
constexpr int RSTAGE_BYTES = RA_BYTES + RB_BYTES;
constexpr int RY_SUB = RN * 128;       // one 64-channel staging sub-tile: 256 tokens x 128 B
constexpr int ROFF_Y = RSTAGES * RSTAGE_BYTES;
constexpr int ROFF_BAR = ROFF_Y + 2 * RY_SUB;
constexpr int RS_SMEM = ROFF_BAR + 128 + 1024;
static_assert(RS_SMEM <= 232448, "outproj shared memory exceeds 227 KB");
constexpr int kRsThreads = 192;       // 6 warps
constexpr int kMaxWorld = 8;

struct RsArgs {
    uint16_t* dst[kMaxWorld];  // receive buffer of each rank: [world][rows][N] bf16
    unsigned int* err;
    int N, K, rows, rank;      // rows: tokens per rank
    int n_ct, ntiles;
};

__global__ void __launch_bounds__(kRsThreads, 1)
outproj_rs_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                  const RsArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + ROFF_BAR);   // [RSTAGES]
    uint64_t* empty = full + RSTAGES;                               // [RSTAGES]
    uint64_t* acc_full = empty + RSTAGES;                           // [2]
    uint64_t* acc_empty = acc_full + 2;                             // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* ysm = sm + ROFF_Y;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int nk = args.K / RK;

    if (tid == 0) {
        for (int s = 0; s < RSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], 4);
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&map_w);
        tma_prefetch_desc(&map_x);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (local operands only)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < args.ntiles; tile += gridDim.x) {
                const int ct = tile % args.n_ct, tt = tile / args.n_ct;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait_or_abort(&empty[stage], phase ^ 1u, args.err, abort_flag)) break;
                    uint8_t* st = sm + stage * RSTAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], RSTAGE_BYTES);
                    tma_load_2d(st, &map_w, &full[stage], kb * RK, ct * RM);
                    tma_load_2d(st + RA_BYTES, &map_x, &full[stage], kb * RK, tt * RN);
                    if (++stage == RSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (*abort_flag) break;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            constexpr uint32_t idesc = idesc_bf16(RM, RN, false, false);
            for (int tile = blockIdx.x; tile < args.ntiles; tile += gridDim.x, ++local) {
                const int abuf = local & 1;
                const uint32_t aphase = static_cast<uint32_t>(local >> 1) & 1u;
                if (!mbar_wait_or_abort(&acc_empty[abuf], aphase ^ 1u, args.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + abuf * RN;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait_or_abort(&full[stage], phase, args.err, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(sm + stage * RSTAGE_BYTES);
                    const uint32_t sb = sa + RA_BYTES;
#pragma unroll
                    for (int k = 0; k < RK / 16; ++k)
                        umma_bf16_ss(d_tmem, sdesc_sw128(sa + k * 32, 16, 1024), sdesc_sw128(sb + k * 32, 16, 1024),
                                     idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    umma_commit(&empty[stage]);
                    if (++stage == RSTAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (*abort_flag) break;
                umma_commit(&acc_full[abuf]);
            }
        }
    } else {
        // ---------------- epilogue: 4 warps, TMEM lanes 32*(warp%4) .. +31
        const int quad = warp & 3;
        const int cl = quad * 32 + lane;            // channel within the tile (= TMEM lane)
        const int et = tid - 64;                    // 0..127
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        uint8_t* ysub = ysm + (cl >> 6) * RY_SUB;
        const uint32_t ccol = cl & 63;
        int local = 0;
        for (int tile = blockIdx.x; tile < args.ntiles; tile += gridDim.x, ++local) {
            const int ct = tile % args.n_ct, tt = tile / args.n_ct;
            const int abuf = local & 1;
            const uint32_t aphase = static_cast<uint32_t>(local >> 1) & 1u;
            named_bar(1, 128);                          // the previous tile's copy-out left the staging buffer
            const bool ok = mbar_wait_or_abort(&acc_full[abuf], aphase, args.err, abort_flag);
            tc_fence_after();
#pragma unroll 1
            for (int blk = 0; blk < RN / 32; ++blk) {
                float acc[32];
                tmem_ld32(tmem + lane_off + abuf * RN + blk * 32, acc);
                tmem_ld_wait();
#pragma unroll
                for (int u = 0; u < 32; ++u)
                    *reinterpret_cast<uint16_t*>(ysub + sw128_off(blk * 32 + u, ccol)) = f32_to_bf16_bits(acc[u]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[abuf]);
            named_bar(1, 128);
            if (ok && !*abort_flag) {
                // the tile's 256 tokens belong to one rank (rows % 256 == 0): copy them into
                // slot `rank` of its receive buffer, 16 bytes per store, row by row
                const int t0 = tt * RN;
                const int owner = t0 / args.rows;
                uint16_t* dst = args.dst[owner] + (static_cast<long>(args.rank) * args.rows + (t0 - owner * args.rows)) *
                                                      args.N + ct * RM;
#pragma unroll 4
                for (int idx = et; idx < RN * 16; idx += 128) {
                    const int row = idx >> 4, c16 = idx & 15;
                    const uint4 v = *reinterpret_cast<const uint4*>(ysm + (c16 >> 3) * RY_SUB + sw128_chunk(row, c16 & 7));
                    *reinterpret_cast<uint4*>(dst + static_cast<long>(row) * args.N + c16 * 8) = v;
                }
            }
        }
        __threadfence_system();                        // the stores reach the owners before the kernel ends
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// out[r, c] = bf16(sum_s recv[s][r][c]), 8 channels per thread, in slot order.
__global__ void __launch_bounds__(256)
outproj_reduce_kernel(const uint16_t* __restrict__ recv, uint16_t* __restrict__ out, long n8, long slot_elems,
                      int world) {
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < world; ++s) {
            const uint4 v = __ldcg(reinterpret_cast<const uint4*>(recv + s * slot_elems) + i);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] += __uint_as_float(u[j] << 16);
                acc[2 * j + 1] += __uint_as_float(u[j] & 0xffff0000u);
            }
        }
        reinterpret_cast<uint4*>(out)[i] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                                      pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
    }
}

std::once_flag g_rs_attr_once[64];
int g_rs_attr_status[64];
int g_rs_sms[64];

}  // namespace
}  // namespace gdn

extern "C" int gdn_outproj_rs_fwd(const void* x, const void* W, void* const* recv, int M, int N, int K, int rank,
                                  int world, void* stream) {
    using namespace gdn;
    if (!x || !W || !recv) return fail(GDN_ERR_NULL, "gdn_outproj_rs_fwd: x, W and recv are required");
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
        return fail(GDN_ERR_SHAPE, "gdn_outproj_rs_fwd: need 1 <= world <= %d and 0 <= rank < world (got %d, %d)",
                    kMaxWorld, rank, world);
    if (M <= 0 || N <= 0 || K <= 0 || N % RM != 0 || K % RK != 0 || M % (RN * world) != 0)
        return fail(GDN_ERR_SHAPE,
                    "gdn_outproj_rs_fwd: need N %% 128 == 0, K %% 64 == 0 and M %% (256 * world) == 0 "
                    "(got M=%d N=%d K=%d world=%d)",
                    M, N, K, world);
    if (!aligned16(x) || !aligned16(W)) return fail(GDN_ERR_ALIGN, "gdn_outproj_rs_fwd: x and W must be 16-byte aligned");
    RsArgs a;
    for (int s = 0; s < kMaxWorld; ++s) a.dst[s] = nullptr;
    for (int s = 0; s < world; ++s) {
        if (!recv[s]) return fail(GDN_ERR_NULL, "gdn_outproj_rs_fwd: recv[%d] is NULL", s);
        if (!aligned16(recv[s])) return fail(GDN_ERR_ALIGN, "gdn_outproj_rs_fwd: recv[%d] must be 16-byte aligned", s);
        a.dst[s] = static_cast<uint16_t*>(recv[s]);
    }
    int st = check_sm100();
    if (st != GDN_OK) return st;
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(g_rs_attr_once[dev & 63], [dev]() {
        g_rs_attr_status[dev & 63] =
            cudaFuncSetAttribute(outproj_rs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RS_SMEM) == cudaSuccess
                ? GDN_OK
                : GDN_ERR_CUDA;
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_rs_sms[dev & 63] = sms > 0 ? sms : 148;
    });
    if (g_rs_attr_status[dev & 63] != GDN_OK)
        return fail(GDN_ERR_CUDA, "gdn_outproj_rs_fwd: cannot grant %d B of shared memory", RS_SMEM);
    CUtensorMap mw, mx;
    {
        uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
        uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
        uint32_t box[2] = {RK, RM};
        if ((st = make_map_bf16(&mw, W, 2, dims, strides, box, true)) != GDN_OK) return st;
    }
    {
        uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
        uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
        uint32_t box[2] = {RK, RN};
        if ((st = make_map_bf16(&mx, x, 2, dims, strides, box, true)) != GDN_OK) return st;
    }
    a.err = device_error_word();
    a.N = N;
    a.K = K;
    a.rows = M / world;
    a.rank = rank;
    a.n_ct = N / RM;
    const long ntiles = static_cast<long>(a.n_ct) * (M / RN);
    if (ntiles > 0x7fffffffL) return fail(GDN_ERR_SHAPE, "gdn_outproj_rs_fwd: too many tiles");
    a.ntiles = static_cast<int>(ntiles);
    const int grid = static_cast<int>(ntiles < g_rs_sms[dev & 63] ? ntiles : g_rs_sms[dev & 63]);
    outproj_rs_kernel<<<grid, kRsThreads, RS_SMEM, static_cast<cudaStream_t>(stream)>>>(mw, mx, a);
    return launch_status("gdn_outproj_rs_fwd");
}

extern "C" int gdn_outproj_reduce(const void* recv, void* out, int rows, int N, int world, void* stream) {
    using namespace gdn;
    if (!recv || !out) return fail(GDN_ERR_NULL, "gdn_outproj_reduce: recv and out are required");
    if (rows <= 0 || N <= 0 || N % 8 != 0 || world < 1 || world > kMaxWorld)
        return fail(GDN_ERR_SHAPE, "gdn_outproj_reduce: need rows > 0, N %% 8 == 0 and 1 <= world <= %d", kMaxWorld);
    if (!aligned16(recv) || !aligned16(out))
        return fail(GDN_ERR_ALIGN, "gdn_outproj_reduce: recv and out must be 16-byte aligned");
    int st = check_sm100();
    if (st != GDN_OK) return st;
    const long slot = static_cast<long>(rows) * N;
    const long n8 = slot / 8;
    const long blocks = (n8 + 255) / 256;
    const int grid = static_cast<int>(blocks < 148 * 8 ? blocks : 148 * 8);
    outproj_reduce_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(recv), static_cast<uint16_t*>(out), n8, slot, world);
    return launch_status("gdn_outproj_reduce");
}
