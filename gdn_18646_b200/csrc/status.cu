// status.cu -- thread-local error strings, device checks, the device-side
// error word, and TMA tensor-map encoding through the driver entry point.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tensormap.h"

namespace gdn {

namespace {
thread_local std::string t_last_error = "no error";

// One word per device, set by kernels that gave up on a bounded wait.
__device__ unsigned int g_device_error_word;

constexpr int kMaxDevices = 64;
std::once_flag g_dev_once[kMaxDevices];
int g_dev_status[kMaxDevices];
unsigned int* g_err_ptr[kMaxDevices];

std::once_flag g_encode_once;
PFN_encodeTiled g_encode = nullptr;
}  // namespace

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

static int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (*dev < 0 || *dev >= kMaxDevices) return fail(GDN_ERR_DEVICE, "device index %d out of range", *dev);
    return GDN_OK;
}

int check_sm100() {
    int dev = 0;
    int st = current_device(&dev);
    if (st != GDN_OK) return st;
    std::call_once(g_dev_once[dev], [dev]() {
        int major = 0, minor = 0;
        cudaError_t e1 = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaError_t e2 = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            g_dev_status[dev] = GDN_ERR_CUDA;
            return;
        }
        if (major != 10 || minor != 0) {
            g_dev_status[dev] = GDN_ERR_DEVICE;
            return;
        }
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) {
            g_dev_status[dev] = GDN_ERR_CUDA;
            return;
        }
        g_err_ptr[dev] = static_cast<unsigned int*>(p);
        g_dev_status[dev] = GDN_OK;
    });
    if (g_dev_status[dev] == GDN_ERR_DEVICE)
        return fail(GDN_ERR_DEVICE, "device %d is not an sm_100 (B200) part; this library is built for sm_100a only", dev);
    if (g_dev_status[dev] != GDN_OK)
        return fail(GDN_ERR_CUDA, "device %d: attribute / symbol query failed", dev);
    return GDN_OK;
}

unsigned int* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    return g_err_ptr[dev];
}

int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return GDN_OK;
}

PFN_encodeTiled tensor_map_encoder() {
    std::call_once(g_encode_once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
    });
    return g_encode;
}

int make_map_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
    PFN_encodeTiled enc = tensor_map_encoder();
    if (!enc) return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                     const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                     reinterpret_cast<const cuuint64_t*>(strides_bytes),
                     reinterpret_cast<const cuuint32_t*>(box),
                     reinterpret_cast<const cuuint32_t*>(elem_strides), CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return GDN_OK;
}

}  // namespace gdn

namespace gdn {
namespace {
thread_local int t_launch_overlap = 0;
}  // namespace
bool launch_overlap() { return t_launch_overlap != 0; }
}  // namespace gdn

extern "C" int gdn_set_launch_overlap(int on) {
    gdn::t_launch_overlap = on ? 1 : 0;
    return GDN_OK;
}

extern "C" const char* gdn_last_error(void) { return gdn::t_last_error.c_str(); }

extern "C" const char* gdn_version(void) { return "gdn_b200 0.1.0 (sm_100a)"; }

extern "C" int gdn_check_device_error(void) {
    int st = gdn::check_sm100();
    if (st != GDN_OK) return st;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return gdn::fail(GDN_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
    unsigned int word = 0;
    e = cudaMemcpy(&word, gdn::device_error_word(), sizeof(word), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return gdn::fail(GDN_ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
    if (word != 0) {
        unsigned int zero = 0;
        cudaMemcpy(gdn::device_error_word(), &zero, sizeof(zero), cudaMemcpyHostToDevice);
        if (word & gdn::DERR_TIMEOUT)
            return gdn::fail(GDN_ERR_DEVICE_TIMEOUT, "a kernel gave up on a bounded wait (device error word 0x%x)", word);
        return gdn::fail(GDN_ERR_SHAPE,
                         "gdn_prefill_varlen_fwd: cu_seqlens held offsets that are negative, decreasing or past Ttot; "
                         "those sequences were skipped (device error word 0x%x)",
                         word);
    }
    return GDN_OK;
}
