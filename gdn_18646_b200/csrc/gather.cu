// gather.cu -- the all-gather of a head-sharded prefill output, one token window
// at a time, by the copy engines over NVLink.
//
// Config 4 splits the value heads over the GPUs of a node (one process each):
// rank r computes o for its H/world heads over the whole sequence, and every
// rank needs o of all heads.  Each rank holds a gathered buffer [world][o shape]
// whose slot r the prefill writes in place; the other slots are filled from the
// peers' buffers (CUDA IPC mappings).  Pulling a token window with one strided
// copy per peer (cudaMemcpy2DAsync between device pointers on different GPUs:
// a peer-to-peer copy-engine transfer) uses no SM, so it runs beside the next
// window's prefill, whose cooperative launch wants every SM.  The caller orders
// a pull after the peers' prefill of that window (a 1-element all-reduce on the
// copy stream) and before the peers rewrite their slots (one at the next call's
// start).
#include "common.cuh"

extern "C" int gdn_gather_window(void* gathered, const void* const* peer_gathered, int world, int rank, int B, int T,
                                 int H_local, int dv, int layout, int t0, int Tw, void* stream) {
    using namespace gdn;
    if (!gathered || !peer_gathered)
        return fail(GDN_ERR_NULL, "gdn_gather_window: gathered and peer_gathered are required");
    if (world < 1 || rank < 0 || rank >= world || B <= 0 || T <= 0 || H_local <= 0 || dv <= 0)
        return fail(GDN_ERR_SHAPE, "gdn_gather_window: bad world=%d rank=%d B=%d T=%d H_local=%d dv=%d", world, rank,
                    B, T, H_local, dv);
    if (layout != GDN_LAYOUT_BHTD && layout != GDN_LAYOUT_BTHD)
        return fail(GDN_ERR_DTYPE, "gdn_gather_window: layout must be GDN_LAYOUT_BHTD or GDN_LAYOUT_BTHD");
    if (t0 < 0 || Tw <= 0 || static_cast<long>(t0) + Tw > T)
        return fail(GDN_ERR_SHAPE, "gdn_gather_window: window [%d, %d + %d) outside T=%d", t0, t0, Tw, T);
    for (int p = 0; p < world; ++p)
        if (p != rank && !peer_gathered[p]) return fail(GDN_ERR_NULL, "gdn_gather_window: no buffer for rank %d", p);
    const size_t row = static_cast<size_t>(dv) * 2;                       // one token of one head, bytes
    const size_t slot = static_cast<size_t>(B) * H_local * T * row;      // one rank's o
    // a window is `height` runs of `width` bytes, `pitch` apart
    size_t off, width, pitch, height;
    if (layout == GDN_LAYOUT_BHTD) {                                       // [B, H_local, T, dv]
        off = t0 * row;
        width = Tw * row;
        pitch = T * row;
        height = static_cast<size_t>(B) * H_local;
    } else {                                                               // [B, T, H_local, dv]
        off = t0 * row * H_local;
        width = Tw * row * H_local;
        pitch = T * row * H_local;
        height = B;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 1; i < world; ++i) {
        const int p = (rank + i) % world;                                  // ranks start on different peers
        const size_t at = p * slot + off;
        const cudaError_t e = cudaMemcpy2DAsync(static_cast<uint8_t*>(gathered) + at, pitch,
                                                static_cast<const uint8_t*>(peer_gathered[p]) + at, pitch, width,
                                                height, cudaMemcpyDefault, s);
        if (e != cudaSuccess)
            return fail(GDN_ERR_CUDA, "gdn_gather_window: copy from rank %d: %s", p, cudaGetErrorString(e));
    }
    return GDN_OK;
}
