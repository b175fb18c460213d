// host_prefill.cu -- the prefill over HOST buffers, with the copies overlapped.
//
// A caller whose q, k, v, gates and state live in host memory pays for moving
// them over PCIe; copied one after another around a gdn_prefill_fwd_ws call,
// the copies take ~18x the prefill at config 1 (B=4, T=4096, 16 heads of 128).
// This entry point cuts the token axis into segments (multiples of the
// 64-token chunk but the last) and runs a three-stage pipeline:
//
//   copy-in stream   the gates (and mask) whole, once; then segment i's q, k,
//                    v -> device slot i % 2
//   caller's stream  prefill of segment i from slot i % 2, the state carried
//                    from segment i-1 through a device ping-pong pair
//   copy-out stream  segment i's output (and, after the last, the final
//                    state) -> host
//
// so the host-to-device copies, the prefill and the device-to-host copies of
// neighbouring segments run at the same time (the two copy directions use
// separate copy engines).  The call then lasts about as long as its
// host-to-device bytes take plus a tail: the last segment's prefill and
// read-back and the final state's read-back.  The automatic plan keeps the
// copies few and the tail short: segments of `seg` tokens, then halving
// lengths down to one chunk at the end (e.g. 1024 x 3, 512, 256, 128, 64, 64
// at config 1).  Each segment is an ordinary prefill call with a
// state carried in fp32, and segment boundaries fall on chunk boundaries, so
// the result is the one gdn_prefill_fwd gives on the whole sequence.
//
// Every copy is one cudaMemcpy2DAsync (strided rows of the host tensor into a
// dense device slot) or cudaMemcpyAsync with cudaMemcpyDefault, so host and
// device pointers are both accepted; host memory must be page-locked for the
// copies to overlap.  A copy costs ~4 us on the copy engine beyond its bytes,
// so a segment makes three (q, k, v) and the segment prefill reads its gates
// in place from the whole arrays (row stride T).
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace gdn {
namespace {

constexpr size_t kAlign = 256;
constexpr size_t kSegTargetBytes = 48u << 20;  // q, k, v bytes of the largest automatic segment (~0.9 ms over PCIe 5)

inline size_t up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct HostPlan {
    int seg = 0, nseg = 0;              // largest segment, segment count
    std::vector<int> start;             // segment i is tokens [start[i], start[i+1])
    size_t q = 0, k = 0, v = 0;                       // offsets inside an input slot
    size_t in_slot = 0, out_slot = 0, st = 0, gate = 0;
    size_t off_in = 0, off_out = 0, off_st = 0, off_gate = 0, off_par = 0, off_ws = 0, ws = 0, total = 0;
};

bool shape_ok(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype, int layout) {
    return B > 0 && T > 0 && Hqk > 0 && Hv > 0 && Hv % Hqk == 0 && (dk == 64 || dk == 128) &&
           (dv == 64 || dv == 128 || dv == 256) && (gate_dtype == GDN_DTYPE_BF16 || gate_dtype == GDN_DTYPE_F32) &&
           (layout == GDN_LAYOUT_BHTD || layout == GDN_LAYOUT_BTHD);
}

// Largest automatic segment: the multiple of 64 tokens whose q, k, v come
// closest to kSegTargetBytes from below (at least one chunk, at most T rounded up).
int auto_segment(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype) {
    (void)gate_dtype;
    const size_t per_tok = static_cast<size_t>(B) * (2 * Hqk * dk * 2 + Hv * dv * 2);
    long seg = static_cast<long>(kSegTargetBytes / per_tok) / GDN_CHUNK * GDN_CHUNK;
    const long tmax = (static_cast<long>(T) + GDN_CHUNK - 1) / GDN_CHUNK * GDN_CHUNK;
    if (seg < GDN_CHUNK) seg = GDN_CHUNK;
    if (seg > tmax) seg = tmax;
    return static_cast<int>(seg);
}

bool make_plan(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype, int seg_tokens, HostPlan& p) {
    p.seg = seg_tokens > 0 ? seg_tokens : auto_segment(B, T, Hqk, Hv, dk, dv, gate_dtype);
    if (p.seg % GDN_CHUNK != 0) return false;
    if (p.seg > T) p.seg = (T + GDN_CHUNK - 1) / GDN_CHUNK * GDN_CHUNK;
    p.start.clear();
    if (seg_tokens > 0) {                      // uniform segments, the last one ragged
        for (long t = 0; t < T; t += p.seg) p.start.push_back(static_cast<int>(t));
    } else {                                   // from the end: the ragged last chunk, then 64, 128, ... up to seg
        std::vector<int> len;
        long left = T;
        int next = static_cast<int>((T - 1) % GDN_CHUNK) + 1;
        while (left > 0) {
            const int l = static_cast<int>(std::min<long>(next, left));
            len.push_back(l);
            left -= l;
            if (len.size() > 1) next = std::min(2 * next, p.seg);
            else next = GDN_CHUNK;
        }
        long t = 0;
        for (auto it = len.rbegin(); it != len.rend(); ++it) {
            p.start.push_back(static_cast<int>(t));
            t += *it;
        }
    }
    p.start.push_back(T);
    p.nseg = static_cast<int>(p.start.size()) - 1;
    const size_t L = static_cast<size_t>(p.seg), es = gate_dtype == GDN_DTYPE_F32 ? 4 : 2;
    p.q = 0;
    p.k = p.q + up(B * Hqk * L * dk * 2);
    p.v = p.k + up(B * Hqk * L * dk * 2);
    p.in_slot = p.v + up(B * Hv * L * dv * 2);
    p.out_slot = up(B * Hv * L * dv * 2);
    p.st = up(static_cast<size_t>(B) * Hv * dk * dv * 4);
    p.gate = up(static_cast<size_t>(B) * Hv * T * es);     // a and b whole; mask [B, T] after them
    p.ws = gdn_prefill_workspace_bytes(B, p.seg, Hv, dk, dv);
    if (p.ws == 0) return false;
    p.off_in = 0;
    p.off_out = p.off_in + 2 * p.in_slot;
    p.off_st = p.off_out + 2 * p.out_slot;
    p.off_gate = p.off_st + 2 * p.st;
    p.off_par = p.off_gate + 2 * p.gate + up(static_cast<size_t>(B) * T * 4);
    p.off_ws = p.off_par + 2 * up(static_cast<size_t>(Hv) * 4);
    p.total = p.off_ws + up(p.ws);
    return true;
}

// Per-device copy streams and the events that order the pipeline, made once.
struct Pipe {
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t start = nullptr, in_done[2] = {}, comp_done[2] = {}, out_done[2] = {};
    int status = GDN_OK;
    std::mutex mu;
};
constexpr int kMaxDev = 64;
Pipe g_pipe[kMaxDev];
std::once_flag g_pipe_once[kMaxDev];

int pipe_for_device(Pipe** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev)
        return fail(GDN_ERR_CUDA, "gdn_prefill_host: no current CUDA device");
    Pipe& p = g_pipe[dev];
    std::call_once(g_pipe_once[dev], [&p]() {
        bool ok = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming) == cudaSuccess;
        for (int i = 0; i < 2 && ok; ++i)
            ok = cudaEventCreateWithFlags(&p.in_done[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&p.comp_done[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&p.out_done[i], cudaEventDisableTiming) == cudaSuccess;
        p.status = ok ? GDN_OK : GDN_ERR_CUDA;
    });
    if (p.status != GDN_OK) return fail(GDN_ERR_CUDA, "gdn_prefill_host: creating the copy streams failed");
    *out = &p;
    return GDN_OK;
}

// rows x width bytes, source rows spaced by spitch, into dense rows (or back)
inline cudaError_t copy_rows(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t rows,
                             cudaStream_t s) {
    return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyDefault, s);
}

}  // namespace
}  // namespace gdn

extern "C" size_t gdn_prefill_host_workspace_bytes(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype,
                                                   int seg_tokens) {
    using namespace gdn;
    if (!shape_ok(B, T, Hqk, Hv, dk, dv, gate_dtype, GDN_LAYOUT_BHTD) || seg_tokens < 0) return 0;
    HostPlan p;
    return make_plan(B, T, Hqk, Hv, dk, dv, gate_dtype, seg_tokens, p) ? p.total : 0;
}

extern "C" int gdn_prefill_host_segment(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype, int seg_tokens) {
    using namespace gdn;
    if (!shape_ok(B, T, Hqk, Hv, dk, dv, gate_dtype, GDN_LAYOUT_BHTD) || seg_tokens < 0) return -1;
    HostPlan p;
    return make_plan(B, T, Hqk, Hv, dk, dv, gate_dtype, seg_tokens, p) ? p.seg : -1;
}

extern "C" int gdn_prefill_host_plan(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype, int seg_tokens,
                                     int* starts, int cap) {
    using namespace gdn;
    if (!shape_ok(B, T, Hqk, Hv, dk, dv, gate_dtype, GDN_LAYOUT_BHTD) || seg_tokens < 0) return -1;
    HostPlan p;
    if (!make_plan(B, T, Hqk, Hv, dk, dv, gate_dtype, seg_tokens, p)) return -1;
    for (int i = 0; starts && i <= p.nseg && i < cap; ++i) starts[i] = p.start[i];
    return p.nseg;
}

extern "C" int gdn_prefill_host(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                                const void* b_logits, int gate_dtype, float dt_bias, const float* dt_bias_vec,
                                const float* mask, const float* state_in, void* out, float* state_out, int B, int T,
                                int Hqk, int Hv, int dk, int dv, int layout, float scale, int seg_tokens,
                                void* workspace, size_t workspace_bytes, void* stream) {
    using namespace gdn;
    if (!q || !k || !v || !A_log || !a || !b_logits || !out)
        return fail(GDN_ERR_NULL, "gdn_prefill_host: q, k, v, A_log, a, b_logits and out are required");
    if (!shape_ok(B, T, Hqk, Hv, dk, dv, gate_dtype, layout))
        return fail(GDN_ERR_SHAPE,
                    "gdn_prefill_host: bad shape or code (B=%d T=%d Hqk=%d Hv=%d dk=%d dv=%d gate_dtype=%d layout=%d)",
                    B, T, Hqk, Hv, dk, dv, gate_dtype, layout);
    if (seg_tokens < 0 || seg_tokens % GDN_CHUNK != 0)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_host: seg_tokens must be 0 (automatic) or a multiple of %d (got %d)",
                    GDN_CHUNK, seg_tokens);
    HostPlan p;
    if (!make_plan(B, T, Hqk, Hv, dk, dv, gate_dtype, seg_tokens, p))
        return fail(GDN_ERR_SHAPE, "gdn_prefill_host: no segment plan for these shapes");
    if (!workspace || workspace_bytes < p.total)
        return fail(GDN_ERR_SHAPE, "gdn_prefill_host: workspace of %zu B required, %zu B given", p.total,
                    workspace ? workspace_bytes : static_cast<size_t>(0));
    if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0)
        return fail(GDN_ERR_ALIGN, "gdn_prefill_host: workspace must be 256-byte aligned");
    int st = check_sm100();
    if (st != GDN_OK) return st;
    Pipe* pp = nullptr;
    if ((st = pipe_for_device(&pp)) != GDN_OK) return st;
    Pipe& P = *pp;
    std::lock_guard<std::mutex> lock(P.mu);

    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t es = gate_dtype == GDN_DTYPE_F32 ? 4 : 2;
    const bool bhtd = layout == GDN_LAYOUT_BHTD;
    float* stbuf[2] = {reinterpret_cast<float*>(ws + p.off_st), reinterpret_cast<float*>(ws + p.off_st + p.st)};
    uint8_t* ga_d = ws + p.off_gate;
    uint8_t* gb_d = ws + p.off_gate + p.gate;
    float* gm_d = reinterpret_cast<float*>(ws + p.off_gate + 2 * p.gate);
    float* alog_d = reinterpret_cast<float*>(ws + p.off_par);
    float* dtb_d = reinterpret_cast<float*>(ws + p.off_par + up(static_cast<size_t>(Hv) * 4));
    const size_t state_bytes = static_cast<size_t>(B) * Hv * dk * dv * 4;
    const char* what = nullptr;
    cudaError_t e = cudaSuccess;
    int nseg_done = 0;

    // the copy streams start after the caller's earlier work
    if ((e = cudaEventRecord(P.start, cs)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(P.in, P.start, 0)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(P.out, P.start, 0)) != cudaSuccess)
        return fail(GDN_ERR_CUDA, "gdn_prefill_host: ordering the copy streams: %s", cudaGetErrorString(e));
    const size_t gate_bytes = static_cast<size_t>(B) * Hv * T * es;
    if ((e = cudaMemcpyAsync(alog_d, A_log, Hv * 4, cudaMemcpyDefault, P.in)) != cudaSuccess ||
        (dt_bias_vec && (e = cudaMemcpyAsync(dtb_d, dt_bias_vec, Hv * 4, cudaMemcpyDefault, P.in)) != cudaSuccess) ||
        (e = cudaMemcpyAsync(ga_d, a, gate_bytes, cudaMemcpyDefault, P.in)) != cudaSuccess ||
        (e = cudaMemcpyAsync(gb_d, b_logits, gate_bytes, cudaMemcpyDefault, P.in)) != cudaSuccess ||
        (mask && (e = cudaMemcpyAsync(gm_d, mask, static_cast<size_t>(B) * T * 4, cudaMemcpyDefault, P.in)) !=
                     cudaSuccess) ||
        (state_in && (e = cudaMemcpyAsync(stbuf[1], state_in, state_bytes, cudaMemcpyDefault, P.in)) != cudaSuccess))
        what = "copying A_log, dt_bias, the gates, the mask and state_in";

    for (int i = 0; i < p.nseg && !what && st == GDN_OK; ++i) {
        const int s = i & 1;
        const size_t t0 = static_cast<size_t>(p.start[i]);
        const size_t len = static_cast<size_t>(p.start[i + 1] - p.start[i]);
        uint8_t* in = ws + p.off_in + s * p.in_slot;
        uint8_t* o = ws + p.off_out + s * p.out_slot;
        // ---- copy-in of q, k, v: wait until the prefill two segments back has read this slot
        if (i >= 2 && (e = cudaStreamWaitEvent(P.in, P.comp_done[s], 0)) != cudaSuccess) {
            what = "ordering the copy-in stream";
            break;
        }
        const uint8_t* qh = static_cast<const uint8_t*>(q);
        const uint8_t* kh = static_cast<const uint8_t*>(k);
        const uint8_t* vh = static_cast<const uint8_t*>(v);
        if (bhtd) {   // rows (b, h), each len tokens of a T-token row
            e = copy_rows(in + p.q, len * dk * 2, qh + t0 * dk * 2, static_cast<size_t>(T) * dk * 2, len * dk * 2,
                          static_cast<size_t>(B) * Hqk, P.in);
            if (e == cudaSuccess)
                e = copy_rows(in + p.k, len * dk * 2, kh + t0 * dk * 2, static_cast<size_t>(T) * dk * 2, len * dk * 2,
                              static_cast<size_t>(B) * Hqk, P.in);
            if (e == cudaSuccess)
                e = copy_rows(in + p.v, len * dv * 2, vh + t0 * dv * 2, static_cast<size_t>(T) * dv * 2, len * dv * 2,
                              static_cast<size_t>(B) * Hv, P.in);
        } else {      // rows b, each len tokens x H heads of a T-token row
            const size_t rq = static_cast<size_t>(Hqk) * dk * 2, rv = static_cast<size_t>(Hv) * dv * 2;
            e = copy_rows(in + p.q, len * rq, qh + t0 * rq, T * rq, len * rq, B, P.in);
            if (e == cudaSuccess) e = copy_rows(in + p.k, len * rq, kh + t0 * rq, T * rq, len * rq, B, P.in);
            if (e == cudaSuccess) e = copy_rows(in + p.v, len * rv, vh + t0 * rv, T * rv, len * rv, B, P.in);
        }
        if (e == cudaSuccess) e = cudaEventRecord(P.in_done[s], P.in);
        if (e != cudaSuccess) {
            what = "copying a segment in";
            break;
        }
        // ---- prefill on the caller's stream, after the copy-in and after the
        //      read-back two segments back has drained this output slot
        if ((e = cudaStreamWaitEvent(cs, P.in_done[s], 0)) != cudaSuccess ||
            (i >= 2 && (e = cudaStreamWaitEvent(cs, P.out_done[s], 0)) != cudaSuccess)) {
            what = "ordering the prefill";
            break;
        }
        const float* sin = i == 0 ? (state_in ? stbuf[1] : nullptr) : stbuf[(i - 1) & 1];
        st = prefill_segment(in + p.q, in + p.k, in + p.v, alog_d, ga_d + t0 * es, gb_d + t0 * es, gate_dtype, dt_bias,
                             dt_bias_vec ? dtb_d : nullptr, mask ? gm_d + t0 : nullptr, sin, o, stbuf[i & 1], B,
                             static_cast<int>(len), Hqk, Hv, dk, dv, layout, scale, ws + p.off_ws, p.ws, cs, T);
        if (st != GDN_OK) break;                  // the prefill's own message stands
        if ((e = cudaEventRecord(P.comp_done[s], cs)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(P.out, P.comp_done[s], 0)) != cudaSuccess) {
            what = "ordering the copy-out stream";
            break;
        }
        // ---- copy-out
        if (bhtd) {
            e = copy_rows(static_cast<uint8_t*>(out) + t0 * dv * 2, static_cast<size_t>(T) * dv * 2, o, len * dv * 2,
                          len * dv * 2, static_cast<size_t>(B) * Hv, P.out);
        } else {
            const size_t rv = static_cast<size_t>(Hv) * dv * 2;
            e = copy_rows(static_cast<uint8_t*>(out) + t0 * rv, T * rv, o, len * rv, len * rv, B, P.out);
        }
        if (e == cudaSuccess && i == p.nseg - 1 && state_out)
            e = cudaMemcpyAsync(state_out, stbuf[i & 1], state_bytes, cudaMemcpyDefault, P.out);
        if (e == cudaSuccess) e = cudaEventRecord(P.out_done[s], P.out);
        if (e != cudaSuccess) {
            what = "copying a segment out";
            break;
        }
        nseg_done = i + 1;
    }
    // join both copy streams back into the caller's stream, also after an error
    cudaError_t ej = cudaEventRecord(P.in_done[0], P.in);
    if (ej == cudaSuccess) ej = cudaStreamWaitEvent(cs, P.in_done[0], 0);
    if (ej == cudaSuccess) ej = cudaEventRecord(P.out_done[0], P.out);
    if (ej == cudaSuccess) ej = cudaStreamWaitEvent(cs, P.out_done[0], 0);
    if (st != GDN_OK) return st;
    if (what) return fail(GDN_ERR_CUDA, "gdn_prefill_host: %s (segment %d): %s", what, nseg_done, cudaGetErrorString(e));
    if (ej != cudaSuccess)
        return fail(GDN_ERR_CUDA, "gdn_prefill_host: joining the copy streams: %s", cudaGetErrorString(ej));
    return GDN_OK;
}
