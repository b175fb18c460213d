/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet hot path.
 *
 * Every entry point takes raw DEVICE pointers (gdn_prefill_host also host
 * ones), explicit shapes, a CUDA
 * stream (passed as void*, a cudaStream_t; NULL = legacy default stream) and
 * returns an int status (GDN_OK == 0).  Launches are asynchronous on that
 * stream; no entry point synchronises, and only gdn_prefill_fwd allocates
 * (its workspace, stream-ordered; gdn_prefill_fwd_ws takes it from the
 * caller instead).  On error
 * nothing is launched and gdn_last_error() describes the problem (the message
 * is per calling thread).
 *
 * bf16 tensors are raw 16-bit buffers (__nv_bfloat16 / torch.bfloat16).
 * Each declaration names the reference interface it replaces
 * (diacccc/GDN_18646, file:line).
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
enum {
    GDN_OK = 0,
    GDN_ERR_NULL = 1,        /* a required pointer is NULL                     */
    GDN_ERR_SHAPE = 2,       /* a size is out of range or inconsistent         */
    GDN_ERR_DTYPE = 3,       /* unknown dtype / layout code                    */
    GDN_ERR_ALIGN = 4,       /* a pointer is not 16-byte aligned               */
    GDN_ERR_UNSUPPORTED = 5, /* head dims or widths this build does not cover  */
    GDN_ERR_CUDA = 6,        /* a CUDA runtime/driver call or launch failed    */
    GDN_ERR_DEVICE = 7,      /* the current device is not an sm_100 part       */
    GDN_ERR_DEVICE_TIMEOUT = 8, /* a kernel gave up on a bounded wait          */
    GDN_ERR_ARG = 9          /* an option value (schedule, gate layout) out of range */
};

/* dtype codes for gate / activation inputs */
enum { GDN_DTYPE_BF16 = 0, GDN_DTYPE_F32 = 1 };

/* activation layouts: [B, H, T, D] (the reference's) or [B, T, H, D] */
enum { GDN_LAYOUT_BHTD = 0, GDN_LAYOUT_BTHD = 1 };

/* Chunk length of the prefill kernel (the reference's C_DIM,
 * kernels/prefill_chunked.cu:18). */
#define GDN_CHUNK 64

/*
 * Chunked gated-delta-rule prefill.
 * Replaces gdn_prefill() / the "prefill" pybind op,
 * kernels/prefill_chunked.cu:422-504 and :512-521 (math: reference/prefill_ref.py:11-132).
 *
 *   q, k       bf16 [B, Hqk, T, dk] (layout BHTD) or [B, T, Hqk, dk] (BTHD)
 *   v          bf16 [B, Hv, T, dv]  or [B, T, Hv, dv]
 *   A_log      f32  [Hv]
 *   a, b_logits [B, Hv, T] in gate_dtype (bf16 or f32)
 *   dt_bias    scalar, used when dt_bias_vec == NULL; else dt_bias_vec f32 [Hv]
 *   mask       f32 [B, T] or NULL (all ones)
 *   state_in   f32 [B, Hv, dk, dv] or NULL (zeros)     (the reference's empty tensor)
 *   out        bf16, same layout as v
 *   state_out  f32 [B, Hv, dk, dv] (may be NULL: final state not written)
 *   scale      0.0f -> 1/sqrt(dk)  (reference/prefill_ref.py:45-46)
 * Value head h reads q/k head h / (Hv / Hqk) (grouped value heads; Hqk == Hv
 * is the reference's case).  Supported: dk in {64, 128}, dv in {64, 128, 256},
 * any T >= 1 (a ragged last chunk is handled like the reference's padding),
 * Hv % Hqk == 0.  Pointers must be 16-byte aligned.
 */
int gdn_prefill_fwd(const void* q, const void* k, const void* v,
                    const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                    float dt_bias, const float* dt_bias_vec,
                    const float* mask, const float* state_in,
                    void* out, float* state_out,
                    int B, int T, int Hqk, int Hv, int dk, int dv, int layout,
                    float scale, void* stream);

/*
 * Bytes of device workspace gdn_prefill_fwd_ws needs (0 for invalid shapes):
 * one chunk record per (batch, value head, 64-token chunk), 59 KB at dk=128,
 * 43 KB at dk=64, plus one fp32 state [B, Hv, dk, dv] and a 4-byte ready flag
 * per record (rounded up to 128 B).  No counterpart in the
 * reference, whose kernel keeps everything in shared memory.
 */
size_t gdn_prefill_workspace_bytes(int B, int T, int Hv, int dk, int dv);

/*
 * Prefill launch schedule (default GDN_SCHEDULE_AUTO).  gdn_prefill_set_schedule
 * sets the default for calls made from the CALLING HOST THREAD only (other
 * threads keep theirs); gdn_prefill_fwd_ex takes the schedule per call.
 *   SINGLE  one prep launch over all chunks, then one chain launch;
 *   PIECED  the chunks cut into up to 4 pieces, the chain of piece k running
 *           in the same launch as the prep of piece k+1;
 *   STREAM  after the gates, a prep launch over the first chunks of every
 *           sequence (as many as a cost model finds best, possibly none),
 *           then one cooperative launch: the chain CTAs and, on every other
 *           SM, prep workers producing the remaining chunk records
 *           chunk-major; a chain CTA waits (bounded) for each record's ready
 *           flag.  Needs fewer chain CTAs (B * Hv * ceil(dv/128)) than SMs;
 *   AUTO    the one a cost model predicts fastest.
 * Results are identical up to fp32 summation order.  No counterpart in the
 * reference (single kernel).
 */
enum { GDN_SCHEDULE_AUTO = 0, GDN_SCHEDULE_SINGLE = 1, GDN_SCHEDULE_PIECED = 2, GDN_SCHEDULE_STREAM = 3 };
int gdn_prefill_set_schedule(int mode);      /* GDN_ERR_ARG for an unknown mode */

/* Kernel launches one gdn_prefill_fwd call makes on the current device under
 * the calling thread's schedule (3 for SINGLE, 2 or 3 for STREAM), or -1 for
 * invalid shapes / no device; _ex: under the given schedule. */
int gdn_prefill_launch_count(int B, int T, int Hv, int dk, int dv);
int gdn_prefill_launch_count_ex(int B, int T, int Hv, int dk, int dv, int schedule);

/*
 * Per-call options of gdn_prefill_fwd_ex.  No counterpart in the reference.
 *   schedule     GDN_SCHEDULE_* for this call (AUTO: the cost model's choice).
 *   gate_layout  GDN_GATES_BHT: a, b_logits [B, Hv, T] (the reference's layout);
 *                GDN_GATES_BTH: one row of gate_ld elements per token, [B, T, gate_ld],
 *                head h at column h -- e.g. the a and b halves of a [B, T, 2 Hv]
 *                projection output read in place (b_logits = a + Hv, gate_ld = 2 Hv).
 *   gate_ld      GDN_GATES_BTH: elements between consecutive tokens' rows (>= Hv).
 */
enum { GDN_GATES_BHT = 0, GDN_GATES_BTH = 1 };
typedef struct {
    int schedule;
    int gate_layout;
    long gate_ld;
} gdn_prefill_opts;

/*
 * gdn_prefill_fwd_ws with per-call options (opts == NULL: AUTO schedule, BHT
 * gates).  The mask stays [B, T].  Errors as gdn_prefill_fwd_ws, plus
 * GDN_ERR_ARG for an unknown schedule or gate layout and GDN_ERR_SHAPE for a
 * gate_ld below Hv.
 */
int gdn_prefill_fwd_ex(const void* q, const void* k, const void* v,
                       const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                       float dt_bias, const float* dt_bias_vec,
                       const float* mask, const float* state_in,
                       void* out, float* state_out,
                       int B, int T, int Hqk, int Hv, int dk, int dv, int layout,
                       float scale, const gdn_prefill_opts* opts,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * gdn_prefill_fwd with a caller-provided workspace (device memory,
 * 128-byte aligned, at least gdn_prefill_workspace_bytes(B, T, Hv, dk, dv)
 * bytes, not used by other work on the stream while the call runs).
 * gdn_prefill_fwd itself takes the workspace from the stream-ordered
 * allocator (cudaMallocAsync / cudaFreeAsync on `stream`).
 */
int gdn_prefill_fwd_ws(const void* q, const void* k, const void* v,
                       const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                       float dt_bias, const float* dt_bias_vec,
                       const float* mask, const float* state_in,
                       void* out, float* state_out,
                       int B, int T, int Hqk, int Hv, int dk, int dv, int layout,
                       float scale, void* workspace, size_t workspace_bytes, void* stream);

/*
 * gdn_prefill_fwd_ws over the token window [t0, t0 + Tw) of tensors that hold T
 * tokens per sequence.  q, k, v, out, a, b_logits and mask are the WHOLE tensors
 * (read and written in place at the window's tokens; nothing is copied);
 * state_in is the state before token t0 (NULL: zeros), state_out the state
 * after token t0 + Tw - 1.  The workspace is sized for the window:
 * gdn_prefill_workspace_bytes(B, Tw, Hv, dk, dv).  Windows chained through
 * their states give the whole call's o and final state, bit-identical when
 * every window starts on a 64-token chunk boundary.  Used to overlap the
 * all-gather of a head-sharded o with the prefill (a window's o is shipped
 * while the next window runs).  No counterpart in the reference.
 * Errors: GDN_ERR_SHAPE when the window leaves [0, T); otherwise as
 * gdn_prefill_fwd_ws.
 */
int gdn_prefill_window_ws(const void* q, const void* k, const void* v,
                          const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                          float dt_bias, const float* dt_bias_vec,
                          const float* mask, const float* state_in,
                          void* out, float* state_out,
                          int B, int T, int t0, int Tw, int Hqk, int Hv, int dk, int dv, int layout,
                          float scale, void* workspace, size_t workspace_bytes, void* stream);

/*
 * gdn_prefill_fwd for callers that cannot allocate device memory.  No
 * counterpart in the reference, whose kernel needs no workspace.
 *
 * The prefill needs a workspace (one record per 64-token chunk, see
 * gdn_prefill_workspace_bytes).  Some callers cannot get one at call time:
 * an engine that reserved the GPU's memory up front for its own pools (a
 * cudaMalloc would fail or fragment that reservation), or a plugin whose
 * host forbids allocation inside its execute callback.  This entry point
 * takes the workspace from a 32 MiB array compiled into the library (held on
 * every GPU that loads the library until the process exits) and makes no
 * cudaMalloc, cudaMallocAsync or other allocating call.
 *
 *   - Limit: problems with gdn_prefill_workspace_bytes(B, T, Hv, dk, dv) > 32 MiB
 *     return GDN_ERR_UNSUPPORTED (about 540 chunk records at dk = 128, e.g.
 *     8 sequences of 4096 tokens); use gdn_prefill_fwd_ws for larger ones.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, once per device); make that first call before
 *     any stream capture.  The address is kept for the life of the process:
 *     after a cudaDeviceReset (or anything else that recreates the device's
 *     primary context) this entry point must not be called again.
 *   - Every call uses the same array, which keeps the previous call's
 *     contents; each call writes every value it uses before using it, so
 *     nothing needs clearing.  Calls that overlap on the GPU (different
 *     streams, different host threads) race on it: order them.
 * Same arguments, status codes and results as gdn_prefill_fwd.
 */
int gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v,
                            const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                            float dt_bias, const float* dt_bias_vec,
                            const float* mask, const float* state_in,
                            void* out, float* state_out,
                            int B, int T, int Hqk, int Hv, int dk, int dv, int layout,
                            float scale, void* stream);

/*
 * Variable-length prefill: N sequences packed along the token axis (no padding).
 * No reference counterpart (the reference kernel takes equal-length batches,
 * kernels/prefill_chunked.cu:422-504); per sequence the result is that of
 * gdn_prefill_fwd on that sequence alone.
 *
 *   q, k        bf16 [Ttot, Hqk, dk];  v, out bf16 [Ttot, Hv, dv]
 *   a, b_logits [Hv, Ttot] in gate_dtype
 *   cu_seqlens  int32 [N + 1], DEVICE memory: sequence i is tokens
 *               [cu_seqlens[i], cu_seqlens[i+1]); cu_seqlens[0] = 0,
 *               non-decreasing, cu_seqlens[N] = Ttot.  Empty sequences pass
 *               their state through.
 *   max_len     host int, at least the longest sequence (sizes the workspace
 *               and the launch; a longer sequence is processed only up to
 *               max_len rounded up to 64 tokens).
 *   state_in    f32 [N, Hv, dk, dv] or NULL (zeros);  state_out f32 [N, Hv, dk, dv] or NULL
 * Offsets that are negative, decreasing or past Ttot cannot be seen on the host
 * (the array is on the device): such a sequence is skipped and
 * gdn_check_device_error() reports GDN_ERR_SHAPE.  Always one prep and one
 * chain launch after the gates (3 launches).  Mask is not supported here.
 * Workspace: gdn_prefill_varlen_workspace_bytes(N, max_len, Hv, dk, dv).
 */
size_t gdn_prefill_varlen_workspace_bytes(int N, int max_len, int Hv, int dk, int dv);
int gdn_prefill_varlen_fwd_ws(const void* q, const void* k, const void* v,
                              const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                              float dt_bias, const float* dt_bias_vec,
                              const int* cu_seqlens, int N, int Ttot, int max_len,
                              const float* state_in, void* out, float* state_out,
                              int Hqk, int Hv, int dk, int dv, float scale,
                              void* workspace, size_t workspace_bytes, void* stream);
int gdn_prefill_varlen_fwd(const void* q, const void* k, const void* v,
                           const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                           float dt_bias, const float* dt_bias_vec,
                           const int* cu_seqlens, int N, int Ttot, int max_len,
                           const float* state_in, void* out, float* state_out,
                           int Hqk, int Hv, int dk, int dv, float scale, void* stream);

/*
 * Prefill over HOST buffers (the reference's pybind op with CPU tensors moved
 * to the GPU around it, kernels/prefill_chunked.cu:512-521): the same
 * arguments and result as gdn_prefill_fwd, but q, k, v, a, b_logits, mask,
 * state_in, out and state_out may be host memory (page-locked, for the copies
 * to overlap) or device memory; A_log and dt_bias_vec too.  The token axis is
 * cut into segments of seg_tokens tokens (0 = automatic, else a multiple of
 * 64); segment i+1 is copied in while segment i runs on `stream` and segment
 * i-1 is copied out, on two copy streams of the library's own that wait on
 * `stream` at the start and that `stream` waits on at the end.  The result is
 * the one gdn_prefill_fwd gives on the whole sequence.  Host outputs are
 * valid after `stream` completes.  Calls on one device are serialised on the
 * host (a mutex) while they enqueue.
 * Workspace: device memory, 256-byte aligned, of
 * gdn_prefill_host_workspace_bytes(B, T, Hqk, Hv, dk, dv, gate_dtype, seg_tokens)
 * bytes (two segments of inputs and outputs, two states, the gates whole, the
 * prefill's own workspace for one segment).  gdn_prefill_host_segment returns
 * the largest segment a call would use, gdn_prefill_host_plan the segment
 * count and (when starts != NULL) up to cap segment boundaries
 * starts[0] = 0 < ... < starts[nseg] = T; both -1 for invalid shapes.  The
 * automatic plan (seg_tokens 0) uses full segments, then halving ones down to
 * a single chunk at the end, so the last prefill and read-back are short.
 * These three are host-only.
 */
size_t gdn_prefill_host_workspace_bytes(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype,
                                        int seg_tokens);
int gdn_prefill_host_segment(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype, int seg_tokens);
int gdn_prefill_host_plan(int B, int T, int Hqk, int Hv, int dk, int dv, int gate_dtype, int seg_tokens,
                          int* starts, int cap);
int gdn_prefill_host(const void* q, const void* k, const void* v,
                     const float* A_log, const void* a, const void* b_logits, int gate_dtype,
                     float dt_bias, const float* dt_bias_vec,
                     const float* mask, const float* state_in,
                     void* out, float* state_out,
                     int B, int T, int Hqk, int Hv, int dk, int dv, int layout,
                     float scale, int seg_tokens, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Gradients of the prefill (training): dq, dk, dv, da, db, dA_log, ddt_bias and
 * the initial state, given dO (and optionally the gradient of the final state).
 * No reference counterpart (the reference has no backward).  The derivative of
 * the same recurrence (per token S' = g S, r = S'^T k, d = b'(v - r),
 * S <- S' + k d^T, o = m scale q^T S), computed in fp32.
 *   q, k bf16 [B, H, T, dk]; v bf16 [B, H, T, dv]   (layout BHTD, Hqk == Hv)
 *   A_log f32 [H]; a, b_logits [B, H, T] in gate_dtype; dt_bias / dt_bias_vec as
 *   gdn_prefill_fwd; mask f32 [B, T] or NULL; state_in f32 [B, H, dk, dv] or NULL
 *   dO [B, H, T, dv] in do_dtype (bf16 or f32); dS_final f32 [B, H, dk, dv] or NULL
 *   dq, dk f32 [B, H, T, dk]; dv f32 [B, H, T, dv]; da, db f32 [B, H, T]
 *   dA_log, ddt_bias f32 [H] (per head; for a scalar dt_bias sum them);
 *   dstate_in f32 [B, H, dk, dv] or NULL.
 * dk, dv in {64, 128}.  Two algorithms (gdn_prefill_bwd_set_algorithm):
 *   chunked (the default): per 64-token chunk, the chunk's matrices and the
 *     per-token gradients on tcgen05 (bf16 hi/lo operands, fp32 accumulate) from
 *     the state at every chunk start and its gradient at every chunk end, which two
 *     recurrences over the chunks produce; q, k, v, dO, dq, dk, dv 16-byte aligned
 *     (GDN_ERR_ALIGN).  Workspace about B H T (dk dv / 8 + 10 dv + 6 dk + 1328)
 *     bytes (config 1: 1.42 GB);
 *   token-recurrent: fp32 on CUDA cores, in token windows, last first: a checkpoint
 *     pass stores the state at every window start, and only one window's per-token
 *     states are held at a time.  Workspace about B H dk dv 4 (T / W + W) bytes for
 *     windows of W tokens (config 1: 1.2 GB).  The window is max(256, sqrt T)
 *     tokens, or the calling thread's gdn_prefill_bwd_set_window.
 * Workspace: gdn_prefill_bwd_workspace_bytes(B, T, H, dk, dv), 16-byte aligned; the
 * workspace size and the call must see the same algorithm and window settings.
 */
size_t gdn_prefill_bwd_workspace_bytes(int B, int T, int H, int dk, int dv);
/* The calling thread's window for gdn_prefill_bwd, in tokens (0 = automatic).
 * GDN_ERR_ARG for a negative value. */
int gdn_prefill_bwd_set_window(int tokens);
/* The calling thread's backward algorithm:
 *   GDN_BWD_TOKEN    the token-recurrent windows above;
 *   GDN_BWD_CHUNKED  chunk by chunk (64 tokens): only the state at every chunk start and
 *                    its gradient at every chunk end are carried, the per-token gradients
 *                    come from chunk-local products (workspace above; no windows);
 *   GDN_BWD_AUTO     the library's choice (the default): chunked.
 * The workspace size and the call must see the same setting.  GDN_ERR_ARG otherwise. */
enum { GDN_BWD_AUTO = 0, GDN_BWD_TOKEN = 1, GDN_BWD_CHUNKED = 2 };
int gdn_prefill_bwd_set_algorithm(int algorithm);
int gdn_prefill_bwd(const void* q, const void* k, const void* v, const float* A_log,
                    const void* a, const void* b_logits, int gate_dtype, float dt_bias,
                    const float* dt_bias_vec, const float* mask, const float* state_in,
                    const void* dO, int do_dtype, const float* dS_final,
                    float* dq, float* dk, float* dv, float* da, float* db,
                    float* dA_log, float* ddt_bias, float* dstate_in,
                    int B, int T, int H, int dk_dim, int dv_dim, float scale,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Single-token decode step, state updated in place if state_out == state_in.
 * Replaces gdn_decode_cuda(), kernels/decode.cu:131-162, and its torch wrapper
 * gdn_decode_forward(), kernels/decode.cu:172-214 (math: reference/decode_ref.py:11-61).
 *
 *   q, k       bf16 [B, Hqk, dk];  v bf16 [B, Hv, dv]
 *   a, b       [B, Hv] in gate_dtype
 *   A_log, dt_bias  f32 [Hv] (dt_bias may be NULL = 0)
 *   state_in   f32 [B, Hv, dk, dv];  state_out f32 [B, Hv, dk, dv] (may alias state_in)
 *   out        f32 [B, Hv, dv]
 *   scale      0.0f -> 1/sqrt(dk)
 * Supported: dk, dv in {64, 128, 256}.
 */
int gdn_decode_step(const void* q, const void* k, const void* v,
                    const void* a, const void* b, int gate_dtype,
                    const float* A_log, const float* dt_bias,
                    const float* state_in, float* state_out, float* out,
                    int B, int Hqk, int Hv, int dk, int dv, float scale, void* stream);

/*
 * gdn_decode_step with options.  flags: GDN_DECODE_L2NORM_QK L2-normalises q and k
 * per head first (fp32 sum of squares, eps 1e-6, result rounded to bf16), the
 * layer's q/k norm, so the projection before it needs no cross-CTA reduction.
 * No reference counterpart (the reference layer normalises in its own glue).
 */
enum { GDN_DECODE_L2NORM_QK = 1 };
int gdn_decode_step_ex(const void* q, const void* k, const void* v,
                       const void* a, const void* b, int gate_dtype,
                       const float* A_log, const float* dt_bias,
                       const float* state_in, float* state_out, float* out,
                       int B, int Hqk, int Hv, int dk, int dv, float scale, int flags, void* stream);

/*
 * gdn_decode_step_ex followed by the layer's gated output norm of each head's o
 * row, in the same kernel: y = (o * rsqrt(mean(o^2) + eps)) * norm_gamma *
 * silu(z), bf16 (gdn_gated_rmsnorm_fwd over rows of dv with an fp32 o, up to the
 * order of the fp32 sum of squares).  z bf16 [B, Hv, dv], norm_gamma bf16 [dv],
 * y bf16 [B, Hv, dv], all 8-byte aligned; out (the fp32 o) may be NULL.  Saves
 * the norm launch between the recurrence and the output projection of a decode
 * step.  No reference counterpart (the reference layer norms in its own glue).
 */
int gdn_decode_step_gated(const void* q, const void* k, const void* v,
                          const void* a, const void* b, int gate_dtype,
                          const float* A_log, const float* dt_bias,
                          const float* state_in, float* state_out, float* out,
                          const void* z, const void* norm_gamma, float eps, void* y,
                          int B, int Hqk, int Hv, int dk, int dv, float scale, int flags, void* stream);

/*
 * RMSNorm, bf16 in/out, fp32 math: y = x * rsqrt(mean(x^2) + eps) * gamma.
 * Replaces rmsnorm_forward(), kernels/rmsnorm.cu:280-293 (math: reference/rmsnorm_ref.py:9-28).
 * x, y bf16 [R, D]; gamma bf16 [D].  D % 8 == 0, D <= 8192 (D <= 4096 when x is f32).
 */
int gdn_rmsnorm_fwd(const void* x, const void* gamma, void* y, int R, int D, float eps,
                    void* stream);

/*
 * Gated output RMSNorm: y = RMSNorm(x) * gamma * SiLU(z) (per row of D).
 * No counterpart in the reference (the BASELINE layer's gated norm; the
 * RMSNorm part follows reference/rmsnorm_ref.py:24-28).
 * x [R, D] in x_dtype (bf16 or f32); z bf16 [R, D]; gamma bf16 [D]; y bf16 [R, D].
 * D % 8 == 0, D <= 8192 (D <= 4096 when x is f32).
 */
int gdn_gated_rmsnorm_fwd(const void* x, int x_dtype, const void* z, const void* gamma, void* y,
                          int R, int D, float eps, void* stream);

/*
 * One channel segment of gdn_decode_proj_fwd: output channels c in [0, C) of
 * weight W [C, D] bf16, written to y[b * ldy + c] (bf16).
 *   conv_w         bf16 [C, 4] or NULL.  With it: y = SiLU(conv4(history, x.W[c]))
 *                  with the rounding points of gdn_proj_conv_silu_fwd; without it:
 *                  y = bf16(x . W[c]) (a plain GEMV row, e.g. z, a, b, W_o).
 *   conv_state_in  bf16 [B, C, 3] or NULL (zeros): the last 3 projected values
 *                  per channel, oldest first (what gdn_proj_conv_silu_fwd and the
 *                  prefill leave in conv_state_out).
 *   conv_state_out bf16 [B, C, 3] or NULL; receives (h1, h2, this step's value);
 *                  may be the same buffer as conv_state_in.
 *   l2_group       0, or g >= 8 dividing 128 and C: each g-wide group of y
 *                  is L2-normalised (fp32, eps 1e-6) before the store.
 * C % 16 == 0; W, conv_w and conv_state_in 16-byte aligned.
 */
typedef struct {
    const void* W;
    void* y;
    const void* conv_w;
    const void* conv_state_in;
    void* conv_state_out;
    int C;
    int ldy;
    int l2_group;
} gdn_proj_segment;

/*
 * Input projections of one decode step (one token per sequence) in a single
 * launch: up to 8 segments (e.g. q | k | v with conv + SiLU, q/k L2-normalised
 * per head, then z, a, b as plain rows) over the same x [B, D] bf16, with an
 * optional fused RMSNorm of x (norm_gamma bf16 [D] or NULL, eps).  Replaces the
 * reference's per-step 4-token recompute, gdn_layer.py:58-69
 * (_decode_fused_proj_step), with a 1-token GEMV over the cached conv history.
 * 1 <= B <= 8, D % 256 == 0, and the B token rows must leave room for two weight
 * stages in shared memory: any D <= 5888 at B = 8, D <= 8192 at B <= 4.
 */
int gdn_decode_proj_fwd(const void* x, const void* norm_gamma, float eps, int B, int D,
                        const gdn_proj_segment* segs, int nseg, void* stream);

/*
 * Fused input projection + causal depthwise conv1d (kernel 4) + SiLU.
 * Replaces fused_proj_conv_silu(), kernels/fused_proj_conv_silu.cu:298-355
 * (math: reference/fused_proj_conv_silu_ref.py:33-67).
 *   x bf16 [B, T, D]; W bf16 [Dout, D]; conv_w bf16 [Dout, 4]; y bf16 [B, T, Dout]
 *   conv_state_in  bf16 [B, Dout, 3] or NULL: the 3 projected tokens preceding x
 *                  (oldest first; NULL = zeros, the reference's causal padding)
 *   conv_state_out bf16 [B, Dout, 3] or NULL: receives the last 3 projected tokens
 *   l2norm_group   0, or a head size g (Dout % g == 0): each g-wide group of the
 *                  output is L2-normalised (fp32, eps 1e-6) before the bf16 store.
 * D % 64 == 0, Dout % 128 == 0.
 */
int gdn_proj_conv_silu_fwd(const void* x, const void* W, const void* conv_w, void* y,
                           int B, int T, int D, int Dout,
                           const void* conv_state_in, void* conv_state_out,
                           int l2norm_group, void* stream);

/*
 * gdn_proj_conv_silu_fwd over up to 6 output segments in one launch, all from
 * the same x [B, T, D] bf16: each segment has its own weights W [Dout, D], output
 * y [B, T, Dout] and, optionally, conv weights (NULL: a plain projection
 * y = bf16(x . W^T), no conv or SiLU), conv histories and per-head L2 norm.
 * One persistent launch walks the tiles of all segments, so e.g. a layer's
 * q | k | v projections share one pass over the tiles (no per-call tail) while
 * their outputs stay separate tensors.  Each segment follows the rules of
 * gdn_proj_conv_silu_fwd (Dout % 128 == 0, l2norm_group 0 or a divisor of 128).
 * No reference counterpart (kernels/fused_proj_conv_silu.cu:298-355 is one segment).
 */
typedef struct {
    const void* W;              /* bf16 [Dout, D] */
    void* y;                    /* bf16 [B, T, Dout] */
    const void* conv_w;         /* bf16 [Dout, 4] or NULL (plain projection) */
    const void* conv_state_in;  /* bf16 [B, Dout, 3] or NULL (zeros); conv segments only */
    void* conv_state_out;       /* bf16 [B, Dout, 3] or NULL; conv segments only */
    int Dout;
    int l2norm_group;
} gdn_proj_out_seg;
int gdn_proj_multi_fwd(const void* x, int B, int T, int D, const gdn_proj_out_seg* segs, int nseg,
                       void* stream);

/* Human-readable description of the calling thread's last error. */
const char* gdn_last_error(void);

/*
 * Per calling host thread (default 0): with on != 0 the decode-step kernels
 * (gdn_decode_proj_fwd, gdn_decode_step[_ex], gdn_rmsnorm_fwd,
 * gdn_gated_rmsnorm_fwd) launch with programmatic stream serialisation: each
 * lets the next kernel of the stream launch early and waits for its own
 * predecessors before reading their outputs, and gdn_decode_proj_fwd streams its
 * weights before that wait.  Weight operands must therefore not be written by
 * the kernels just before it on the stream.  Works inside CUDA graph capture.
 * No counterpart in the reference.
 */
int gdn_set_launch_overlap(int on);

/*
 * Multi-GPU entries (one process per GPU of a node; peer buffers are CUDA IPC
 * mappings of the other ranks' device memory).  No counterpart in the
 * reference, which runs on one GPU.
 *
 * gdn_outproj_rs_fwd: the head-sharded output projection fused with its
 * reduce-scatter.  x bf16 [M, K] (this rank's gated-normed head outputs), W
 * bf16 [N, K] (its columns of the projection); the partial product x W^T is
 * written tile by tile into recv[d] + rank * (M / world) * N, the slot of
 * rank d's receive buffer [world][M / world][N] for the rows d owns
 * ([d * M / world, (d + 1) * M / world)).  recv[r] for every rank r, 16-byte
 * aligned.  Needs N % 128 == 0, K % 64 == 0, M % (256 * world) == 0,
 * 1 <= world <= 8.  The caller orders it after the previous reduction on every
 * rank and orders gdn_outproj_reduce after every rank's launch.
 * gdn_outproj_reduce: out bf16 [rows, N] = the sum of the world slots of recv
 * [world][rows][N] (fp32 accumulation).
 */
int gdn_outproj_rs_fwd(const void* x, const void* W, void* const* recv, int M, int N, int K, int rank,
                       int world, void* stream);
int gdn_outproj_reduce(const void* recv, void* out, int rows, int N, int world, void* stream);

/*
 * The all-gather of a head-sharded prefill output, one token window at a time.
 * gathered: this rank's buffer [world][B][H_local][T][dv] (layout BHTD) or
 * [world][B][T][H_local][dv] (BTHD) bf16, whose slot `rank` holds this rank's o;
 * peer_gathered[p]: rank p's gathered buffer mapped into this process (entry
 * `rank` unused).  Copies tokens [t0, t0 + Tw) of slot p from every peer p
 * into slot p of `gathered`, one strided copy-engine transfer per peer on
 * `stream` (no kernel, no SM).  The caller orders it after each peer wrote
 * that window (gdn_prefill_window_ws on the peer) and before any peer rewrites
 * it.  Errors: GDN_ERR_NULL, GDN_ERR_SHAPE (window outside [0, T)),
 * GDN_ERR_DTYPE (layout), GDN_ERR_CUDA.
 */
int gdn_gather_window(void* gathered, const void* const* peer_gathered, int world, int rank, int B, int T,
                      int H_local, int dv, int layout, int t0, int Tw, void* stream);

/* Library version string. */
const char* gdn_version(void);

/*
 * Reads and clears the device-side error word of the current device (set by a
 * kernel that gave up on a bounded wait, or by a varlen prefill that met
 * invalid offsets).  Synchronises the device.  Returns GDN_OK,
 * GDN_ERR_DEVICE_TIMEOUT, GDN_ERR_SHAPE (invalid varlen offsets) or GDN_ERR_CUDA.
 */
int gdn_check_device_error(void);

/*
 * Test hooks of the prefill kernels on the current device, for exercising the
 * bounded waits without faulting the GPU.  No counterpart in the reference.
 *   wait_budget_cycles  > 0: the cycle budget of every bounded wait of the
 *                       prefill kernels (0 restores the default, about 2^31 cycles);
 *   unpublished_record  >= 0: the streamed schedule's prep workers leave the ready
 *                       flag of that chunk record (index b * Hv * nchunks + h *
 *                       nchunks + chunk) unset; -1 publishes every record.
 * With both set, a streamed prefill's chain CTA gives up waiting for that record:
 * every role of the CTA drains (its copies land, its MMAs complete) and returns,
 * gdn_check_device_error() reports GDN_ERR_DEVICE_TIMEOUT, and that call's outputs
 * are undefined.  Reset both (0, -1) before ordinary use.  Synchronous.
 * Errors: GDN_ERR_ARG (negative budget, record below -1), GDN_ERR_CUDA.
 */
int gdn_test_prefill_hooks(long long wait_budget_cycles, long long unpublished_record);

#ifdef __cplusplus
}
#endif
#endif /* GDN_B200_H */
