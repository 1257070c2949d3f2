/*
 * qb_gdn — the Gated DeltaNet recurrence on B200 (sm_100a) behind a C ABI.
 *
 * Drop-in for quotebound's recurrence entry points:
 *   gated_delta(q, k, v, g, beta, state, train)            src/deltanet.h:17-19, src/deltanet.cpp:49-61
 *   gated_delta_trainable(q, k, v, g, beta, state)         src/delta_grad.h:14-16, src/delta_grad.cpp:201-212
 *   gated_delta_vjp({q, k, v, g, beta, state}, dy, dstate) src/delta_grad.h:18-20, src/delta_grad.cpp:155-199
 * plus the per-token path of deltanet(..., rows) (src/deltanet.cpp:102-117, src/exact.cpp:144-159)
 * and the gate / beta / q-k norm graph around the recurrence (src/deltanet.cpp:22-33, 94-100).
 *
 * Conventions (the reference's own C ABI, src/constrain_capi.h:7-9): every call that can fail
 * returns -1 and writes a NUL-terminated reason into err (cut to errlen); nothing throws across
 * the boundary.  0 is success.
 *
 * Memory: every tensor pointer is DEVICE memory owned by the caller, contiguous, row-major in the
 * reference's layouts:
 *   q, k        [B, T, Hk, Dk]         (in_dtype)
 *   v, dy       [B, T, Hv, Dv]         (in_dtype)
 *   y, dv       [B, T, Hv, Dv]         (out_dtype);  dq, dk [B, T, Hk, Dk] (out_dtype)
 *   g, beta     [B, T, Hv]             float32 (and dg, dbeta)
 *   state       [N, Hv, Dv, Dk]        float32 (h0, hT, dh0, dhT); N = B, or the sequence count
 * Value head hv reads key head hv / (Hv / Hk) (src/delta_grad.cpp:35).
 *
 * Streams: `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls are asynchronous
 * on it and never synchronise the device.  Host-side validation runs before any launch, so a call
 * that fails validation has enqueued nothing.
 *
 * Workspace: the recurrence calls take (ws, ws_bytes), 256-byte aligned; query the size with
 * qb_gdn_workspace_bytes.  It opens with the call's status block (qb_gdn_status).  The same workspace
 * must not be used by two calls in flight at once.
 */
#ifndef QB_GDN_H
#define QB_GDN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { QB_DTYPE_F32 = 0, QB_DTYPE_BF16 = 1 };

/* Which calls a workspace / saved-state size is asked for. */
enum { QB_OP_FWD = 0, QB_OP_BWD = 1, QB_OP_LAYER_FWD = 2, QB_OP_LAYER_BWD = 3, QB_OP_BWD_CKPT = 4 };

/* Which kernels run the recurrence.  AUTO takes the tensor-core chunked path where the shape has
 * one (Dk = Dv = 128) and the row-parallel path elsewhere; the other two force one path (CHUNKED
 * fails on a shape it does not cover). */
enum { QB_ALGO_AUTO = 0, QB_ALGO_ROWS = 1, QB_ALGO_CHUNKED = 2 };

/* Shape and dtypes of one recurrence call.
 * Varlen (new in this build; the reference right-pads, src/data.cpp:24-38): with cu_seqlens the
 * batch is B = 1, sequence n covers steps [cu[n], cu[n+1]) of T, its state starts from h0[n] (or
 * zero) and ends in hT[n].  cu_seqlens is the device copy the kernels read; cu_seqlens_host holds
 * the same n_seqs + 1 offsets on the host for validation and grid sizing.  Both NULL: N = B
 * sequences of T steps. */
typedef struct qb_gdn_desc {
  int32_t B, T, Hk, Hv, Dk, Dv;
  int32_t n_seqs;
  const int32_t* cu_seqlens;
  const int32_t* cu_seqlens_host;
  int32_t in_dtype;  /* q, k, v, dy: QB_DTYPE_BF16 or QB_DTYPE_F32 */
  int32_t out_dtype; /* y, dq, dk, dv */
  int32_t algo;      /* QB_ALGO_*; a training forward and its backward must use the same path */
} qb_gdn_desc;

/* Library version string; never fails. */
const char* qb_gdn_version(void);

/* How many kernels this library has launched in this process so far (all devices and streams). */
int64_t qb_gdn_launches(void);

/* Bytes of workspace `op` needs for this shape (at least 256, the status block); -1 on an invalid
 * shape. */
int64_t qb_gdn_workspace_bytes(const qb_gdn_desc* d, int32_t op, char* err, int errlen);

/* Bytes of the saved-for-backward buffer a training forward fills: the chunk-start states (ckpt, see
 * qb_gdn_ckpt_bytes; the counterpart of src/delta_grad.cpp:172-181's ckpt) followed, on the tensor-core
 * path, by data derived from the inputs (gates, operand images, the chunks' delta rows). */
int64_t qb_gdn_saved_bytes(const qb_gdn_desc* d, char* err, int errlen);

/* gated_delta: y and the final state(s).  h0 NULL = zero initial state; hT NULL = not written.
 * saved non-NULL (training forward, gated_delta_trainable) also stores the chunk-start states for
 * qb_gdn_bwd.  Replaces src/deltanet.h:17-19 (gated_delta) and, with saved, src/delta_grad.h:14-16. */
int qb_gdn_fwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* g,
               const float* beta, const float* h0, void* y, float* hT, void* saved, void* ws,
               int64_t ws_bytes, void* stream, char* err, int errlen);

/* gated_delta_vjp: cotangents of (q, k, v, g, beta, h0) given dy and the final-state cotangent dhT
 * (NULL = zero).  saved: the buffer a training qb_gdn_fwd filled with the same inputs, or NULL to
 * recompute it inside (then ws must also cover qb_gdn_saved_bytes).  dh0 NULL = not written.
 * Replaces src/delta_grad.h:18-20 (same argument order q, k, v, g, beta, state). */
int qb_gdn_bwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* g,
               const float* beta, const float* h0, const void* dy, const float* dhT, const void* saved,
               void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0, void* ws,
               int64_t ws_bytes, void* stream, char* err, int errlen);

/* The chunk-start states as a format of their own, for callers that checkpoint activations
 * (src/model.cpp:397-404 wraps every layer in mx::checkpoint) and so keep only what the backward cannot
 * cheaply redo: ckpt [N_chunks, Hv, Dv, Dk] float32, the state at the start of every 64-step chunk,
 * chunks numbered sequence by sequence (fixed-length batches: [B, ceil(T / 64), Hv, Dv, Dk], exactly
 * the reference's ckpt, src/delta_grad.cpp:172-181).  Every saved buffer of a training qb_gdn_fwd
 * begins with it (its first qb_gdn_ckpt_bytes bytes; on the tensor-core path rounded to tf32, which is
 * how its backward reads it); the rest of saved is derived data.
 * qb_gdn_bwd_from_ckpt is gated_delta_vjp (src/delta_grad.cpp:155-199) given those states: the derived
 * data is recomputed chunk by chunk in parallel (no sequential forward), then the backward runs.
 * Workspace: qb_gdn_workspace_bytes(d, QB_OP_BWD_CKPT).  h0 is not read (ckpt[chunk 0] is it). */
int64_t qb_gdn_ckpt_bytes(const qb_gdn_desc* d, char* err, int errlen);
int qb_gdn_bwd_from_ckpt(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* g,
                         const float* beta, const float* h0, const void* dy, const float* dhT, const float* ckpt,
                         void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0, void* ws, int64_t ws_bytes,
                         void* stream, char* err, int errlen);

/* The recurrence with the norm and gate graph around it fused in (deltanet()'s middle,
 * src/deltanet.cpp:94-100, compute_g :22-33): q, k are the raw conv outputs [B, T, Hk, Dk] (bf16),
 * normalised inside as the model does (rms_norm rounded to bf16, times the bf16 scalar 1/Dk for q and
 * 1/sqrt(Dk) for k); a, b [B, T, Hv] float32 give log g = -exp(A_log) softplus(a + dt_bias) and
 * beta = sigmoid(b); A_log, dt_bias [Hv] float32.  Needs the chunked path (bf16, Dk = Dv = 128).
 * saved (training) must hold qb_gdn_layer_saved_bytes(d); the workspace is
 * qb_gdn_workspace_bytes(d, QB_OP_LAYER_FWD / QB_OP_LAYER_BWD).  The backward returns dq, dk for the
 * raw rows, da, db [B, T, Hv], and this call's per-head sums dA_log, ddt_bias [Hv] (fixed-order,
 * overwritten; across GPUs that split the batch, sum them with one all-reduce). */
int64_t qb_gdn_layer_saved_bytes(const qb_gdn_desc* d, char* err, int errlen);
int qb_gdn_layer_fwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* a,
                     const float* b, const float* A_log, const float* dt_bias, const float* h0, void* y,
                     float* hT, void* saved, void* ws, int64_t ws_bytes, void* stream, char* err,
                     int errlen);
int qb_gdn_layer_bwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* a,
                     const float* b, const float* A_log, const float* dt_bias, const float* h0,
                     const void* dy, const float* dhT, const void* saved, void* dq, void* dk, void* dv,
                     float* da, float* db, float* dA_log, float* ddt_bias, float* dh0, void* ws,
                     int64_t ws_bytes, void* stream, char* err, int errlen);

/* One decode step for N independent sequences (gated_delta with T = 1, src/deltanet.cpp:49-61 as
 * the decode path calls it, src/generate.cpp forward(..., cache)):
 *   q, k [N, Hk, Dk]; v [N, Hv, Dv]; g, beta [N, Hv]; state_in [N, Hv, Dv, Dk] float32;
 *   y [N, Hv, Dv] (out_dtype); state_out [N, Hv, Dv, Dk] (may equal state_in). */
int qb_gdn_step(int32_t N, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv, int32_t in_dtype,
                int32_t out_dtype, const void* q, const void* k, const void* v, const float* g,
                const float* beta, const float* state_in, void* y, float* state_out, void* stream,
                char* err, int errlen);

/* Exact speculative verify (deltanet(..., rows), src/deltanet.cpp:102-117; RowStates,
 * src/model.h:84-89): V tokens of each of N sequences run as V one-token steps, bit for bit equal
 * to V calls of qb_gdn_step, and every row's state is kept:
 *   q, k [N, V, Hk, Dk]; v [N, V, Hv, Dv]; g, beta [N, V, Hv]; state_in [N, Hv, Dv, Dk];
 *   y [N, V, Hv, Dv]; states [N, V, Hv, Dv, Dk] (row j = the state after token j). */
int qb_gdn_verify(int32_t N, int32_t V, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv, int32_t in_dtype,
                  int32_t out_dtype, const void* q, const void* k, const void* v, const float* g,
                  const float* beta, const float* state_in, void* y, float* states, void* stream, char* err,
                  int errlen);

/* keep_rows for the recurrence's cache (src/exact.cpp:151-159): state_out[n] = states[n, keep[n]-1].
 * keep: device int32 [N], each in [1, V] (a value outside leaves state_out[n] unchanged and sets
 * status[0] = 1 when status is non-NULL). */
int qb_gdn_keep_rows(int32_t N, int32_t V, int32_t Hv, int32_t Dk, int32_t Dv, const float* states,
                     const int32_t* keep, float* state_out, int32_t* status, void* stream, char* err,
                     int errlen);

/* The gate / beta / q-k norm graph around the recurrence (src/deltanet.cpp:94-100, compute_g
 * :22-33), forward:
 *   qn = q * rsqrt(mean(q^2) + 1e-6) / Dk;  kn = k * rsqrt(mean(k^2) + 1e-6) / sqrt(Dk);
 *   beta = sigmoid(b);  g = exp(-exp(A_log) * softplus(a + dt_bias)).
 * q, k, qn, kn [P, Hk, Dk] (in_dtype for q, k; out_dtype for qn, kn); a, b, g, beta [P, Hv] float32;
 * A_log, dt_bias [Hv] float32.  P = B * T tokens. */
int qb_gdn_gate_fwd(int64_t P, int32_t Hk, int32_t Hv, int32_t Dk, int32_t in_dtype, int32_t out_dtype,
                    const void* q, const void* k, const float* a, const float* b, const float* A_log,
                    const float* dt_bias, void* qn, void* kn, float* g, float* beta, void* stream, char* err,
                    int errlen);

/* Its backward: dq, dk (out_dtype) through the norms from dqn, dkn (in_dtype); da, db [P, Hv]; and
 * this call's per-head sums dA_log, ddt_bias [Hv] (float32, overwritten; a fixed-order reduction,
 * no atomics).  Across GPUs that split the batch, sum dA_log and ddt_bias with one all-reduce. */
int qb_gdn_gate_bwd(int64_t P, int32_t Hk, int32_t Hv, int32_t Dk, int32_t in_dtype, int32_t out_dtype,
                    const void* q, const void* k, const float* a, const float* b, const float* A_log,
                    const float* dt_bias, const void* dqn, const void* dkn, const float* dg,
                    const float* dbeta, void* dq, void* dk, float* da, float* db, float* dA_log,
                    float* ddt_bias, void* ws, int64_t ws_bytes, void* stream, char* err, int errlen);

/* Workspace bytes qb_gdn_gate_bwd needs for P tokens and Hv heads. */
int64_t qb_gdn_gate_workspace_bytes(int64_t P, int32_t Hv);

/* ---- Around the recurrence: the conv before it and the gated norm after it ----------------------
 *
 * The causal depthwise conv1d + SiLU of deltanet() (src/deltanet.cpp:74-93), fused with the q / k / v
 * split.  x [B, T, conv_dim] holds the projected channels q | k | v (conv_dim = 2 Hk Dk + Hv Dv, the
 * reference's in_proj_qkv output); w [conv_dim, K] the per-channel taps (the reference's [conv_dim, K,
 * 1]); the conv state [N, K - 1, conv_dim] the last K - 1 inputs of each sequence (LayerCache.conv,
 * src/model.h:72-76).  Each token's window is its K - 1 predecessors in the same sequence, the carried
 * state before a sequence's start (zeros when state_in is NULL); u = conv rounded to dtype, output
 * silu(u) rounded to dtype, written to q [B, T, Hk, Dk], k [B, T, Hk, Dk], v [B, T, Hv, Dv] -- the raw
 * rows qb_gdn_layer_fwd normalises.  Varlen as in qb_gdn_desc.  Hk Dk and Hv Dv multiples of 8. */
typedef struct qb_gdn_conv_desc {
  int32_t B, T, Hk, Hv, Dk, Dv;
  int32_t K; /* taps: 2, 3 or 4 (Qwen3.5: 4) */
  int32_t n_seqs;
  const int32_t* cu_seqlens;
  const int32_t* cu_seqlens_host;
  int32_t dtype; /* x, w, q, k, v, the states and their cotangents: QB_DTYPE_BF16 or QB_DTYPE_F32 */
} qb_gdn_conv_desc;

/* Workspace bytes of qb_gdn_conv_fwd / qb_gdn_conv_bwd (the backward's figure covers dw). */
int64_t qb_gdn_conv_workspace_bytes(const qb_gdn_conv_desc* d, char* err, int errlen);

/* Forward; state_out (NULL = not written) receives the new conv state (src/deltanet.cpp:75-77). */
int qb_gdn_conv_fwd(const qb_gdn_conv_desc* d, const void* x, const void* w, const void* state_in, void* q, void* k,
                    void* v, void* state_out, void* ws, int64_t ws_bytes, void* stream, char* err, int errlen);

/* Backward: dx [B, T, conv_dim] from the cotangents dq, dk, dv and dstate_out (the new state's; NULL =
 * zero); dw [conv_dim, K] float32 summed over every token in a fixed order (NULL = not computed);
 * dstate_in [N, K - 1, conv_dim] (NULL = not written). */
int qb_gdn_conv_bwd(const qb_gdn_conv_desc* d, const void* x, const void* w, const void* state_in, const void* dq,
                    const void* dk, const void* dv, const void* dstate_out, void* dx, float* dw, void* dstate_in,
                    void* ws, int64_t ws_bytes, void* stream, char* err, int errlen);

/* The conv's part of the exact speculative verify (deltanet(..., rows), src/deltanet.cpp:79-87): B = N
 * sequences of T = V drafted tokens each (x [N, V, conv_dim]) run as V one-token steps of
 * qb_gdn_conv_fwd, bit for bit, every token's conv window kept: states [N, V, K - 1, conv_dim], row j
 * the state after token j (RowStates.conv, src/model.h:84-89).  state_in is required. */
int qb_gdn_conv_verify(const qb_gdn_conv_desc* d, const void* x, const void* w, const void* state_in, void* q, void* k,
                       void* v, void* states, void* stream, char* err, int errlen);

/* keep_rows for the conv state (src/exact.cpp:151-159: cache.conv = rows.conv[n - 1]): state_out[n] =
 * states[n, keep[n] - 1]; keep as in qb_gdn_keep_rows. */
int qb_gdn_keep_conv_rows(int32_t N, int32_t V, int32_t K, int32_t conv_dim, int32_t dtype, const void* states,
                          const int32_t* keep, void* state_out, int32_t* status, void* stream, char* err, int errlen);

/* The gated RMSNorm after the recurrence (src/deltanet.cpp:35-45, :122; Qwen3NextRMSNormGated): per
 * (token, value head) row, n = rms_norm(y, w, eps) rounded to dtype, o = silu(z) n in float32 rounded
 * to dtype.  y, z, o [P, Hv, Dv] (dtype), w [Dv] float32, Dv in {32, 64, 128, 256}; y, z, o (and in the
 * backward dout, dy, dz) aligned to min(16, Dv / 32 x the element size) bytes (each lane moves its part of
 * a row as one vector). */
int qb_gdn_gated_norm_fwd(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const void* y, const void* z,
                          const float* w, void* o, void* stream, char* err, int errlen);
/* Workspace bytes of the backward's dw. */
int64_t qb_gdn_gated_norm_workspace_bytes(int64_t P, int32_t Hv, int32_t Dv);
/* Backward: dy, dz (dtype) and dw [Dv] float32 summed over the rows in a fixed order (NULL = not
 * computed; then ws may be NULL). */
int qb_gdn_gated_norm_bwd(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const void* y, const void* z,
                          const float* w, const void* dout, void* dy, void* dz, float* dw, void* ws, int64_t ws_bytes,
                          void* stream, char* err, int errlen);

/* Device status of the last qb_gdn_fwd / qb_gdn_bwd / qb_gdn_layer_fwd / qb_gdn_layer_bwd call that
 * used this workspace.  Every such workspace opens with a 256-byte status block that the call clears on
 * its stream before its first kernel.  The tensor-core kernels wait on copies and products with
 * bounded waits (about one second of wall time or 2^24 polls); a wait that gives up records its code
 * (the first one of the call wins), lets what it waited for land, frees its tensor memory and returns,
 * so the call never hangs or traps -- but its outputs are then NOT valid.  Calls are asynchronous, so
 * the code is read here: this synchronises `stream` (the stream of that call) and writes the code to
 * *code.  The reference's counterpart is the runtime_error its backward throws
 * (src/delta_grad.cpp:164-170), which has no asynchronous case.  Codes (0 = no failure):
 *    1  prep: the K / Q tiles          2  prep: K K^T, Q K^T
 *   10  forward walk: a chunk's tiles  11, 12, 13  forward walk: its three product rounds
 *   14  forward walk: the last chunk's output product   15  forward walk: a chunk's P image
 *   20  reverse walk: a chunk's images and gates   26  reverse walk: a chunk's P image and rows
 *   21, 22, 23  reverse walk: its three product rounds
 *   30  gradient: the [K; Q] image     31  gradient: a value head's P image and gates
 *   37  gradient: a slice's tiles      34, 35, 36  gradient: its product rounds (slice, K K^T, finalize)
 * The row-parallel kernels have no such waits; their calls always leave 0. */
int qb_gdn_status(const void* ws, int32_t* code, void* stream, char* err, int errlen);

/* Test hook of the failure path above: from now on, in every call of this process, the bounded wait
 * with this code gives up after `polls` polls (code 0 turns the hook off).  The wait then runs out on
 * a normal input, as a lost arrival would make it, and a test can check that the call returns, that
 * qb_gdn_status reports the code and that the next call is correct.  Not for production use.  No
 * counterpart in the reference. */
int qb_gdn_set_wait_limit(int32_t code, int32_t polls, char* err, int errlen);

/* The finite check of the reference's training step (src/train.cpp:266-271 refuses a step whose loss
 * or gradient norm is not finite), as a device count for host code to act on: writes the number of
 * NaN or infinite entries among the n elements of x (QB_DTYPE_F32 or QB_DTYPE_BF16) into the device
 * word *count (cleared first), asynchronously on `stream`. */
int qb_gdn_count_nonfinite(const void* x, int64_t n, int32_t dtype, unsigned long long* count, void* stream,
                           char* err, int errlen);

/* qb_gdn_gate_bwd without a workspace argument, for callers that cannot allocate device memory:
 * code running inside a fixed memory budget or a pre-allocated pool, plugins handed only their input
 * and output buffers, and hosts that forbid cudaMalloc / cudaFree on the hot path because those calls
 * synchronise the device.  It allocates nothing: its partial sums go to a fixed array of 148 x 256 x 2
 * floats (296 KiB) in the library's own device memory, which every GPU that loads the library holds
 * until the process exits.  Value heads beyond 256 are refused with an error.  The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress, with that device current), and
 * so does the first call in a new context of the device (after cudaDeviceReset, say, the old address
 * is gone); make that first call before any stream capture.  All calls share the one array, so two calls that
 * overlap on the GPU (other streams, other threads) race on it and must be ordered by the caller;
 * nothing in it needs clearing between calls.  Arguments and results are those of qb_gdn_gate_bwd.
 * This entry point has no counterpart in the reference. */
int qb_gdn_gate_bwd_noalloc(int64_t P, int32_t Hk, int32_t Hv, int32_t Dk, int32_t in_dtype, int32_t out_dtype,
                            const void* q, const void* k, const float* a, const float* b, const float* A_log,
                            const float* dt_bias, const void* dqn, const void* dkn, const float* dg,
                            const float* dbeta, void* dq, void* dk, float* da, float* db, float* dA_log,
                            float* ddt_bias, void* stream, char* err, int errlen);

#ifdef __cplusplus
}
#endif

#endif /* QB_GDN_H */
