// The C ABI of include/qb_gdn.h: host-side validation, workspace carving and kernel dispatch.
// Error convention of the reference's C ABI (src/constrain_capi.h:7-9): -1 and a NUL-terminated
// reason in err; nothing throws across the boundary.  Validation mirrors the spirit of
// src/delta_grad.cpp:164-170 (name the offending shapes).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include "../../include/qb_gdn.h"
#include "gdn_cc.cuh"
#include "gdn_chunk.cuh"
#include "gdn_common.cuh"
#include "gdn_gate.cuh"
#include "gdn_simt.cuh"
#include "launch_count.cuh"
#include "status.cuh"

using namespace qbgdn;

namespace qbgdn {
static std::atomic<int64_t> g_launches{0};
void note_launch(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
int64_t launches() { return g_launches.load(std::memory_order_relaxed); }

// ---- the status block (status.cuh) ----
static std::atomic<int> g_test_code{0};
static std::atomic<uint32_t> g_test_polls{0};
void set_test_wait_limit(int code, uint32_t polls) {
  g_test_polls.store(polls);
  g_test_code.store(code);
}

__global__ void status_init_kernel(int* status, int code, uint32_t polls) {
  const int i = threadIdx.x;
  if (i < kStatusBytes / 4) status[i] = i == 4 ? code : i == 5 ? (int)polls : 0;
}

cudaError_t init_status(int* status, cudaStream_t st) {
  const int code = g_test_code.load();
  if (code == 0) return cudaMemsetAsync(status, 0, kStatusBytes, st);
  status_init_kernel<<<1, kStatusBytes / 4, 0, st>>>(status, code, g_test_polls.load());
  note_launch();
  return cudaGetLastError();
}

// Counts the entries of x that are NaN or infinite into *count (one atomic add per block).
template <typename T>
__global__ void count_nonfinite_kernel(const T* __restrict__ x, int64_t n, unsigned long long* count) {
  unsigned c = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    c += isfinite(to_f(x[i])) ? 0u : 1u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  __shared__ unsigned part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    if (t) atomicAdd(count, t);
  }
}
}  // namespace qbgdn

namespace {

constexpr int kChunkSteps = 64;

int fail(char* err, int errlen, const char* fmt, ...) {
  if (err && errlen > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
    err[errlen - 1] = '\0';
  }
  return -1;
}

int cuda_fail(cudaError_t e, const char* what, char* err, int errlen) {
  return fail(err, errlen, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }
bool dtype_ok(int32_t d) { return d == QB_DTYPE_F32 || d == QB_DTYPE_BF16; }

struct Plan {
  int N;                // sequences
  int64_t tokens;       // B * T
  int64_t n_chunks;     // sum over sequences of ceil(len / 64)
  bool varlen;
  bool chunked;         // tensor-core chunked path
  int rpb;              // rows per block (row-parallel forward)
};

int check_desc(const qb_gdn_desc* d, Plan* p, char* err, int errlen) {
  if (!d) return fail(err, errlen, "gated delta: null descriptor");
  if (d->B < 1 || d->T < 0 || d->Hk < 1 || d->Hv < 1 || d->Dk < 1 || d->Dv < 1)
    return fail(err, errlen, "gated delta: bad shape (B %d, T %d, Hk %d, Hv %d, Dk %d, Dv %d)", d->B, d->T, d->Hk,
                d->Hv, d->Dk, d->Dv);
  if (d->Dk != 32 && d->Dk != 64 && d->Dk != 128 && d->Dk != 256)
    return fail(err, errlen, "gated delta: needs Dk in {32, 64, 128, 256} (Dk %d, Dv %d, Hk %d, Hv %d)", d->Dk, d->Dv,
                d->Hk, d->Hv);
  if (d->Hv % d->Hk)
    return fail(err, errlen, "gated delta: value heads must be a multiple of key heads (Hk %d, Hv %d)", d->Hk,
                d->Hv);
  if (!dtype_ok(d->in_dtype) || !dtype_ok(d->out_dtype))
    return fail(err, errlen, "gated delta: dtypes must be QB_DTYPE_F32 or QB_DTYPE_BF16 (in %d, out %d)",
                d->in_dtype, d->out_dtype);
  if (d->algo < QB_ALGO_AUTO || d->algo > QB_ALGO_CHUNKED)
    return fail(err, errlen, "gated delta: unknown algo %d", d->algo);
  p->varlen = d->cu_seqlens || d->cu_seqlens_host;
  p->tokens = (int64_t)d->B * d->T;
  if (p->varlen) {
    if (!d->cu_seqlens || !d->cu_seqlens_host)
      return fail(err, errlen, "gated delta: varlen needs both cu_seqlens (device) and cu_seqlens_host");
    if (d->B != 1) return fail(err, errlen, "gated delta: varlen needs B == 1 (B %d)", d->B);
    if (d->n_seqs < 1) return fail(err, errlen, "gated delta: varlen needs n_seqs >= 1 (n_seqs %d)", d->n_seqs);
    const int32_t* cu = d->cu_seqlens_host;
    if (cu[0] != 0) return fail(err, errlen, "gated delta: cu_seqlens[0] must be 0 (got %d)", cu[0]);
    int64_t nc = 0;
    for (int n = 0; n < d->n_seqs; ++n) {
      if (cu[n + 1] < cu[n])
        return fail(err, errlen, "gated delta: cu_seqlens must be non-decreasing (cu[%d] = %d > cu[%d] = %d)", n,
                    cu[n], n + 1, cu[n + 1]);
      nc += (cu[n + 1] - cu[n] + kChunkSteps - 1) / kChunkSteps;
    }
    if (cu[d->n_seqs] != d->T)
      return fail(err, errlen, "gated delta: cu_seqlens[%d] = %d must equal T = %d", d->n_seqs, cu[d->n_seqs], d->T);
    p->N = d->n_seqs;
    p->n_chunks = nc;
  } else {
    p->N = d->B;
    p->n_chunks = (int64_t)d->B * ((d->T + kChunkSteps - 1) / kChunkSteps);
  }
  const bool chunk_ok = chunked_supported(d->Dk, d->Dv) && d->in_dtype == QB_DTYPE_BF16;
  if (d->algo == QB_ALGO_CHUNKED && !chunk_ok)
    return fail(err, errlen, "gated delta: the chunked path needs Dk = Dv = 128 and bf16 activations (Dk %d, Dv %d)",
                d->Dk, d->Dv);
  p->chunked = d->algo == QB_ALGO_CHUNKED || (d->algo == QB_ALGO_AUTO && chunk_ok);
  p->rpb = simt_rows_per_block(d->Dv);
  return 0;
}

int64_t saved_bytes_of(const qb_gdn_desc* d, const Plan& p) {
  if (p.chunked) return chunked_saved_bytes(d->Hv, d->Hk, p.n_chunks, p.tokens, false);
  return p.n_chunks * d->Hv * (int64_t)d->Dv * d->Dk * 4;
}

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Workspace of the row-parallel forward and the CUDA-core backward: [status block] [chunk_off (varlen)]
// [the backward's chunk intermediates (gdn_cc.cuh)] [saved (recompute)]
struct SimtWs {
  int* status;
  int64_t* chunk_off;
  char* cc;
  float* saved;
};

int64_t simt_ws_bytes(const qb_gdn_desc* d, const Plan& p, int op, bool with_saved, SimtWs* out, char* base) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* at = base ? base + off : nullptr;
    off += align256(bytes);
    return at;
  };
  SimtWs w{};
  w.status = (int*)take(kStatusBytes);
  w.chunk_off = (int64_t*)take(p.varlen ? (p.N + 1) * 8 : 0);
  if (op == QB_OP_BWD) {
    w.cc = take(cc_ws_layout(d->Hk, d->Hv, d->Dk, d->Dv, p.n_chunks, nullptr, nullptr));
    if (with_saved) w.saved = (float*)take(saved_bytes_of(d, p));
  }
  if (out) *out = w;
  return off;
}

// The backward of a chunked forward runs the row-parallel kernels until the chunked ones exist.
bool chunked_bwd_of(const Plan& p) { return p.chunked && chunked_bwd_ready(); }

int64_t ws_bytes_of(const qb_gdn_desc* d, const Plan& p, int op, bool with_saved) {
  if (op == QB_OP_FWD ? p.chunked : chunked_bwd_of(p))
    return chunked_ws_bytes(d->Hv, d->Hk, p.N, p.n_chunks, p.tokens, p.varlen, op, with_saved, false);
  return simt_ws_bytes(d, p, op, with_saved, nullptr, nullptr);
}

}  // namespace

extern "C" {

const char* qb_gdn_version(void) { return "qb_gdn 0.1 (sm_100a)"; }

int64_t qb_gdn_launches(void) { return launches(); }

static int check_layer(const qb_gdn_desc* d, Plan* p, char* err, int errlen) {
  if (check_desc(d, p, err, errlen)) return -1;
  if (!p->chunked)
    return fail(err, errlen,
                "gated delta layer: the fused norm/gate path runs on the chunked kernels: needs Dk = Dv = 128, bf16 "
                "activations and algo AUTO or CHUNKED (Dk %d, Dv %d, in_dtype %d, algo %d)",
                d->Dk, d->Dv, d->in_dtype, d->algo);
  if (d->Hv > 4096) return fail(err, errlen, "gated delta layer: too many value heads (%d)", d->Hv);
  return 0;
}

int64_t qb_gdn_workspace_bytes(const qb_gdn_desc* d, int32_t op, char* err, int errlen) {
  Plan p;
  if (op == QB_OP_LAYER_FWD || op == QB_OP_LAYER_BWD) {
    if (check_layer(d, &p, err, errlen)) return -1;
    return chunked_ws_bytes(d->Hv, d->Hk, p.N, p.n_chunks, p.tokens, p.varlen, op == QB_OP_LAYER_FWD ? 0 : 1,
                            op == QB_OP_LAYER_BWD, true);
  }
  if (check_desc(d, &p, err, errlen)) return -1;
  if (op == QB_OP_BWD_CKPT) {
    if (chunked_bwd_of(p))
      return chunked_ws_bytes(d->Hv, d->Hk, p.N, p.n_chunks, p.tokens, p.varlen, QB_OP_BWD, true, false, true);
    return simt_ws_bytes(d, p, QB_OP_BWD, false, nullptr, nullptr);
  }
  if (op != QB_OP_FWD && op != QB_OP_BWD) return fail(err, errlen, "gated delta: unknown op %d", op);
  // the backward's figure covers recomputing the saved states (saved == NULL)
  return ws_bytes_of(d, p, op, op == QB_OP_BWD);
}

int64_t qb_gdn_layer_saved_bytes(const qb_gdn_desc* d, char* err, int errlen) {
  Plan p;
  if (check_layer(d, &p, err, errlen)) return -1;
  return chunked_saved_bytes(d->Hv, d->Hk, p.n_chunks, p.tokens, true);
}

int qb_gdn_layer_fwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* a, const float* b,
                     const float* A_log, const float* dt_bias, const float* h0, void* y, float* hT, void* saved,
                     void* ws, int64_t ws_bytes, void* stream, char* err, int errlen) {
  Plan p;
  if (check_layer(d, &p, err, errlen)) return -1;
  if (!q || !k || !v || !a || !b || !A_log || !dt_bias || !y)
    return fail(err, errlen, "gated delta layer forward: q, k, v, a, b, A_log, dt_bias and y must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(y, 16) || (h0 && !aligned(h0, 16)) ||
      (hT && !aligned(hT, 16)) || (saved && !aligned(saved, 256)))
    return fail(err, errlen, "gated delta layer forward: q, k, v, y, h0, hT need 16-byte alignment and saved 256-byte");
  const int64_t need = chunked_ws_bytes(d->Hv, d->Hk, p.N, p.n_chunks, p.tokens, p.varlen, 0, false, true);
  if (!ws || ws_bytes < need || !aligned(ws, 256))
    return fail(err, errlen, "gated delta layer forward: a 256-byte aligned workspace of %lld bytes is needed (got %lld)",
                (long long)need, (long long)ws_bytes);
  cudaError_t e = init_status((int*)ws, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "gated delta layer forward", err, errlen);
  if (p.tokens == 0) return 0;
  ChunkFwdArgs f{};
  f.B = d->B, f.T = d->T, f.Hk = d->Hk, f.Hv = d->Hv, f.Dk = d->Dk, f.Dv = d->Dv, f.N = p.N, f.n_chunks = p.n_chunks;
  f.cu = d->cu_seqlens, f.q = q, f.k = k, f.v = v, f.h0 = h0, f.y = y, f.hT = hT, f.saved = saved;
  f.in_bf16 = 1, f.out_bf16 = d->out_dtype == QB_DTYPE_BF16;
  f.a_raw = a, f.b_raw = b, f.A_log = A_log, f.dt_bias = dt_bias;
  e = chunked_fwd(f, ws, (cudaStream_t)stream, (int*)ws);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta layer forward", err, errlen);
}

int qb_gdn_layer_bwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* a, const float* b,
                     const float* A_log, const float* dt_bias, const float* h0, const void* dy, const float* dhT,
                     const void* saved, void* dq, void* dk, void* dv, float* da, float* db, float* dA_log,
                     float* ddt_bias, float* dh0, void* ws, int64_t ws_bytes, void* stream, char* err, int errlen) {
  Plan p;
  if (check_layer(d, &p, err, errlen)) return -1;
  if (!q || !k || !v || !a || !b || !A_log || !dt_bias || !dy || !dq || !dk || !dv || !da || !db || !dA_log ||
      !ddt_bias)
    return fail(err, errlen, "gated delta layer backward: inputs and every gradient except dh0 must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(dy, 16) || !aligned(dq, 16) ||
      !aligned(dk, 16) || !aligned(dv, 16) || (h0 && !aligned(h0, 16)) || (dhT && !aligned(dhT, 16)) ||
      (dh0 && !aligned(dh0, 16)) || (saved && !aligned(saved, 256)))
    return fail(err, errlen, "gated delta layer backward: tensors need 16-byte alignment and saved 256-byte");
  const int64_t need = chunked_ws_bytes(d->Hv, d->Hk, p.N, p.n_chunks, p.tokens, p.varlen, 1, saved == nullptr, true);
  if (!ws || ws_bytes < need || !aligned(ws, 256))
    return fail(err, errlen, "gated delta layer backward: a 256-byte aligned workspace of %lld bytes is needed (got %lld)",
                (long long)need, (long long)ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaError_t e = init_status((int*)ws, st)) return cuda_fail(e, "gated delta layer backward", err, errlen);
  if (p.tokens == 0) {
    cudaError_t e = cudaMemsetAsync(dA_log, 0, d->Hv * 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ddt_bias, 0, d->Hv * 4, st);
    if (e == cudaSuccess && dh0)
      e = dhT ? cudaMemcpyAsync(dh0, dhT, (size_t)p.N * d->Hv * d->Dv * d->Dk * 4, cudaMemcpyDeviceToDevice, st)
              : cudaMemsetAsync(dh0, 0, (size_t)p.N * d->Hv * d->Dv * d->Dk * 4, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta layer backward", err, errlen);
  }
  ChunkBwdArgs x{};
  x.B = d->B, x.T = d->T, x.Hk = d->Hk, x.Hv = d->Hv, x.Dk = d->Dk, x.Dv = d->Dv, x.N = p.N, x.n_chunks = p.n_chunks;
  x.cu = d->cu_seqlens, x.q = q, x.k = k, x.v = v, x.dy = dy, x.h0 = h0, x.dhT = dhT, x.saved = saved;
  x.dq = dq, x.dk = dk, x.dv = dv, x.dg = da, x.dbeta = db, x.dh0 = dh0;
  x.in_bf16 = 1, x.out_bf16 = d->out_dtype == QB_DTYPE_BF16;
  x.a_raw = a, x.b_raw = b, x.A_log = A_log, x.dt_bias = dt_bias, x.dA_log = dA_log, x.ddt_bias = ddt_bias;
  cudaError_t e = chunked_bwd(x, ws, st);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta layer backward", err, errlen);
}

int64_t qb_gdn_saved_bytes(const qb_gdn_desc* d, char* err, int errlen) {
  Plan p;
  if (check_desc(d, &p, err, errlen)) return -1;
  return saved_bytes_of(d, p);
}

int qb_gdn_fwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* g, const float* beta,
               const float* h0, void* y, float* hT, void* saved, void* ws, int64_t ws_bytes, void* stream, char* err,
               int errlen) {
  Plan p;
  if (check_desc(d, &p, err, errlen)) return -1;
  if (!q || !k || !v || !g || !beta || !y)
    return fail(err, errlen, "gated delta forward: q, k, v, g, beta and y must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(y, 16) || (h0 && !aligned(h0, 16)) ||
      (hT && !aligned(hT, 16)) || (saved && !aligned(saved, 256)))
    return fail(err, errlen, "gated delta forward: q, k, v, y, h0, hT need 16-byte alignment and saved 256-byte");
  const int64_t need = ws_bytes_of(d, p, QB_OP_FWD, false);
  if (!ws || ws_bytes < need)
    return fail(err, errlen, "gated delta forward: workspace of %lld bytes needed (got %lld)", (long long)need,
                (long long)ws_bytes);
  if (!aligned(ws, 256)) return fail(err, errlen, "gated delta forward: workspace needs 256-byte alignment");
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaError_t e = init_status((int*)ws, st)) return cuda_fail(e, "gated delta forward", err, errlen);
  if (p.tokens == 0) return 0;
  if (p.chunked) {
    ChunkFwdArgs a{};
    a.B = d->B, a.T = d->T, a.Hk = d->Hk, a.Hv = d->Hv, a.Dk = d->Dk, a.Dv = d->Dv, a.N = p.N;
    a.n_chunks = p.n_chunks;
    a.cu = d->cu_seqlens;
    a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = h0, a.y = y, a.hT = hT;
    a.saved = saved;
    a.in_bf16 = d->in_dtype == QB_DTYPE_BF16, a.out_bf16 = d->out_dtype == QB_DTYPE_BF16;
    cudaError_t e = chunked_fwd(a, ws, st, (int*)ws);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta forward (chunked)", err, errlen);
  }
  SimtWs w;
  simt_ws_bytes(d, p, QB_OP_FWD, false, &w, (char*)ws);
  cudaError_t e;
  if (p.varlen && saved) {
    if ((e = launch_chunk_offsets(d->cu_seqlens, p.N, w.chunk_off, st)) != cudaSuccess)
      return cuda_fail(e, "gated delta forward", err, errlen);
  }
  SimtArgs a{};
  a.T = d->T, a.Hk = d->Hk, a.Hv = d->Hv, a.Dk = d->Dk, a.Dv = d->Dv, a.rows_per_block = p.rpb;
  a.cu = d->cu_seqlens;
  a.chunk_off = p.varlen ? w.chunk_off : nullptr;
  a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = h0, a.y = y, a.hT = hT;
  a.ckpt = (float*)saved;
  e = simt_launch(SimtKind::Fwd, a, p.N, d->in_dtype == QB_DTYPE_BF16, d->out_dtype == QB_DTYPE_BF16, st);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta forward", err, errlen);
}

int qb_gdn_bwd(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* g, const float* beta,
               const float* h0, const void* dy, const float* dhT, const void* saved, void* dq, void* dk, void* dv,
               float* dg, float* dbeta, float* dh0, void* ws, int64_t ws_bytes, void* stream, char* err,
               int errlen) {
  Plan p;
  if (check_desc(d, &p, err, errlen)) return -1;
  if (!q || !k || !v || !g || !beta || !dy || !dq || !dk || !dv || !dg || !dbeta)
    return fail(err, errlen, "gated delta backward: q, k, v, g, beta, dy, dq, dk, dv, dg, dbeta must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(dy, 16) || !aligned(dq, 16) ||
      !aligned(dk, 16) || !aligned(dv, 16) || (h0 && !aligned(h0, 16)) || (dhT && !aligned(dhT, 16)) ||
      (dh0 && !aligned(dh0, 16)) || (saved && !aligned(saved, 256)))
    return fail(err, errlen, "gated delta backward: tensors need 16-byte alignment and saved 256-byte");
  const int64_t need = ws_bytes_of(d, p, QB_OP_BWD, saved == nullptr);
  if (!ws || ws_bytes < need)
    return fail(err, errlen, "gated delta backward: workspace of %lld bytes needed (got %lld)", (long long)need,
                (long long)ws_bytes);
  if (!aligned(ws, 256)) return fail(err, errlen, "gated delta backward: workspace needs 256-byte alignment");
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaError_t e = init_status((int*)ws, st)) return cuda_fail(e, "gated delta backward", err, errlen);
  if (p.tokens == 0) {
    if (dh0 && dhT) {
      cudaError_t e = cudaMemcpyAsync(dh0, dhT, (size_t)p.N * d->Hv * d->Dv * d->Dk * 4, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return cuda_fail(e, "gated delta backward", err, errlen);
    } else if (dh0) {
      cudaError_t e = cudaMemsetAsync(dh0, 0, (size_t)p.N * d->Hv * d->Dv * d->Dk * 4, st);
      if (e != cudaSuccess) return cuda_fail(e, "gated delta backward", err, errlen);
    }
    return 0;
  }
  if (chunked_bwd_of(p)) {
    ChunkBwdArgs a{};
    a.B = d->B, a.T = d->T, a.Hk = d->Hk, a.Hv = d->Hv, a.Dk = d->Dk, a.Dv = d->Dv, a.N = p.N;
    a.n_chunks = p.n_chunks;
    a.cu = d->cu_seqlens;
    a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = h0, a.dy = dy, a.dhT = dhT;
    a.saved = saved;
    a.dq = dq, a.dk = dk, a.dv = dv, a.dg = dg, a.dbeta = dbeta, a.dh0 = dh0;
    a.in_bf16 = d->in_dtype == QB_DTYPE_BF16, a.out_bf16 = d->out_dtype == QB_DTYPE_BF16;
    cudaError_t e = chunked_bwd(a, ws, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta backward (chunked)", err, errlen);
  }
  SimtWs w;
  simt_ws_bytes(d, p, QB_OP_BWD, saved == nullptr, &w, (char*)ws);
  const int in_bf16 = d->in_dtype == QB_DTYPE_BF16, out_bf16 = d->out_dtype == QB_DTYPE_BF16;
  cudaError_t e;
  if (p.varlen && (e = launch_chunk_offsets(d->cu_seqlens, p.N, w.chunk_off, st)) != cudaSuccess)
    return cuda_fail(e, "gated delta backward", err, errlen);
  SimtArgs a{};
  a.T = d->T, a.Hk = d->Hk, a.Hv = d->Hv, a.Dk = d->Dk, a.Dv = d->Dv, a.rows_per_block = p.rpb;
  a.cu = d->cu_seqlens;
  a.chunk_off = p.varlen ? w.chunk_off : nullptr;
  a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = h0;
  float* ck = (float*)saved;
  if (!ck) {  // recompute the chunk starts with the same forward, y discarded into the dv buffer
    ck = w.saved;
    SimtArgs f = a;
    f.y = dv;  // same shape and dtype as y; overwritten by the backward below
    f.ckpt = ck;
    if ((e = simt_launch(SimtKind::Fwd, f, p.N, in_bf16, out_bf16, st)) != cudaSuccess)
      return cuda_fail(e, "gated delta backward (recompute)", err, errlen);
  }
  CcArgs c{};
  cc_ws_layout(d->Hk, d->Hv, d->Dk, d->Dv, p.n_chunks, w.cc, &c);
  c.geo = Geo{d->T, d->Hk, d->Hv, p.N, (d->T + kChunkSteps - 1) / kChunkSteps, d->cu_seqlens,
              p.varlen ? w.chunk_off : nullptr};
  c.n_chunks = p.n_chunks, c.Dk = d->Dk, c.Dv = d->Dv;
  c.q = q, c.k = k, c.v = v, c.dy = dy, c.g = g, c.beta = beta, c.ckpt = ck, c.dhT = dhT;
  c.dq = dq, c.dk = dk, c.dv = dv, c.dg = dg, c.dbeta = dbeta, c.dh0 = dh0;
  if ((e = cc_bwd(c, p.N, in_bf16, out_bf16, st)) != cudaSuccess) return cuda_fail(e, "gated delta backward", err, errlen);
  return 0;
}

int64_t qb_gdn_ckpt_bytes(const qb_gdn_desc* d, char* err, int errlen) {
  Plan p;
  if (check_desc(d, &p, err, errlen)) return -1;
  return p.n_chunks * d->Hv * (int64_t)d->Dv * d->Dk * 4;
}

int qb_gdn_bwd_from_ckpt(const qb_gdn_desc* d, const void* q, const void* k, const void* v, const float* g,
                         const float* beta, const float* h0, const void* dy, const float* dhT, const float* ckpt,
                         void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0, void* ws, int64_t ws_bytes,
                         void* stream, char* err, int errlen) {
  Plan p;
  if (check_desc(d, &p, err, errlen)) return -1;
  if (!q || !k || !v || !g || !beta || !dy || !ckpt || !dq || !dk || !dv || !dg || !dbeta)
    return fail(err, errlen, "gated delta backward from ckpt: inputs, ckpt and every gradient but dh0 must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(dy, 16) || !aligned(dq, 16) ||
      !aligned(dk, 16) || !aligned(dv, 16) || !aligned(ckpt, 16) || (dhT && !aligned(dhT, 16)) ||
      (dh0 && !aligned(dh0, 16)))
    return fail(err, errlen, "gated delta backward from ckpt: tensors need 16-byte alignment");
  const bool chunked = chunked_bwd_of(p);
  if (chunked && p.n_chunks > 65535)
    return fail(err, errlen, "gated delta backward from ckpt: at most 65535 chunks per call (got %lld)",
                (long long)p.n_chunks);
  const int64_t need = chunked ? chunked_ws_bytes(d->Hv, d->Hk, p.N, p.n_chunks, p.tokens, p.varlen, QB_OP_BWD, true,
                                                  false, true)
                               : simt_ws_bytes(d, p, QB_OP_BWD, false, nullptr, nullptr);
  if (!ws || ws_bytes < need || !aligned(ws, 256))
    return fail(err, errlen, "gated delta backward from ckpt: a 256-byte aligned workspace of %lld bytes is needed "
                "(got %lld)", (long long)need, (long long)ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaError_t e = init_status((int*)ws, st)) return cuda_fail(e, "gated delta backward from ckpt", err, errlen);
  if (p.tokens == 0) {
    if (!dh0) return 0;
    const size_t bytes = (size_t)p.N * d->Hv * d->Dv * d->Dk * 4;
    cudaError_t e = dhT ? cudaMemcpyAsync(dh0, dhT, bytes, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(dh0, 0, bytes, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta backward from ckpt", err, errlen);
  }
  const int in_bf16 = d->in_dtype == QB_DTYPE_BF16, out_bf16 = d->out_dtype == QB_DTYPE_BF16;
  cudaError_t e;
  if (chunked) {
    ChunkBwdArgs a{};
    a.B = d->B, a.T = d->T, a.Hk = d->Hk, a.Hv = d->Hv, a.Dk = d->Dk, a.Dv = d->Dv, a.N = p.N;
    a.n_chunks = p.n_chunks;
    a.cu = d->cu_seqlens;
    a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = h0, a.dy = dy, a.dhT = dhT, a.saved = nullptr;
    a.dq = dq, a.dk = dk, a.dv = dv, a.dg = dg, a.dbeta = dbeta, a.dh0 = dh0;
    a.in_bf16 = in_bf16, a.out_bf16 = out_bf16;
    a.ckpt_in = ckpt;
    e = chunked_bwd(a, ws, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta backward from ckpt (chunked)", err, errlen);
  }
  SimtWs w;
  simt_ws_bytes(d, p, QB_OP_BWD, false, &w, (char*)ws);
  if (p.varlen && (e = launch_chunk_offsets(d->cu_seqlens, p.N, w.chunk_off, st)) != cudaSuccess)
    return cuda_fail(e, "gated delta backward from ckpt", err, errlen);
  CcArgs c{};
  cc_ws_layout(d->Hk, d->Hv, d->Dk, d->Dv, p.n_chunks, w.cc, &c);
  c.geo = Geo{d->T, d->Hk, d->Hv, p.N, (d->T + kChunkSteps - 1) / kChunkSteps, d->cu_seqlens,
              p.varlen ? w.chunk_off : nullptr};
  c.n_chunks = p.n_chunks, c.Dk = d->Dk, c.Dv = d->Dv;
  c.q = q, c.k = k, c.v = v, c.dy = dy, c.g = g, c.beta = beta, c.ckpt = ckpt, c.dhT = dhT;
  c.dq = dq, c.dk = dk, c.dv = dv, c.dg = dg, c.dbeta = dbeta, c.dh0 = dh0;
  e = cc_bwd(c, p.N, in_bf16, out_bf16, st);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta backward from ckpt", err, errlen);
}

int qb_gdn_status(const void* ws, int32_t* code, void* stream, char* err, int errlen) {
  if (!ws || !code) return fail(err, errlen, "gated delta status: ws and code must be non-null");
  if (!aligned(ws, 256)) return fail(err, errlen, "gated delta status: ws is not a workspace (256-byte alignment)");
  cudaStream_t st = (cudaStream_t)stream;
  int32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, ws, sizeof v, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "gated delta status", err, errlen);
  *code = v;
  return 0;
}

int qb_gdn_set_wait_limit(int32_t code, int32_t polls, char* err, int errlen) {
  if (code < 0 || polls < 1) return fail(err, errlen, "gated delta wait limit: code %d >= 0 and polls %d >= 1", code, polls);
  set_test_wait_limit(code, (uint32_t)polls);
  return 0;
}

int qb_gdn_count_nonfinite(const void* x, int64_t n, int32_t dtype, unsigned long long* count, void* stream, char* err,
                           int errlen) {
  if (n < 0 || !dtype_ok(dtype)) return fail(err, errlen, "gated delta finite check: bad arguments (n %lld, dtype %d)",
                                             (long long)n, dtype);
  if (!count || (n > 0 && !x)) return fail(err, errlen, "gated delta finite check: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(count, 0, sizeof *count, st);
  if (e == cudaSuccess && n > 0) {
    const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8);
    if (dtype == QB_DTYPE_BF16)
      count_nonfinite_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, count);
    else
      count_nonfinite_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(x), n, count);
    note_launch();
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta finite check", err, errlen);
}

static int check_rows(int32_t N, int32_t V, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv, int32_t in_dtype,
                      int32_t out_dtype, const char* what, char* err, int errlen) {
  if (N < 0 || V < 1 || Hk < 1 || Hv < 1 || Dv < 1)
    return fail(err, errlen, "%s: bad shape (N %d, V %d, Hk %d, Hv %d, Dk %d, Dv %d)", what, N, V, Hk, Hv, Dk, Dv);
  if (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256)
    return fail(err, errlen, "%s: needs Dk in {32, 64, 128, 256} (Dk %d)", what, Dk);
  if (Hv % Hk) return fail(err, errlen, "%s: value heads must be a multiple of key heads (Hk %d, Hv %d)", what, Hk, Hv);
  if (!dtype_ok(in_dtype) || !dtype_ok(out_dtype))
    return fail(err, errlen, "%s: dtypes must be QB_DTYPE_F32 or QB_DTYPE_BF16 (in %d, out %d)", what, in_dtype,
                out_dtype);
  return 0;
}

int qb_gdn_step(int32_t N, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv, int32_t in_dtype, int32_t out_dtype,
                const void* q, const void* k, const void* v, const float* g, const float* beta, const float* state_in,
                void* y, float* state_out, void* stream, char* err, int errlen) {
  if (check_rows(N, 1, Hk, Hv, Dk, Dv, in_dtype, out_dtype, "gated delta step", err, errlen)) return -1;
  if (!q || !k || !v || !g || !beta || !state_in || !y || !state_out)
    return fail(err, errlen, "gated delta step: every pointer must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(state_in, 16) || !aligned(state_out, 16))
    return fail(err, errlen, "gated delta step: q, k and the states need 16-byte alignment");
  if (N == 0) return 0;
  SimtArgs a{};
  a.T = 1, a.Hk = Hk, a.Hv = Hv, a.Dk = Dk, a.Dv = Dv, a.rows_per_block = simt_rows_per_block(Dv);
  a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = state_in, a.y = y, a.hT = state_out;
  cudaError_t e = simt_launch(SimtKind::Step, a, N, in_dtype == QB_DTYPE_BF16, out_dtype == QB_DTYPE_BF16,
                              (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta step", err, errlen);
}

int qb_gdn_verify(int32_t N, int32_t V, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv, int32_t in_dtype,
                  int32_t out_dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                  const float* state_in, void* y, float* states, void* stream, char* err, int errlen) {
  if (check_rows(N, V, Hk, Hv, Dk, Dv, in_dtype, out_dtype, "gated delta verify", err, errlen)) return -1;
  if (!q || !k || !v || !g || !beta || !state_in || !y || !states)
    return fail(err, errlen, "gated delta verify: every pointer must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(state_in, 16) || !aligned(states, 16))
    return fail(err, errlen, "gated delta verify: q, k and the states need 16-byte alignment");
  if (N == 0) return 0;
  SimtArgs a{};
  a.T = V, a.Hk = Hk, a.Hv = Hv, a.Dk = Dk, a.Dv = Dv, a.rows_per_block = simt_rows_per_block(Dv);
  a.q = q, a.k = k, a.v = v, a.g = g, a.beta = beta, a.h0 = state_in, a.y = y, a.ckpt = states;
  cudaError_t e = simt_launch(SimtKind::Verify, a, N, in_dtype == QB_DTYPE_BF16, out_dtype == QB_DTYPE_BF16,
                              (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta verify", err, errlen);
}

int qb_gdn_keep_rows(int32_t N, int32_t V, int32_t Hv, int32_t Dk, int32_t Dv, const float* states,
                     const int32_t* keep, float* state_out, int32_t* status, void* stream, char* err, int errlen) {
  if (N < 0 || V < 1 || Hv < 1 || Dk < 1 || Dv < 1)
    return fail(err, errlen, "gated delta keep_rows: bad shape (N %d, V %d, Hv %d, Dk %d, Dv %d)", N, V, Hv, Dk, Dv);
  if (!states || !keep || !state_out) return fail(err, errlen, "gated delta keep_rows: null pointer");
  if (!aligned(states, 16) || !aligned(state_out, 16) || ((int64_t)Hv * Dv * Dk) % 4)
    return fail(err, errlen, "gated delta keep_rows: states need 16-byte alignment and Hv*Dv*Dk a multiple of 4");
  if (N == 0) return 0;
  cudaError_t e = launch_keep_rows(N, V, (int64_t)Hv * Dv * Dk, states, keep, state_out, status, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta keep_rows", err, errlen);
}

int qb_gdn_gate_fwd(int64_t P, int32_t Hk, int32_t Hv, int32_t Dk, int32_t in_dtype, int32_t out_dtype, const void* q,
                    const void* k, const float* a, const float* b, const float* A_log, const float* dt_bias, void* qn,
                    void* kn, float* g, float* beta, void* stream, char* err, int errlen) {
  if (P < 0 || Hk < 1 || Hv < 1 || Hv > 256 || (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256) ||
      !dtype_ok(in_dtype) || !dtype_ok(out_dtype))
    return fail(err, errlen, "gated delta gate: bad arguments (P %lld, Hk %d, Hv %d (<= 256), Dk %d, dtypes %d/%d)",
                (long long)P, Hk, Hv, Dk, in_dtype, out_dtype);
  if (!q || !k || !a || !b || !A_log || !dt_bias || !qn || !kn || !g || !beta)
    return fail(err, errlen, "gated delta gate: every pointer must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16)) return fail(err, errlen, "gated delta gate: q, k need 16-byte alignment");
  if (P == 0) return 0;
  GateArgs ga{};
  ga.P = P, ga.Hk = Hk, ga.Hv = Hv, ga.Dk = Dk;
  ga.q = q, ga.k = k, ga.a = a, ga.b = b, ga.A_log = A_log, ga.dt_bias = dt_bias;
  ga.qn = qn, ga.kn = kn, ga.g = g, ga.beta = beta;
  cudaError_t e = gate_fwd(ga, in_dtype == QB_DTYPE_BF16, out_dtype == QB_DTYPE_BF16, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta gate", err, errlen);
}

int64_t qb_gdn_gate_workspace_bytes(int64_t P, int32_t Hv) {
  return align256((int64_t)gate_head_blocks(P) * Hv * 2 * 4);
}

int qb_gdn_gate_bwd(int64_t P, int32_t Hk, int32_t Hv, int32_t Dk, int32_t in_dtype, int32_t out_dtype, const void* q,
                    const void* k, const float* a, const float* b, const float* A_log, const float* dt_bias,
                    const void* dqn, const void* dkn, const float* dg, const float* dbeta, void* dq, void* dk,
                    float* da, float* db, float* dA_log, float* ddt_bias, void* ws, int64_t ws_bytes, void* stream,
                    char* err, int errlen) {
  if (P < 0 || Hk < 1 || Hv < 1 || Hv > 256 || (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256) ||
      !dtype_ok(in_dtype) || !dtype_ok(out_dtype))
    return fail(err, errlen, "gated delta gate backward: bad arguments (P %lld, Hk %d, Hv %d (<= 256), Dk %d)",
                (long long)P, Hk, Hv, Dk);
  if (!q || !k || !a || !b || !A_log || !dt_bias || !dqn || !dkn || !dg || !dbeta || !dq || !dk || !da || !db ||
      !dA_log || !ddt_bias)
    return fail(err, errlen, "gated delta gate backward: every pointer must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(dqn, 16) || !aligned(dkn, 16))
    return fail(err, errlen, "gated delta gate backward: q, k, dqn, dkn need 16-byte alignment");
  const int64_t need = qb_gdn_gate_workspace_bytes(P, Hv);
  if (!ws || ws_bytes < need)
    return fail(err, errlen, "gated delta gate backward: workspace of %lld bytes needed (got %lld)", (long long)need,
                (long long)ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (P == 0) {
    cudaError_t e = cudaMemsetAsync(dA_log, 0, Hv * 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ddt_bias, 0, Hv * 4, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta gate backward", err, errlen);
  }
  GateArgs ga{};
  ga.P = P, ga.Hk = Hk, ga.Hv = Hv, ga.Dk = Dk;
  ga.q = q, ga.k = k, ga.a = a, ga.b = b, ga.A_log = A_log, ga.dt_bias = dt_bias;
  ga.dqn = dqn, ga.dkn = dkn, ga.dg = dg, ga.dbeta = dbeta;
  ga.dq = dq, ga.dk = dk, ga.da = da, ga.db = db, ga.dA_log = dA_log, ga.ddt_bias = ddt_bias;
  cudaError_t e = gate_bwd(ga, in_dtype == QB_DTYPE_BF16, out_dtype == QB_DTYPE_BF16, (float*)ws, st);
  return e == cudaSuccess ? 0 : cuda_fail(e, "gated delta gate backward", err, errlen);
}

}  // extern "C"
