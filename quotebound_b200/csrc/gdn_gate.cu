// The gate / beta / q-k norm graph that feeds the recurrence (src/deltanet.cpp:94-100, compute_g
// :22-33) and its chain rule.  HBM-bound elementwise work: one warp per (token, key head) row of
// q and k, coalesced 16-byte loads, warp-shuffle reductions; per-head parameter gradients summed
// in a fixed order (block partials, then one block over the partials) with no atomics.
#include <cuda.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "../../include/qb_gdn.h"
#include "gdn_common.cuh"
#include "gdn_gate.cuh"
#include "launch_count.cuh"

namespace qbgdn {

__device__ __forceinline__ float softplus_f(float x) {
  // logaddexp(x, 0) = max(x, 0) + log1p(exp(-|x|))
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

template <int NPT, typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gdn_gate_fwd_kernel(GateArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t rows = a.P * a.Hk;
  const float sq = 1.f / a.Dk, sk = rsqrtf((float)a.Dk);
  for (int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); w < 2 * rows; w += warps) {
    const bool is_k = w >= rows;
    const int64_t row = is_k ? w - rows : w;
    const Tin* src = static_cast<const Tin*>(is_k ? a.k : a.q) + row * a.Dk + lane * NPT;
    float x[NPT];
    load_vec<NPT>(src, x);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NPT; ++i) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / a.Dk + 1e-6f) * (is_k ? sk : sq);
    Tout* dst = static_cast<Tout*>(is_k ? a.kn : a.qn) + row * a.Dk + lane * NPT;
#pragma unroll
    for (int i = 0; i < NPT; ++i) dst[i] = from_f<Tout>(x[i] * r);
  }
  const int64_t n = a.P * a.Hv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)(i % a.Hv);
    const float x = a.a[i] + a.dt_bias[h];
    a.g[i] = expf(-expf(a.A_log[h]) * softplus_f(x));
    a.beta[i] = sigmoid_f(a.b[i]);
  }
}

// dq = s (r dqn - r^3 (q . dqn) q / Dk), r = rsqrt(mean(q^2) + eps), s the 1/Dk or 1/sqrt(Dk) scale.
template <int NPT, typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gdn_gate_bwd_rows(GateArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t rows = a.P * a.Hk;
  const float sq = 1.f / a.Dk, sk = rsqrtf((float)a.Dk);
  for (int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); w < 2 * rows; w += warps) {
    const bool is_k = w >= rows;
    const int64_t row = is_k ? w - rows : w;
    const size_t off = row * a.Dk + lane * NPT;
    float x[NPT], dx[NPT];
    load_vec<NPT>(static_cast<const Tin*>(is_k ? a.k : a.q) + off, x);
    load_vec<NPT>(static_cast<const Tin*>(is_k ? a.dkn : a.dqn) + off, dx);
    float ss = 0.f, sd = 0.f;
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      ss = fmaf(x[i], x[i], ss);
      sd = fmaf(x[i], dx[i], sd);
    }
    ss = warp_sum(ss);
    sd = warp_sum(sd);
    const float r = rsqrtf(ss / a.Dk + 1e-6f), s = is_k ? sk : sq;
    const float c = r * r * r * sd / a.Dk;
    Tout* dst = static_cast<Tout*>(is_k ? a.dk : a.dq) + off;
#pragma unroll
    for (int i = 0; i < NPT; ++i) dst[i] = from_f<Tout>(s * (r * dx[i] - c * x[i]));
  }
}

// da, db per element; per-block partial sums of dA_log (= sum dlogg * logg) and ddt_bias (= sum da).
// Block j covers tokens [j * per, (j+1) * per); thread t handles head t % Hv, tokens t / Hv + k * stride.
__global__ void __launch_bounds__(256) gdn_gate_bwd_heads(GateArgs a, int64_t per, float* partial) {
  extern __shared__ float sh[];  // [blockDim.x][2]
  const int tid = threadIdx.x;
  const int lanes_per_head = blockDim.x / a.Hv;  // >= 1 (host guarantees Hv <= blockDim.x)
  const int h = tid % a.Hv, sub = tid / a.Hv;
  float acc_a = 0.f, acc_d = 0.f;
  if (sub < lanes_per_head) {
    const int64_t t0 = blockIdx.x * per, t1 = min(a.P, t0 + per);
    const float eA = expf(a.A_log[h]);
    for (int64_t t = t0 + sub; t < t1; t += lanes_per_head) {
      const int64_t i = t * a.Hv + h;
      const float x = a.a[i] + a.dt_bias[h];
      const float lg = -eA * softplus_f(x);
      const float dl = a.dg[i] * expf(lg);  // d loss / d log g
      const float dx = dl * (-eA * sigmoid_f(x));
      a.da[i] = dx;
      acc_d += dx;
      acc_a = fmaf(dl, lg, acc_a);
      const float bb = sigmoid_f(a.b[i]);
      a.db[i] = a.dbeta[i] * bb * (1.f - bb);
    }
  }
  sh[2 * tid] = acc_a;
  sh[2 * tid + 1] = acc_d;
  __syncthreads();
  if (tid < a.Hv) {
    float sa = 0.f, sd = 0.f;
    for (int s = 0; s < lanes_per_head; ++s) {
      sa += sh[2 * (s * a.Hv + tid)];
      sd += sh[2 * (s * a.Hv + tid) + 1];
    }
    partial[((int64_t)blockIdx.x * a.Hv + tid) * 2] = sa;
    partial[((int64_t)blockIdx.x * a.Hv + tid) * 2 + 1] = sd;
  }
}

__global__ void gdn_gate_bwd_finish(int nblk, int Hv, const float* partial, float* dA_log, float* ddt_bias) {
  for (int h = threadIdx.x; h < Hv; h += blockDim.x) {
    float sa = 0.f, sd = 0.f;
    for (int j = 0; j < nblk; ++j) {
      sa += partial[((int64_t)j * Hv + h) * 2];
      sd += partial[((int64_t)j * Hv + h) * 2 + 1];
    }
    dA_log[h] = sa;
    ddt_bias[h] = sd;
  }
}

template <typename Tin, typename Tout>
static cudaError_t gate_fwd_t(const GateArgs& a, cudaStream_t st) {
  const int64_t work = 2 * a.P * a.Hk;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 7) / 8, 148 * 8));
  switch (a.Dk / 32) {
    case 1: gdn_gate_fwd_kernel<1, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    case 2: gdn_gate_fwd_kernel<2, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    case 4: gdn_gate_fwd_kernel<4, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    case 8: gdn_gate_fwd_kernel<8, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename Tin, typename Tout>
static cudaError_t gate_bwd_t(const GateArgs& a, float* partial, cudaStream_t st) {
  const int64_t work = 2 * a.P * a.Hk;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 7) / 8, 148 * 8));
  switch (a.Dk / 32) {
    case 1: gdn_gate_bwd_rows<1, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    case 2: gdn_gate_bwd_rows<2, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    case 4: gdn_gate_bwd_rows<4, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    case 8: gdn_gate_bwd_rows<8, Tin, Tout><<<blocks, 256, 0, st>>>(a); note_launch(); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int nblk = gate_head_blocks(a.P);
  const int64_t per = (a.P + nblk - 1) / nblk;
  gdn_gate_bwd_heads<<<nblk, 256, 256 * 2 * sizeof(float), st>>>(a, per, partial);
  note_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  gdn_gate_bwd_finish<<<1, 128, 0, st>>>(nblk, a.Hv, partial, a.dA_log, a.ddt_bias);
  note_launch();
  return cudaGetLastError();
}

int gate_head_blocks(int64_t P) { return (int)std::max<int64_t>(1, std::min<int64_t>(148, (P + 63) / 64)); }

cudaError_t gate_fwd(const GateArgs& a, int in_bf16, int out_bf16, cudaStream_t st) {
  if (in_bf16 && out_bf16) return gate_fwd_t<__nv_bfloat16, __nv_bfloat16>(a, st);
  if (in_bf16) return gate_fwd_t<__nv_bfloat16, float>(a, st);
  if (out_bf16) return gate_fwd_t<float, __nv_bfloat16>(a, st);
  return gate_fwd_t<float, float>(a, st);
}

cudaError_t gate_bwd(const GateArgs& a, int in_bf16, int out_bf16, float* partial, cudaStream_t st) {
  if (in_bf16 && out_bf16) return gate_bwd_t<__nv_bfloat16, __nv_bfloat16>(a, partial, st);
  if (in_bf16) return gate_bwd_t<__nv_bfloat16, float>(a, partial, st);
  if (out_bf16) return gate_bwd_t<float, __nv_bfloat16>(a, partial, st);
  return gate_bwd_t<float, float>(a, partial, st);
}

}  // namespace qbgdn

// ------------------------------------------------------------------------------------------------
// The gate backward for callers that cannot allocate device memory: its per-block partial sums live
// in a fixed array in the library's own device memory instead of a caller-provided workspace.
namespace qbgdn {
namespace {

// Blocks of gdn_gate_bwd_heads (at most 148) x value heads (at most 256) x 2 sums, float32: 296 KiB,
// held by every GPU that loads the library until the process exits.
constexpr int64_t kGateScratchFloats = 148 * 256 * 2;
static __device__ __align__(256) float g_gate_scratch[kGateScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
// device address of g_gate_scratch per device, and the context it was looked up in: a device reset or
// a re-created primary context loads the module anew, so a new context means a fresh lookup
float* g_scratch_ptr[kMaxDevices];
CUcontext g_scratch_ctx[kMaxDevices];

int noalloc_fail(char* err, int errlen, const char* fmt, ...) {
  if (err && errlen > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
    err[errlen - 1] = '\0';
  }
  return -1;
}

// The device address of the scratch array on the current device, looked up once per device and
// context (cudaGetSymbolAddress with that device current).
cudaError_t scratch_on_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  static CUresult (*get_ctx)(CUcontext*) = nullptr;
  if (!get_ctx) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return cudaErrorNotSupported;
    get_ctx = reinterpret_cast<CUresult (*)(CUcontext*)>(fn);
  }
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return cudaErrorDeviceUninitialized;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!ctx || !g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
    // (the lookup itself makes the device's primary context current when none is yet)
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gate_scratch);
    if (e != cudaSuccess) return e;
    if (get_ctx(&ctx) != CUDA_SUCCESS) return cudaErrorDeviceUninitialized;
    g_scratch_ptr[dev] = static_cast<float*>(p);
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace qbgdn

extern "C" int qb_gdn_gate_bwd_noalloc(int64_t P, int32_t Hk, int32_t Hv, int32_t Dk, int32_t in_dtype,
                                       int32_t out_dtype, const void* q, const void* k, const float* a,
                                       const float* b, const float* A_log, const float* dt_bias, const void* dqn,
                                       const void* dkn, const float* dg, const float* dbeta, void* dq, void* dk,
                                       float* da, float* db, float* dA_log, float* ddt_bias, void* stream,
                                       char* err, int errlen) {
  using namespace qbgdn;
  const bool dt_ok = (in_dtype == QB_DTYPE_F32 || in_dtype == QB_DTYPE_BF16) &&
                     (out_dtype == QB_DTYPE_F32 || out_dtype == QB_DTYPE_BF16);
  if (P < 0 || Hk < 1 || Hv < 1 || (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256) || !dt_ok)
    return noalloc_fail(err, errlen, "gated delta gate backward (no-alloc): bad arguments (P %lld, Hk %d, Hv %d, Dk %d)",
                        (long long)P, Hk, Hv, Dk);
  const int64_t need = (int64_t)gate_head_blocks(P) * Hv * 2;
  if (Hv > 256 || need > kGateScratchFloats)
    return noalloc_fail(err, errlen,
                        "gated delta gate backward (no-alloc): Hv = %d needs %lld scratch floats; the fixed scratch "
                        "holds %lld (at most 256 value heads)",
                        Hv, (long long)need, (long long)kGateScratchFloats);
  if (!q || !k || !a || !b || !A_log || !dt_bias || !dqn || !dkn || !dg || !dbeta || !dq || !dk || !da || !db ||
      !dA_log || !ddt_bias)
    return noalloc_fail(err, errlen, "gated delta gate backward (no-alloc): every pointer must be non-null");
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)dqn | (uintptr_t)dkn) % 16)
    return noalloc_fail(err, errlen, "gated delta gate backward (no-alloc): q, k, dqn, dkn need 16-byte alignment");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  if (P == 0) {
    e = cudaMemsetAsync(dA_log, 0, Hv * 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ddt_bias, 0, Hv * 4, st);
  } else {
    float* scratch = nullptr;
    e = scratch_on_current_device(&scratch);
    if (e == cudaSuccess) {
      // Every partial the finishing kernel reads is written first by the heads kernel, so nothing in
      // the scratch needs clearing between calls.
      GateArgs ga{};
      ga.P = P, ga.Hk = Hk, ga.Hv = Hv, ga.Dk = Dk;
      ga.q = q, ga.k = k, ga.a = a, ga.b = b, ga.A_log = A_log, ga.dt_bias = dt_bias;
      ga.dqn = dqn, ga.dkn = dkn, ga.dg = dg, ga.dbeta = dbeta;
      ga.dq = dq, ga.dk = dk, ga.da = da, ga.db = db, ga.dA_log = dA_log, ga.ddt_bias = ddt_bias;
      e = gate_bwd(ga, in_dtype == QB_DTYPE_BF16, out_dtype == QB_DTYPE_BF16, scratch, st);
    }
  }
  if (e != cudaSuccess)
    return noalloc_fail(err, errlen, "gated delta gate backward (no-alloc): CUDA error %d (%s)", (int)e,
                        cudaGetErrorString(e));
  return 0;
}
