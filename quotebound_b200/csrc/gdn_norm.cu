// The gated RMSNorm after the recurrence (src/deltanet.cpp:35-45, :122): per (token, value head) row
// of y [tokens, Hv, Dv], n = rms_norm(y, w, eps) = y rsqrt(mean(y^2) + eps) w rounded to y's dtype, then
// o = (silu(z) n) computed in float32 and rounded to y's dtype (Qwen3NextRMSNormGated's tail, as
// precise_swiglu runs it), z [tokens, Hv, Dv] the gate projection, w [Dv] float32.  Its backward
// (autodiff through those ops, the roundings passing the cotangent through):
//   dn = do silu(z),  dz = do n silu'(z),
//   dy = r (w dn) - y r^3 (sum_e y_e w_e dn_e) / Dv,  dw = sum over rows of dn y r.
// HBM-bound: one warp per row, Dv / 32 elements per lane, warp-shuffle row sums; dw summed per block
// in a fixed row order, then over blocks in order (deterministic, no atomics).
#include "../../include/qb_gdn.h"
#include "capi_util.cuh"
#include "gdn_common.cuh"
#include "launch_count.cuh"

namespace qbgdn {

namespace {

constexpr int NW = 8;           // warps per block
constexpr int NB_MAX = 148 * 4; // blocks of the backward (its dw partials)

template <typename T>
__device__ __forceinline__ float rnd(float x);
template <>
__device__ __forceinline__ float rnd<float>(float x) { return x; }
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

struct NormArgs {
  int64_t rows;  // tokens * Hv
  int Dv;
  float eps;
  const void *y, *z, *dout;
  const float* w;
  void *o, *dy, *dz;
  float* part;  // [blocks, Dv]
};

// Lane l holds elements l + 32 j, j < NV (coalesced across the warp).
template <int NV, typename T>
__global__ void __launch_bounds__(NW * 32) gdn_gated_norm_fwd(NormArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = blockIdx.x * (int64_t)NW + (threadIdx.x >> 5);
  const T* y = static_cast<const T*>(a.y);
  const T* z = static_cast<const T*>(a.z);
  T* o = static_cast<T*>(a.o);
  float w[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) w[j] = a.w[lane + 32 * j];
  for (int64_t r = warp0; r < a.rows; r += (int64_t)gridDim.x * NW) {
    const int64_t base = r * a.Dv;
    float yv[NV], zv[NV], ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      yv[j] = to_f(y[base + lane + 32 * j]);
      zv[j] = to_f(z[base + lane + 32 * j]);
      ss = fmaf(yv[j], yv[j], ss);
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / a.Dv + a.eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float n = rnd<T>(yv[j] * rs * w[j]);
      o[base + lane + 32 * j] = from_f<T>(zv[j] * sigm(zv[j]) * n);
    }
  }
}

template <int NV, typename T>
__global__ void __launch_bounds__(NW * 32) gdn_gated_norm_bwd(NormArgs a) {
  __shared__ float red[NW][NV * 32];
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const int64_t warp0 = blockIdx.x * (int64_t)NW + wi;
  const T* y = static_cast<const T*>(a.y);
  const T* z = static_cast<const T*>(a.z);
  const T* dout = static_cast<const T*>(a.dout);
  T* dy = static_cast<T*>(a.dy);
  T* dz = static_cast<T*>(a.dz);
  float w[NV], dwa[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) w[j] = a.w[lane + 32 * j], dwa[j] = 0.f;
  for (int64_t r = warp0; r < a.rows; r += (int64_t)gridDim.x * NW) {
    const int64_t base = r * a.Dv;
    float yv[NV], zv[NV], gv[NV], ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      yv[j] = to_f(y[base + lane + 32 * j]);
      zv[j] = to_f(z[base + lane + 32 * j]);
      gv[j] = to_f(dout[base + lane + 32 * j]);
      ss = fmaf(yv[j], yv[j], ss);
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / a.Dv + a.eps);
    float dn[NV], dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float s = sigm(zv[j]);
      const float n = rnd<T>(yv[j] * rs * w[j]);
      dn[j] = gv[j] * zv[j] * s;
      dz[base + lane + 32 * j] = from_f<T>(gv[j] * n * s * (1.f + zv[j] * (1.f - s)));
      dot = fmaf(yv[j] * w[j], dn[j], dot);
      dwa[j] = fmaf(dn[j], yv[j] * rs, dwa[j]);
    }
    dot = warp_sum(dot);
    const float c3 = rs * rs * rs * dot / a.Dv;
#pragma unroll
    for (int j = 0; j < NV; ++j) dy[base + lane + 32 * j] = from_f<T>(rs * w[j] * dn[j] - c3 * yv[j]);
  }
  if (a.part) {  // this block's dw: its warps' sums in warp order
#pragma unroll
    for (int j = 0; j < NV; ++j) red[wi][lane + 32 * j] = dwa[j];
    __syncthreads();
    for (int i = threadIdx.x; i < a.Dv; i += NW * 32) {
      float s = 0.f;
      for (int q = 0; q < NW; ++q) s += red[q][i];
      a.part[(int64_t)blockIdx.x * a.Dv + i] = s;
    }
  }
}

__global__ void gdn_gated_norm_dw(const float* part, int blocks, int Dv, float* dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= Dv) return;
  float s = 0.f;
  for (int b = 0; b < blocks; ++b) s += part[(int64_t)b * Dv + i];
  dw[i] = s;
}

int norm_blocks(int64_t rows) {
  const int64_t b = (rows + NW - 1) / NW;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, NB_MAX));
}

template <typename T>
cudaError_t launch_norm(bool bwd, const NormArgs& a, cudaStream_t st) {
  const int nb = norm_blocks(a.rows);
#define QB_NORM_CASE(NV)                                                                   \
  case NV:                                                                                 \
    if (bwd) gdn_gated_norm_bwd<NV, T><<<nb, NW * 32, 0, st>>>(a);                         \
    else gdn_gated_norm_fwd<NV, T><<<nb, NW * 32, 0, st>>>(a);                             \
    break;
  switch (a.Dv / 32) {
    QB_NORM_CASE(1)
    QB_NORM_CASE(2)
    QB_NORM_CASE(4)
    QB_NORM_CASE(8)
    default:
      return cudaErrorInvalidValue;
  }
#undef QB_NORM_CASE
  note_launch();
  return cudaGetLastError();
}

int check_norm(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const char* what, char* err, int errlen) {
  if (P < 0 || Hv < 1 || (Dv != 32 && Dv != 64 && Dv != 128 && Dv != 256) || !(eps >= 0.f) ||
      (dtype != QB_DTYPE_F32 && dtype != QB_DTYPE_BF16))
    return capi_fail(err, errlen, "%s: bad arguments (P %lld, Hv %d, Dv %d in {32, 64, 128, 256}, eps %g, dtype %d)",
                     what, (long long)P, Hv, Dv, (double)eps, dtype);
  return 0;
}

}  // namespace
}  // namespace qbgdn

using namespace qbgdn;

extern "C" {

int qb_gdn_gated_norm_fwd(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const void* y, const void* z,
                          const float* w, void* o, void* stream, char* err, int errlen) {
  if (check_norm(P, Hv, Dv, eps, dtype, "gated delta gated norm", err, errlen)) return -1;
  if (!y || !z || !w || !o) return capi_fail(err, errlen, "gated delta gated norm: every pointer must be non-null");
  if (P == 0) return 0;
  NormArgs a{};
  a.rows = P * Hv, a.Dv = Dv, a.eps = eps, a.y = y, a.z = z, a.w = w, a.o = o;
  cudaError_t e = dtype == QB_DTYPE_BF16 ? launch_norm<__nv_bfloat16>(false, a, (cudaStream_t)stream)
                                         : launch_norm<float>(false, a, (cudaStream_t)stream);
  return capi_cuda(e, "gated delta gated norm", err, errlen);
}

int64_t qb_gdn_gated_norm_workspace_bytes(int64_t P, int32_t Hv, int32_t Dv) {
  if (P < 0 || Hv < 1 || Dv < 1) return -1;
  return (((int64_t)norm_blocks(P * Hv) * Dv * 4 + 255) / 256) * 256;
}

int qb_gdn_gated_norm_bwd(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const void* y, const void* z,
                          const float* w, const void* dout, void* dy, void* dz, float* dw, void* ws, int64_t ws_bytes,
                          void* stream, char* err, int errlen) {
  if (check_norm(P, Hv, Dv, eps, dtype, "gated delta gated norm backward", err, errlen)) return -1;
  if (!y || !z || !w || !dout || !dy || !dz)
    return capi_fail(err, errlen, "gated delta gated norm backward: y, z, w, dout, dy and dz must be non-null");
  const int64_t need = qb_gdn_gated_norm_workspace_bytes(P, Hv, Dv);
  if (dw && (!ws || ws_bytes < need))
    return capi_fail(err, errlen, "gated delta gated norm backward: dw needs a workspace of %lld bytes (got %lld)",
                     (long long)need, (long long)ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (P == 0) return dw ? capi_cuda(cudaMemsetAsync(dw, 0, (size_t)Dv * 4, st), "gated delta gated norm backward", err,
                                    errlen)
                        : 0;
  NormArgs a{};
  a.rows = P * Hv, a.Dv = Dv, a.eps = eps, a.y = y, a.z = z, a.w = w, a.dout = dout, a.dy = dy, a.dz = dz;
  a.part = dw ? static_cast<float*>(ws) : nullptr;
  cudaError_t e = dtype == QB_DTYPE_BF16 ? launch_norm<__nv_bfloat16>(true, a, st) : launch_norm<float>(true, a, st);
  if (e == cudaSuccess && dw) {
    gdn_gated_norm_dw<<<(Dv + 127) / 128, 128, 0, st>>>(a.part, norm_blocks(a.rows), Dv, dw);
    note_launch();
    e = cudaGetLastError();
  }
  return capi_cuda(e, "gated delta gated norm backward", err, errlen);
}

}  // extern "C"
