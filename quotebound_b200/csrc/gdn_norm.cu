// The gated RMSNorm after the recurrence (src/deltanet.cpp:35-45, :122): per (token, value head) row
// of y [tokens, Hv, Dv], n = rms_norm(y, w, eps) = y rsqrt(mean(y^2) + eps) w rounded to y's dtype, then
// o = (silu(z) n) computed in float32 and rounded to y's dtype (Qwen3NextRMSNormGated's tail, as
// precise_swiglu runs it), z [tokens, Hv, Dv] the gate projection, w [Dv] float32.  Its backward
// (autodiff through those ops, the roundings passing the cotangent through):
//   dn = do silu(z),  dz = do n silu'(z),
//   dy = r (w dn) - y r^3 (sum_e y_e w_e dn_e) / Dv,  dw = sum over rows of dn y r.
// HBM-bound: one warp per row, Dv / 32 consecutive elements per lane (one vector load per tensor), a
// full SM of warps, warp-shuffle row sums; dw summed per block in a fixed row order, then over blocks by
// one block per column in a fixed tree order (deterministic, no atomics).
#include "../../include/qb_gdn.h"
#include "capi_util.cuh"
#include "gdn_common.cuh"
#include "launch_count.cuh"

namespace qbgdn {

namespace {

constexpr int NW = 8;           // warps per block
// One row per warp at a time, and as many warps as fit (eight 256-thread blocks per SM in the forward,
// six in the backward, whose dw partials need the registers): measured on B200 at Dv = 128, more
// resident warps keep more loads in flight than more rows per warp do.
// Dv = 256 (eight elements per lane) needs more registers: four and three blocks.
constexpr int RF = 1;           // rows per warp in flight (forward)
constexpr int RB = 1;           // rows per warp in flight (backward)
__host__ __device__ constexpr int fwd_blocks_per_sm(int nv) { return nv >= 8 ? 4 : 8; }
__host__ __device__ constexpr int bwd_blocks_per_sm(int nv) { return nv >= 8 ? 3 : 6; }

template <typename T>
__device__ __forceinline__ float rnd(float x);
template <>
__device__ __forceinline__ float rnd<float>(float x) { return x; }
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// 1 / (1 + e^-x) with the approximate reciprocal (about 1 ulp; 0 once 1 + e^-x passes 2^126)
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// NV consecutive elements of a row as one vector load / store (NV = 1, 2, 4, 8).
template <int NV, typename T>
__device__ __forceinline__ void ldrow(const T* p, float (&o)[NV]) {
  if constexpr (sizeof(T) == 2) {
    if constexpr (NV == 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(p);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
        o[2 * e] = __low2float(h), o[2 * e + 1] = __high2float(h);
      }
    } else if constexpr (NV == 4) {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      const uint32_t u[2] = {w.x, w.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
        o[2 * e] = __low2float(h), o[2 * e + 1] = __high2float(h);
      }
    } else if constexpr (NV == 2) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(p);
      o[0] = __low2float(h), o[1] = __high2float(h);
    } else {
      o[0] = to_f(p[0]);
    }
  } else {
    if constexpr (NV >= 4) {
#pragma unroll
      for (int q = 0; q < NV / 4; ++q) {
        const float4 w = reinterpret_cast<const float4*>(p)[q];
        o[4 * q] = w.x, o[4 * q + 1] = w.y, o[4 * q + 2] = w.z, o[4 * q + 3] = w.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < NV; ++e) o[e] = p[e];
    }
  }
}
template <int NV, typename T>
__device__ __forceinline__ void strow(T* p, const float (&v)[NV]) {
  if constexpr (sizeof(T) == 2) {
    uint32_t u[NV / 2 > 0 ? NV / 2 : 1];
    if constexpr (NV >= 2) {
#pragma unroll
      for (int e = 0; e < NV / 2; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        u[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    if constexpr (NV == 8) *reinterpret_cast<uint4*>(p) = make_uint4(u[0], u[1], u[2], u[3]);
    else if constexpr (NV == 4) *reinterpret_cast<uint2*>(p) = make_uint2(u[0], u[1]);
    else if constexpr (NV == 2) *reinterpret_cast<uint32_t*>(p) = u[0];
    else p[0] = from_f<T>(v[0]);
  } else {
    if constexpr (NV >= 4) {
#pragma unroll
      for (int q = 0; q < NV / 4; ++q)
        reinterpret_cast<float4*>(p)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < NV; ++e) p[e] = v[e];
    }
  }
}

struct NormArgs {
  int64_t rows;  // tokens * Hv
  int Dv;
  float eps;
  const void *y, *z, *dout;
  const float* w;
  void *o, *dy, *dz;
  float* part;  // [blocks, Dv]
};

// Lane l holds elements NV l .. NV l + NV - 1 of a row (one vector per tensor, coalesced across the
// warp); a warp takes RF rows per iteration, all their loads in flight together.
template <int NV, typename T>
__global__ void __launch_bounds__(NW * 32, fwd_blocks_per_sm(NV)) gdn_gated_norm_fwd(NormArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = blockIdx.x * (int64_t)NW + (threadIdx.x >> 5), nwarps = (int64_t)gridDim.x * NW;
  const T* y = static_cast<const T*>(a.y);
  const T* z = static_cast<const T*>(a.z);
  T* o = static_cast<T*>(a.o);
  float w[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) w[j] = a.w[NV * lane + j];
  constexpr int R = RF;
  for (int64_t r0 = warp0; r0 < a.rows; r0 += R * nwarps) {
    float yv[R][NV], zv[R][NV], ss[R];
#pragma unroll
    for (int h = 0; h < R; ++h) {
      const int64_t r = r0 + h * nwarps;
      if (r < a.rows) {
        ldrow<NV, T>(y + r * a.Dv + NV * lane, yv[h]);
        ldrow<NV, T>(z + r * a.Dv + NV * lane, zv[h]);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) yv[h][j] = zv[h][j] = 0.f;
      }
    }
#pragma unroll
    for (int h = 0; h < R; ++h) {
      ss[h] = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) ss[h] = fmaf(yv[h][j], yv[h][j], ss[h]);
      ss[h] = warp_sum(ss[h]);
    }
#pragma unroll
    for (int h = 0; h < R; ++h) {
      const int64_t r = r0 + h * nwarps;
      if (r >= a.rows) continue;
      const float rs = rsqrtf(ss[h] / a.Dv + a.eps);
      float ov[NV];
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const float n = rnd<T>(yv[h][j] * rs * w[j]);
        ov[j] = zv[h][j] * sigm(zv[h][j]) * n;
      }
      strow<NV, T>(o + r * a.Dv + NV * lane, ov);
    }
  }
}

template <int NV, typename T>
__global__ void __launch_bounds__(NW * 32, bwd_blocks_per_sm(NV)) gdn_gated_norm_bwd(NormArgs a) {
  __shared__ float red[NW][NV * 32];
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const int64_t warp0 = blockIdx.x * (int64_t)NW + wi, nwarps = (int64_t)gridDim.x * NW;
  const T* y = static_cast<const T*>(a.y);
  const T* z = static_cast<const T*>(a.z);
  const T* dout = static_cast<const T*>(a.dout);
  T* dy = static_cast<T*>(a.dy);
  T* dz = static_cast<T*>(a.dz);
  float w[NV], dwa[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) w[j] = a.w[NV * lane + j], dwa[j] = 0.f;
  constexpr int R = RB;
  for (int64_t r0 = warp0; r0 < a.rows; r0 += R * nwarps) {
    float yv[R][NV], zv[R][NV], gv[R][NV], ss[R];
#pragma unroll
    for (int h = 0; h < R; ++h) {
      const int64_t r = r0 + h * nwarps;
      if (r < a.rows) {
        ldrow<NV, T>(y + r * a.Dv + NV * lane, yv[h]);
        ldrow<NV, T>(z + r * a.Dv + NV * lane, zv[h]);
        ldrow<NV, T>(dout + r * a.Dv + NV * lane, gv[h]);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) yv[h][j] = zv[h][j] = gv[h][j] = 0.f;
      }
    }
#pragma unroll
    for (int h = 0; h < R; ++h) {
      ss[h] = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) ss[h] = fmaf(yv[h][j], yv[h][j], ss[h]);
      ss[h] = warp_sum(ss[h]);
    }
#pragma unroll
    for (int h = 0; h < R; ++h) {
      const int64_t r = r0 + h * nwarps;
      if (r >= a.rows) continue;  // (uniform across the warp: r is the warp's)
      const float rs = rsqrtf(ss[h] / a.Dv + a.eps);
      float dn[NV], dzv[NV], dot = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const float s = sigm(zv[h][j]);
        const float n = rnd<T>(yv[h][j] * rs * w[j]);
        dn[j] = gv[h][j] * zv[h][j] * s;
        dzv[j] = gv[h][j] * n * s * (1.f + zv[h][j] * (1.f - s));
        dot = fmaf(yv[h][j] * w[j], dn[j], dot);
        dwa[j] = fmaf(dn[j], yv[h][j] * rs, dwa[j]);
      }
      strow<NV, T>(dz + r * a.Dv + NV * lane, dzv);
      dot = warp_sum(dot);
      const float c3 = rs * rs * rs * dot / a.Dv;
      float dyv[NV];
#pragma unroll
      for (int j = 0; j < NV; ++j) dyv[j] = rs * w[j] * dn[j] - c3 * yv[h][j];
      strow<NV, T>(dy + r * a.Dv + NV * lane, dyv);
    }
  }
  if (a.part) {  // this block's dw: its warps' sums in warp order
#pragma unroll
    for (int j = 0; j < NV; ++j) red[wi][NV * lane + j] = dwa[j];
    __syncthreads();
    for (int i = threadIdx.x; i < a.Dv; i += NW * 32) {
      float s = 0.f;
      for (int q = 0; q < NW; ++q) s += red[q][i];
      a.part[(int64_t)blockIdx.x * a.Dv + i] = s;
    }
  }
}

// dw[i] = the blocks' partials summed by one block per column: thread t sums blocks t, t + 256, ... in
// order, then a fixed tree over the threads (the same bits every run).
__global__ void __launch_bounds__(256) gdn_gated_norm_dw(const float* part, int blocks, int Dv, float* dw) {
  __shared__ float sh[256];
  const int i = blockIdx.x, t = threadIdx.x;
  float s = 0.f;
  for (int b = t; b < blocks; b += 256) s += part[(int64_t)b * Dv + i];
  sh[t] = s;
  __syncthreads();
  for (int h = 128; h > 0; h >>= 1) {
    if (t < h) sh[t] += sh[t + h];
    __syncthreads();
  }
  if (t == 0) dw[i] = sh[0];
}

// blocks of a launch: a warp per row, at most one wave (the backward's count is also its dw partials')
int norm_blocks(int64_t rows, int Dv, bool bwd) {
  const int per_sm = bwd ? bwd_blocks_per_sm(Dv / 32) : fwd_blocks_per_sm(Dv / 32);
  const int64_t b = (rows + NW - 1) / NW;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * per_sm));
}

template <typename T>
cudaError_t launch_norm(bool bwd, const NormArgs& a, cudaStream_t st) {
  const int nb = norm_blocks(a.rows, a.Dv, bwd);
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

// A lane's vector of a row: Dv / 32 elements, read and written as 16-byte (or smaller) words.
int64_t norm_align(int32_t Dv, int32_t dtype) {
  return std::min<int64_t>(16, (int64_t)(Dv / 32) * (dtype == QB_DTYPE_BF16 ? 2 : 4));
}

}  // namespace
}  // namespace qbgdn

using namespace qbgdn;

extern "C" {

int qb_gdn_gated_norm_fwd(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const void* y, const void* z,
                          const float* w, void* o, void* stream, char* err, int errlen) {
  if (check_norm(P, Hv, Dv, eps, dtype, "gated delta gated norm", err, errlen)) return -1;
  if (!y || !z || !w || !o) return capi_fail(err, errlen, "gated delta gated norm: every pointer must be non-null");
  const int64_t al = norm_align(Dv, dtype);
  if (!capi_aligned(y, al) || !capi_aligned(z, al) || !capi_aligned(o, al))
    return capi_fail(err, errlen, "gated delta gated norm: y, z and o need %lld-byte alignment", (long long)al);
  if (P == 0) return 0;
  NormArgs a{};
  a.rows = P * Hv, a.Dv = Dv, a.eps = eps, a.y = y, a.z = z, a.w = w, a.o = o;
  cudaError_t e = dtype == QB_DTYPE_BF16 ? launch_norm<__nv_bfloat16>(false, a, (cudaStream_t)stream)
                                         : launch_norm<float>(false, a, (cudaStream_t)stream);
  return capi_cuda(e, "gated delta gated norm", err, errlen);
}

int64_t qb_gdn_gated_norm_workspace_bytes(int64_t P, int32_t Hv, int32_t Dv) {
  if (P < 0 || Hv < 1 || Dv < 1) return -1;
  return (((int64_t)norm_blocks(P * Hv, Dv, true) * Dv * 4 + 255) / 256) * 256;
}

int qb_gdn_gated_norm_bwd(int64_t P, int32_t Hv, int32_t Dv, float eps, int32_t dtype, const void* y, const void* z,
                          const float* w, const void* dout, void* dy, void* dz, float* dw, void* ws, int64_t ws_bytes,
                          void* stream, char* err, int errlen) {
  if (check_norm(P, Hv, Dv, eps, dtype, "gated delta gated norm backward", err, errlen)) return -1;
  if (!y || !z || !w || !dout || !dy || !dz)
    return capi_fail(err, errlen, "gated delta gated norm backward: y, z, w, dout, dy and dz must be non-null");
  const int64_t al = norm_align(Dv, dtype);
  if (!capi_aligned(y, al) || !capi_aligned(z, al) || !capi_aligned(dout, al) || !capi_aligned(dy, al) ||
      !capi_aligned(dz, al))
    return capi_fail(err, errlen, "gated delta gated norm backward: y, z, dout, dy and dz need %lld-byte alignment",
                     (long long)al);
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
    gdn_gated_norm_dw<<<Dv, 256, 0, st>>>(a.part, norm_blocks(a.rows, Dv, true), Dv, dw);
    note_launch();
    e = cudaGetLastError();
  }
  return capi_cuda(e, "gated delta gated norm backward", err, errlen);
}

}  // extern "C"
