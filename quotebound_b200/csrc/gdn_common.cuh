// Shared device helpers for the Gated DeltaNet kernels (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qbgdn {

constexpr int kChunk = 64;  // steps per chunk (src/delta_grad.cpp:11)

// Chunk geometry: chunk index -> sequence, first token, valid steps.
struct Geo {
  int T, Hk, Hv, N;
  int ncs;                   // chunks per sequence (fixed-length batches)
  const int32_t* cu;         // varlen offsets or null
  const int64_t* chunk_off;  // varlen: first chunk of each sequence [N + 1]
};

__device__ __forceinline__ void chunk_info(const Geo& g, int64_t c, int& n, int64_t& tok0, int& L) {
  if (!g.cu) {
    n = (int)(c / g.ncs);
    const int j = (int)(c - (int64_t)n * g.ncs);
    tok0 = (int64_t)n * g.T + (int64_t)j * kChunk;
    L = min(kChunk, g.T - j * kChunk);
    return;
  }
  int lo = 0, hi = g.N - 1;  // last n with chunk_off[n] <= c
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.chunk_off[mid] <= c) lo = mid; else hi = mid - 1;
  }
  n = lo;
  tok0 = g.cu[n] + (c - g.chunk_off[n]) * kChunk;
  L = (int)min((int64_t)kChunk, (int64_t)g.cu[n + 1] - tok0);
}

__device__ __forceinline__ void seq_chunks(const Geo& g, int n, int64_t& c_first, int64_t& nchunks, int64_t& seq0,
                                           int64_t& seq1) {
  if (g.cu) {
    c_first = g.chunk_off[n];
    nchunks = g.chunk_off[n + 1] - c_first;
    seq0 = g.cu[n];
    seq1 = g.cu[n + 1];
  } else {
    c_first = (int64_t)n * g.ncs;
    nchunks = g.ncs;
    seq0 = (int64_t)n * g.T;
    seq1 = seq0 + g.T;
  }
}

// ---- element access for the two activation dtypes ---------------------------------------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Load N consecutive elements starting at p (p aligned to N elements) as floats.
template <int N, typename T>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = to_f(p[i]);
}
template <>
__device__ __forceinline__ void load_vec<4, float>(const float* __restrict__ p, float (&out)[4]) {
  const float4 x = *reinterpret_cast<const float4*>(p);
  out[0] = x.x, out[1] = x.y, out[2] = x.z, out[3] = x.w;
}
template <>
__device__ __forceinline__ void load_vec<4, __nv_bfloat16>(const __nv_bfloat16* __restrict__ p, float (&out)[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&x.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&x.y);
  out[0] = __low2float(a), out[1] = __high2float(a), out[2] = __low2float(b), out[3] = __high2float(b);
}
template <>
__device__ __forceinline__ void load_vec<8, __nv_bfloat16>(const __nv_bfloat16* __restrict__ p, float (&out)[8]) {
  const uint4 x = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    out[2 * i] = __low2float(h), out[2 * i + 1] = __high2float(h);
  }
}

template <int N>
__device__ __forceinline__ void store_vec(float* __restrict__ p, const float (&x)[N]) {
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    if (i + 4 <= N) {
      *reinterpret_cast<float4*>(p + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
    } else {
      for (int j = i; j < N; ++j) p[j] = x[j];
    }
  }
}

// Butterfly sum over the 32 lanes.  Every lane ends with the same value, and the order of the
// additions depends only on the lane pattern, so two kernels that call it on the same values get
// the same bits.
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// One step of one state row S[r, :], this lane holding columns [lane*NPT, lane*NPT + NPT):
//   S~ = g S;  u = S~ . k;  delta = beta (v - u);  S = S~ + delta k;  y = S . q
// Every product and sum is an explicit round-to-nearest intrinsic, so the compiler cannot fuse or
// reorder differently in different kernels: the step, the verify rows and the sequential forward
// all produce the same bits from the same inputs.
template <int NPT>
__device__ __forceinline__ float row_step(float (&s)[NPT], const float (&kk)[NPT], const float (&qq)[NPT], float v,
                                          float g, float beta, float* u_out = nullptr, float* d_out = nullptr) {
  float u = 0.f;
#pragma unroll
  for (int i = 0; i < NPT; ++i) {
    s[i] = __fmul_rn(s[i], g);
    u = __fmaf_rn(s[i], kk[i], u);
  }
  u = warp_sum(u);
  const float d = __fmul_rn(__fsub_rn(v, u), beta);
  float o = 0.f;
#pragma unroll
  for (int i = 0; i < NPT; ++i) {
    s[i] = __fmaf_rn(kk[i], d, s[i]);
    o = __fmaf_rn(s[i], qq[i], o);
  }
  if (u_out) *u_out = u;
  if (d_out) *d_out = d;
  return warp_sum(o);
}

}  // namespace qbgdn
