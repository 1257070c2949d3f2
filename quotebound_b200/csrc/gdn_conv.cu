// The causal depthwise conv1d + SiLU in front of the recurrence, fused with the q / k / v split
// (src/deltanet.cpp:74-93): the projected channels x [tokens, conv_dim] (conv_dim = 2 Hk Dk + Hv Dv,
// in the order q | k | v) are convolved over time with K taps per channel, each token's window being
// the K - 1 inputs before it (the carried conv state at a sequence's start, zeros without one), then
// u = bf16(conv), y = bf16(u sigmoid(u)) -- the dtypes of MLX's conv1d and compiled silu -- and
// written straight into contiguous q [tokens, Hk, Dk], k and v [tokens, Hv, Dv], the raw rows the
// fused recurrence (qb_gdn_layer_fwd) normalises.  The new conv state is the last K - 1 inputs
// (src/deltanet.cpp:75-77).  The backward gives dx, dw and the initial state's cotangent; the verify
// form runs V tokens as V one-token steps bit for bit and keeps every token's conv window
// (src/deltanet.cpp:79-87, RowStates.conv in src/model.h:84-89).
//
// One thread owns 4 consecutive channels (one 8-byte bf16 vector) over a chunk of 64 tokens of one
// sequence, with the K - 1 previous inputs in registers, so x is read once (plus K - 1 rows of halo per
// chunk) and each output written once, all coalesced along the channels.  Each thread's rows stream
// through a queue of its own in shared memory (cp.async into its slot of a ring, a dozen rows in
// flight), so these kernels are not bound by memory latency; what bounds them is the instruction issue
// of the per-element arithmetic (the conv, its bf16 rounding, the SiLU's exponential and reciprocal).
#include <type_traits>

#include "../../include/qb_gdn.h"
#include "capi_util.cuh"
#include "gdn_common.cuh"
#include "gdn_simt.cuh"
#include "launch_count.cuh"

namespace qbgdn {

namespace {

constexpr int CV = 8;     // channels per thread (forward, verify)
constexpr int CVB = 4;    // channels per thread (backward)
constexpr int CVF = 4;    // channels per thread (forward)
constexpr int NTC = 256;  // threads per block

struct ConvArgs {
  Geo geo;
  int key_dim, value_dim, conv_dim;
  const void *x, *w, *state_in;   // x [tokens, conv_dim], w [conv_dim, K], state [N, K-1, conv_dim]
  void *q, *k, *v, *state_out;
  const void *dq, *dk, *dv, *dstate_out;
  void* dx;
  float* dw_part;                 // [chunks, conv_dim, K]
  void* dstate_in;
};

template <typename T>
__device__ __forceinline__ float round_to(float x);
template <>
__device__ __forceinline__ float round_to<float>(float x) { return x; }
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// N channels of a row (N = 4 or 8): a raw vector load, converted when used.
template <int N, typename T>
struct RawV;
template <>
struct RawV<8, __nv_bfloat16> {
  uint4 w;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { w = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void lds(const uint8_t* p, int) { w = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void zero() { w = make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ void cvt(float (&o)[8]) const {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
      o[2 * e] = __low2float(h), o[2 * e + 1] = __high2float(h);
    }
  }
};
template <>
struct RawV<4, __nv_bfloat16> {
  uint2 w;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { w = *reinterpret_cast<const uint2*>(p); }
  __device__ __forceinline__ void lds(const uint8_t* p, int) { w = *reinterpret_cast<const uint2*>(p); }
  __device__ __forceinline__ void zero() { w = make_uint2(0, 0); }
  __device__ __forceinline__ void cvt(float (&o)[4]) const {
    const uint32_t u[2] = {w.x, w.y};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
      o[2 * e] = __low2float(h), o[2 * e + 1] = __high2float(h);
    }
  }
};
template <>
struct RawV<8, float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  }
  __device__ __forceinline__ void lds(const uint8_t* p, int stride) {
    a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + stride);
  }
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void cvt(float (&o)[8]) const {
    o[0] = a.x, o[1] = a.y, o[2] = a.z, o[3] = a.w, o[4] = b.x, o[5] = b.y, o[6] = b.z, o[7] = b.w;
  }
};
template <>
struct RawV<4, float> {
  float4 a;
  __device__ __forceinline__ void load(const float* p) { a = *reinterpret_cast<const float4*>(p); }
  __device__ __forceinline__ void lds(const uint8_t* p, int) { a = *reinterpret_cast<const float4*>(p); }
  __device__ __forceinline__ void zero() { a = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void cvt(float (&o)[4]) const { o[0] = a.x, o[1] = a.y, o[2] = a.z, o[3] = a.w; }
};
template <int N, typename T>
__device__ __forceinline__ void ldv(const T* p, float (&o)[N]) {
  RawV<N, T> r;
  r.load(p);
  r.cvt(o);
}
template <int N, typename T>
__device__ __forceinline__ void stv(T* p, const float (&v)[N]);
template <>
__device__ __forceinline__ void stv<8, __nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint32_t u[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    u[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(u[0], u[1], u[2], u[3]);
}
template <>
__device__ __forceinline__ void stv<4, __nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
  uint32_t u[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    u[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint2*>(p) = make_uint2(u[0], u[1]);
}
template <>
__device__ __forceinline__ void stv<8, float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void stv<4, float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

// A thread's queue of rows in flight: each row's N-channel vector copied by cp.async into this thread's
// own slot of a shared-memory ring (S slots), read back by the same thread once its commit group has
// completed (cp.async.wait_group) -- no barrier and no spin: the hardware counts the groups.  A vector
// of VB bytes is stored as VB / WB words of WB bytes, word w of slot s of thread t at
// ((s * NWD + w) * NTC + t) * WB, so that a warp's reads of one word are contiguous.
template <int N, typename T, int S>
struct RowRing {
  static constexpr int VB = N * (int)sizeof(T), WB = VB >= 16 ? 16 : VB, NWD = VB / WB;
  static constexpr int BYTES = S * NWD * NTC * WB;
  uint8_t* mine;  // this thread's word 0 of slot 0
  __device__ __forceinline__ RowRing(uint8_t* ring) : mine(ring + threadIdx.x * WB) {}
  __device__ __forceinline__ uint8_t* slot(int s) const { return mine + s * NWD * NTC * WB; }
  __device__ __forceinline__ void copy(int s, const T* src) const {  // the row vector at src into slot s
    const uint8_t* g = reinterpret_cast<const uint8_t*>(src);
#pragma unroll
    for (int w = 0; w < NWD; ++w) {
      const uint32_t d = (uint32_t)__cvta_generic_to_shared(slot(s) + w * NTC * WB);
      if constexpr (WB == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(g + w * WB) : "memory");
      else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(g + w * WB) : "memory");
    }
  }
  __device__ __forceinline__ static void commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
  // every group but the newest `pending` has completed
  template <int pending>
  __device__ __forceinline__ static void wait() { asm volatile("cp.async.wait_group %0;" ::"n"(pending) : "memory"); }
  __device__ __forceinline__ void read(int s, RawV<N, T>& r) const { r.lds(slot(s), NTC * WB); }
  __device__ __forceinline__ static int next(int s) { return s + 1 == S ? 0 : s + 1; }
};

// One output of N channels from the window xp[0 .. K-1] (oldest first): the conv in a fixed FMA order
// rounded to T, then its SiLU rounded to T.  Every kernel below calls exactly this, so the sequence
// form, a one-token step and the verify rows give the same bits.
template <int K, typename T, int N>
__device__ __forceinline__ void conv_silu(const float (&xp)[K][N], const float (&wv)[K][N], float (&u)[N],
                                          float (&y)[N]) {
#pragma unroll
  for (int e = 0; e < N; ++e) {
    float acc = 0.f;
#pragma unroll
    for (int m = 0; m < K; ++m) acc = __fmaf_rn(xp[m][e], wv[m][e], acc);
    u[e] = round_to<T>(acc);
    const float s = __fdividef(1.f, __fadd_rn(1.f, __expf(-u[e])));
    y[e] = __fmul_rn(u[e], s);  // rounded to T once, by the store (stv)
  }
}

// The output buffer and offset a channel vector goes to: q, k or v (no vector straddles two).
template <typename T>
__device__ __forceinline__ T* route(T* q, T* k, T* v, const ConvArgs& a, int64_t t, int c) {
  if (c < a.key_dim) return q + t * a.key_dim + c;
  if (c < 2 * a.key_dim) return k + t * a.key_dim + (c - a.key_dim);
  return v + t * a.value_dim + (c - 2 * a.key_dim);
}

template <int K, typename T, int N>
__device__ __forceinline__ void load_w(const ConvArgs& a, int cg, float (&wv)[K][N]) {
  const T* w = static_cast<const T*>(a.w);
#pragma unroll
  for (int e = 0; e < N; ++e)
#pragma unroll
    for (int m = 0; m < K; ++m) wv[m][e] = to_f(w[(size_t)(cg + e) * K + m]);
}

// The K - 1 inputs before token tok0 of the sequence starting at s0 (state rows before the start).
template <int K, typename T, int N>
__device__ __forceinline__ void load_halo(const ConvArgs& a, int n, int64_t s0, int64_t tok0, int cg,
                                          float (&xp)[K][N]) {
  const T* x = static_cast<const T*>(a.x);
  const T* st = static_cast<const T*>(a.state_in);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int64_t t = tok0 - (K - 1) + j;
    if (t >= s0) {
      ldv<N, T>(x + t * a.conv_dim + cg, xp[j]);
    } else if (st) {
      const int64_t p = t - s0 + (K - 1);  // row of the carried state
      ldv<N, T>(st + ((int64_t)n * (K - 1) + p) * a.conv_dim + cg, xp[j]);
    } else {
#pragma unroll
      for (int e = 0; e < N; ++e) xp[j][e] = 0.f;
    }
  }
}

template <int K, int N>
__device__ __forceinline__ void shift(float (&xp)[K][N]) {
#pragma unroll
  for (int j = 0; j < K - 1; ++j)
#pragma unroll
    for (int e = 0; e < N; ++e) xp[j][e] = xp[j + 1][e];
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Forward: grid (chunks, conv_dim / (256 * 8)); chunk c covers up to 64 tokens of one sequence.
template <int K, typename T>
__global__ void __launch_bounds__(NTC, 4) gdn_conv_fwd(ConvArgs a) {
  constexpr int N = CVF, S = 12 * 8 / (N * (int)sizeof(T));  // rows in flight per thread (24 KB a block)
  using Ring = RowRing<N, T, S>;
  __shared__ __align__(16) uint8_t ring_mem[Ring::BYTES];
  const int cg = (blockIdx.y * NTC + threadIdx.x) * N;
  if (cg >= a.conv_dim) return;
  const int64_t c = blockIdx.x;
  int n, L;
  int64_t tok0, cf, nc, s0, s1;
  chunk_info(a.geo, c, n, tok0, L);
  seq_chunks(a.geo, n, cf, nc, s0, s1);
  float wv[K][N], xp[K][N], u[N], y[N];
  load_w<K, T, N>(a, cg, wv);
  load_halo<K, T, N>(a, n, s0, tok0, cg, xp);
  const T* x = static_cast<const T*>(a.x);
  T *q = static_cast<T*>(a.q), *k = static_cast<T*>(a.k), *v = static_cast<T*>(a.v);
  // the chunk's rows stream through the ring: row i + S is copied once row i has been used (the
  // groups of rows past the chunk are empty, so that the count stays one group per row)
  const Ring ring(ring_mem);
#pragma unroll 1
  for (int i = 0; i < S; ++i) {
    if (i < L) ring.copy(i, x + (tok0 + i) * a.conv_dim + cg);
    Ring::commit();
  }
  int sl = 0;  // row i's slot, i % S
#pragma unroll 4
  for (int i = 0; i < L; ++i) {
    Ring::template wait<S - 1>();  // row i's group is complete
    RawV<N, T> r;
    ring.read(sl, r);
    r.cvt(xp[K - 1]);
    conv_silu<K, T, N>(xp, wv, u, y);
    stv<N, T>(route(q, k, v, a, tok0 + i, cg), y);
    shift<K, N>(xp);
    if (i + S < L) ring.copy(sl, x + (tok0 + i + S) * a.conv_dim + cg);  // slot i % S, read above
    Ring::commit();
    sl = Ring::next(sl);
  }
  if (a.state_out && c == cf + nc - 1) {  // the last chunk of the sequence: its window is the new state
    T* so = static_cast<T*>(a.state_out);
#pragma unroll
    for (int j = 0; j < K - 1; ++j) stv<N, T>(so + ((int64_t)n * (K - 1) + j) * a.conv_dim + cg, xp[j]);
  }
}

// Sequences with no tokens: the new state is the old one (their cotangents pass straight through).
template <int K, typename T>
__global__ void __launch_bounds__(NTC) gdn_conv_empty(const int32_t* cu, int conv_dim, const T* src, T* dst) {
  const int n = blockIdx.x;
  if (cu[n + 1] != cu[n]) return;
  for (int i = blockIdx.y * NTC + threadIdx.x; i < (K - 1) * conv_dim; i += gridDim.y * NTC) {
    const int64_t o = (int64_t)n * (K - 1) * conv_dim + i;
    dst[o] = src ? src[o] : from_f<T>(0.f);
  }
}

// ------------------------------------------------------------------------------------------------
// Backward.  With du_t = dy_t silu'(u_t) (u_t the rounded conv output; the rounding passes the
// cotangent through), input t receives du_{t + K-1-m} w_m from the outputs whose windows hold it, the
// taps receive du_t x-window_t, and the carried state's rows receive what falls before the sequence's
// start; the new state's cotangent (dstate_out) adds onto the last K - 1 inputs.  Each chunk
// recomputes u for its own outputs and the K - 1 after it (same sequence).
template <int K, typename T>
__global__ void __launch_bounds__(NTC, 3) gdn_conv_bwd(ConvArgs a) {
  constexpr int N = CVB, S = 12 * 8 / (N * (int)sizeof(T));  // rows of x and dy in flight (48 KB a block)
  using Ring = RowRing<N, T, S>;
  __shared__ __align__(16) uint8_t ring_mem[2 * Ring::BYTES];
  const int cg = (blockIdx.y * NTC + threadIdx.x) * N;
  if (cg >= a.conv_dim) return;
  const int64_t c = blockIdx.x;
  int n, L;
  int64_t tok0, cf, nc, s0, s1;
  chunk_info(a.geo, c, n, tok0, L);
  seq_chunks(a.geo, n, cf, nc, s0, s1);
  const int64_t Ls = s1 - s0;
  const bool first = c == cf;
  float wv[K][N], xp[K][N], u[N], du[K][N], dw[K][N];
  load_w<K, T, N>(a, cg, wv);
  load_halo<K, T, N>(a, n, s0, tok0, cg, xp);
#pragma unroll
  for (int m = 0; m < K; ++m)
#pragma unroll
    for (int e = 0; e < N; ++e) du[m][e] = dw[m][e] = 0.f;
  const T* x = static_cast<const T*>(a.x);
  const T *dq = static_cast<const T*>(a.dq), *dk = static_cast<const T*>(a.dk), *dv = static_cast<const T*>(a.dv);
  const T* dso = static_cast<const T*>(a.dstate_out);
  T* dx = static_cast<T*>(a.dx);
  T* dsi = static_cast<T*>(a.dstate_in);
  // inputs emitted: this chunk's tokens, and for the sequence's first chunk the K - 1 state rows
  const int64_t in_lo = first ? tok0 - (K - 1) : tok0, in_hi = tok0 + L, t_end = tok0 + L + K - 1;
  // rows tok0 .. t_lim - 1 of x and of the output gradient (outputs past the sequence's end have none)
  // stream through two rings, one commit group per row
  const int nrows = (int)(min(t_end, s1) - tok0);
  const Ring ringx(ring_mem), ringg(ring_mem + Ring::BYTES);
#pragma unroll 1
  for (int i = 0; i < S; ++i) {
    if (i < nrows) {
      ringx.copy(i, x + (tok0 + i) * a.conv_dim + cg);
      ringg.copy(i, route(dq, dk, dv, a, tok0 + i, cg));
    }
    Ring::commit();
  }
  int sl = 0;  // row i's slot, i % S
  // one token: du for output t (zero past the sequence's end; u recomputed as the forward rounds it, its
  // sigmoid s as the forward forms it, du = dy s (1 + u (1 - s))), then dx of input t - (K - 1), which has
  // now seen every output that reads it (du[K-1-m] is du_{t-m}).  FAST: a token of the chunk from its
  // K-th on, for which every test below has a known outcome (its row exists, it feeds dw, its input
  // ti = t - (K - 1) lies in the chunk, in the sequence, and before the carried state's rows).
  auto token = [&](int64_t t, auto fast) {
    constexpr bool FAST = decltype(fast)::value;
    const int i = (int)(t - tok0);
    shift<K, N>(du);
    if (FAST || i < nrows) {
      Ring::template wait<S - 1>();  // row i's group is complete
      RawV<N, T> rx, rg;
      ringx.read(sl, rx);
      ringg.read(sl, rg);
      rx.cvt(xp[K - 1]);
      float g[N];
      rg.cvt(g);
#pragma unroll
      for (int e = 0; e < N; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < K; ++m) acc = __fmaf_rn(xp[m][e], wv[m][e], acc);
        u[e] = round_to<T>(acc);
        const float s = __fdividef(1.f, __fadd_rn(1.f, __expf(-u[e])));
        du[K - 1][e] = g[e] * s * (1.f + u[e] * (1.f - s));
      }
      if (FAST || t < tok0 + L) {
#pragma unroll
        for (int m = 0; m < K; ++m)
#pragma unroll
          for (int e = 0; e < N; ++e) dw[m][e] = fmaf(du[K - 1][e], xp[m][e], dw[m][e]);
      }
      shift<K, N>(xp);
      if (i + S < nrows) {  // slots i % S, read above
        ringx.copy(sl, x + (tok0 + i + S) * a.conv_dim + cg);
        ringg.copy(sl, route(dq, dk, dv, a, tok0 + i + S, cg));
      }
      Ring::commit();
      sl = Ring::next(sl);
    } else {
#pragma unroll
      for (int e = 0; e < N; ++e) du[K - 1][e] = 0.f;
    }
    const int64_t ti = t - (K - 1);
    if (FAST || (ti >= in_lo && ti < in_hi)) {
      float d[N];
#pragma unroll
      for (int e = 0; e < N; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < K; ++m) acc = fmaf(du[K - 1 - m][e], wv[m][e], acc);
        d[e] = acc;
      }
      if constexpr (FAST) {
        stv<N, T>(dx + ti * a.conv_dim + cg, d);
      } else {
        const int64_t p = ti - s0 + (K - 1);  // padded position; the new state is positions Ls .. Ls + K - 2
        if (dso && p >= Ls) {
          float ds[N];
          ldv<N, T>(dso + ((int64_t)n * (K - 1) + (p - Ls)) * a.conv_dim + cg, ds);
#pragma unroll
          for (int e = 0; e < N; ++e) d[e] += ds[e];
        }
        if (ti >= s0)
          stv<N, T>(dx + ti * a.conv_dim + cg, d);
        else if (dsi)
          stv<N, T>(dsi + ((int64_t)n * (K - 1) + p) * a.conv_dim + cg, d);
      }
    }
  };
  // the chunk's first K - 1 tokens, its later ones (fast), then the K - 1 outputs after it
  const int64_t f0 = tok0 + (K - 1), f1 = tok0 + L;
  int64_t t = tok0;
#pragma unroll 1
  for (; t < f0 && t < t_end; ++t) token(t, std::false_type{});
#pragma unroll 4
  for (; t < f1; ++t) token(t, std::true_type{});
#pragma unroll 1
  for (; t < t_end; ++t) token(t, std::false_type{});
  if (a.dw_part) {
    float* dp = a.dw_part + (c * a.conv_dim + cg) * K;
#pragma unroll
    for (int e = 0; e < N; ++e)
#pragma unroll
      for (int m = 0; m < K; ++m) dp[e * K + m] = dw[m][e];
  }
}

// dw[ch][m] = the per-chunk partials summed in a fixed order: a block takes 32 consecutive (ch, m) columns,
// its warp g sums chunks g, g + 8, g + 16, ... in order, then the eight warp sums are added in warp order.
__global__ void __launch_bounds__(256) gdn_conv_dw_sum(const float* part, int64_t n_chunks, int64_t per, float* dw) {
  __shared__ float red[8][32];
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int64_t i = blockIdx.x * (int64_t)32 + lane;
  float s = 0.f;
  if (i < per)
    for (int64_t c = g; c < n_chunks; c += 8) s += part[c * per + i];
  red[g][lane] = s;
  __syncthreads();
  if (g == 0 && i < per) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) t += red[q][lane];
    dw[i] = t;
  }
}

// ------------------------------------------------------------------------------------------------
// Verify rows: V tokens of each of N sequences, x [N, V, conv_dim], as V one-token steps; the conv
// window after each token kept in states [N, V, K - 1, conv_dim].  Grid (N, conv_dim / 2048).
template <int K, typename T>
__global__ void __launch_bounds__(NTC) gdn_conv_verify(ConvArgs a, int V) {
  const int cg = (blockIdx.y * NTC + threadIdx.x) * CV;
  if (cg >= a.conv_dim) return;
  const int n = blockIdx.x;
  float wv[K][CV], xp[K][CV], u[CV], y[CV];
  load_w<K, T, CV>(a, cg, wv);
  load_halo<K, T, CV>(a, n, (int64_t)n * V, (int64_t)n * V, cg, xp);
  const T* x = static_cast<const T*>(a.x);
  T *q = static_cast<T*>(a.q), *k = static_cast<T*>(a.k), *v = static_cast<T*>(a.v);
  T* states = static_cast<T*>(a.state_out);
  for (int j = 0; j < V; ++j) {
    const int64_t t = (int64_t)n * V + j;
    ldv<CV, T>(x + t * a.conv_dim + cg, xp[K - 1]);
    conv_silu<K, T, CV>(xp, wv, u, y);
    stv<CV, T>(route(q, k, v, a, t, cg), y);
    shift<K, CV>(xp);
#pragma unroll
    for (int r = 0; r < K - 1; ++r) stv<CV, T>(states + ((t * (K - 1)) + r) * a.conv_dim + cg, xp[r]);
  }
}

// ------------------------------------------------------------------------------------------------
// Host side.
namespace {

struct ConvPlan {
  int N, conv_dim, key_dim, value_dim;
  int64_t n_chunks;
  bool varlen, has_empty;
};

int check_conv(const qb_gdn_conv_desc* d, ConvPlan* p, const char* what, char* err, int errlen) {
  if (!d) return capi_fail(err, errlen, "%s: null descriptor", what);
  if (d->B < 1 || d->T < 0 || d->Hk < 1 || d->Hv < 1 || d->Dk < 1 || d->Dv < 1)
    return capi_fail(err, errlen, "%s: bad shape (B %d, T %d, Hk %d, Hv %d, Dk %d, Dv %d)", what, d->B, d->T, d->Hk,
                     d->Hv, d->Dk, d->Dv);
  if (d->K < 2 || d->K > 4) return capi_fail(err, errlen, "%s: conv taps K must be 2, 3 or 4 (got %d)", what, d->K);
  if (d->dtype != QB_DTYPE_F32 && d->dtype != QB_DTYPE_BF16)
    return capi_fail(err, errlen, "%s: dtype must be QB_DTYPE_F32 or QB_DTYPE_BF16 (got %d)", what, d->dtype);
  p->key_dim = d->Hk * d->Dk, p->value_dim = d->Hv * d->Dv;
  p->conv_dim = 2 * p->key_dim + p->value_dim;
  if (p->key_dim % CV || p->value_dim % CV)
    return capi_fail(err, errlen, "%s: Hk*Dk and Hv*Dv must be multiples of 8 (got %d, %d)", what, p->key_dim,
                     p->value_dim);
  p->varlen = d->cu_seqlens || d->cu_seqlens_host;
  p->has_empty = false;
  if (p->varlen) {
    if (!d->cu_seqlens || !d->cu_seqlens_host)
      return capi_fail(err, errlen, "%s: varlen needs both cu_seqlens (device) and cu_seqlens_host", what);
    if (d->B != 1 || d->n_seqs < 1) return capi_fail(err, errlen, "%s: varlen needs B == 1 and n_seqs >= 1", what);
    const int32_t* cu = d->cu_seqlens_host;
    if (cu[0] != 0 || cu[d->n_seqs] != d->T)
      return capi_fail(err, errlen, "%s: cu_seqlens must start at 0 and end at T = %d", what, d->T);
    int64_t nc = 0;
    for (int i = 0; i < d->n_seqs; ++i) {
      if (cu[i + 1] < cu[i]) return capi_fail(err, errlen, "%s: cu_seqlens must be non-decreasing", what);
      nc += (cu[i + 1] - cu[i] + kChunk - 1) / kChunk;
      p->has_empty = p->has_empty || cu[i + 1] == cu[i];
    }
    p->N = d->n_seqs, p->n_chunks = nc;
  } else {
    p->N = d->B, p->n_chunks = (int64_t)d->B * ((d->T + kChunk - 1) / kChunk);
  }
  return 0;
}

int64_t a256(int64_t x) { return (x + 255) & ~int64_t(255); }

// workspace: [chunk_off (varlen)][dw partials]
int64_t conv_ws(const ConvPlan& p, int K, bool with_dw, char* base, int64_t** chunk_off, float** part) {
  int64_t off = 0;
  if (chunk_off) *chunk_off = base ? (int64_t*)(base + off) : nullptr;
  off += a256(p.varlen ? (int64_t)(p.N + 1) * 8 : 0);
  if (part) *part = base && with_dw ? (float*)(base + off) : nullptr;
  off += a256(with_dw ? p.n_chunks * p.conv_dim * (int64_t)K * 4 : 0);
  return off < 256 ? 256 : off;
}

template <typename T>
cudaError_t launch_conv(int kind, int K, const ConvArgs& a, dim3 grid, int V, cudaStream_t st) {
#define QB_CONV_CASE(KK)                                                                    \
  case KK:                                                                                  \
    if (kind == 0) gdn_conv_fwd<KK, T><<<grid, NTC, 0, st>>>(a);                            \
    else if (kind == 1) gdn_conv_bwd<KK, T><<<grid, NTC, 0, st>>>(a);                       \
    else gdn_conv_verify<KK, T><<<grid, NTC, 0, st>>>(a, V);                                \
    break;
  switch (K) {
    QB_CONV_CASE(2)
    QB_CONV_CASE(3)
    QB_CONV_CASE(4)
    default:
      return cudaErrorInvalidValue;
  }
#undef QB_CONV_CASE
  note_launch();
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_empty(int K, const ConvPlan& p, const int32_t* cu, const void* src, void* dst, cudaStream_t st) {
  const dim3 grid(p.N, 4);
  switch (K) {
    case 2: gdn_conv_empty<2, T><<<grid, NTC, 0, st>>>(cu, p.conv_dim, (const T*)src, (T*)dst); break;
    case 3: gdn_conv_empty<3, T><<<grid, NTC, 0, st>>>(cu, p.conv_dim, (const T*)src, (T*)dst); break;
    default: gdn_conv_empty<4, T><<<grid, NTC, 0, st>>>(cu, p.conv_dim, (const T*)src, (T*)dst); break;
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t dispatch(int dtype, int kind, int K, const ConvArgs& a, dim3 grid, int V, cudaStream_t st) {
  return dtype == QB_DTYPE_BF16 ? launch_conv<__nv_bfloat16>(kind, K, a, grid, V, st)
                                : launch_conv<float>(kind, K, a, grid, V, st);
}
cudaError_t dispatch_empty(int dtype, int K, const ConvPlan& p, const int32_t* cu, const void* src, void* dst,
                           cudaStream_t st) {
  return dtype == QB_DTYPE_BF16 ? launch_empty<__nv_bfloat16>(K, p, cu, src, dst, st)
                                : launch_empty<float>(K, p, cu, src, dst, st);
}

bool vec_aligned(const void* p) { return !p || capi_aligned(p, 16); }

}  // namespace
}  // namespace qbgdn

using namespace qbgdn;

extern "C" {

int64_t qb_gdn_conv_workspace_bytes(const qb_gdn_conv_desc* d, char* err, int errlen) {
  ConvPlan p;
  if (check_conv(d, &p, "gated delta conv", err, errlen)) return -1;
  return conv_ws(p, d->K, true, nullptr, nullptr, nullptr);
}

int qb_gdn_conv_fwd(const qb_gdn_conv_desc* d, const void* x, const void* w, const void* state_in, void* q, void* k,
                    void* v, void* state_out, void* ws, int64_t ws_bytes, void* stream, char* err, int errlen) {
  ConvPlan p;
  if (check_conv(d, &p, "gated delta conv forward", err, errlen)) return -1;
  if (!x || !w || !q || !k || !v)
    return capi_fail(err, errlen, "gated delta conv forward: x, w, q, k and v must be non-null");
  if (!vec_aligned(x) || !vec_aligned(q) || !vec_aligned(k) || !vec_aligned(v) || !vec_aligned(state_in) ||
      !vec_aligned(state_out))
    return capi_fail(err, errlen, "gated delta conv forward: x, q, k, v and the states need 16-byte alignment");
  const int64_t need = conv_ws(p, d->K, false, nullptr, nullptr, nullptr);
  if (!ws || ws_bytes < need || !capi_aligned(ws, 256))
    return capi_fail(err, errlen, "gated delta conv forward: a 256-byte aligned workspace of %lld bytes is needed",
                     (long long)need);
  cudaStream_t st = (cudaStream_t)stream;
  ConvArgs a{};
  int64_t* chunk_off = nullptr;
  conv_ws(p, d->K, false, (char*)ws, &chunk_off, nullptr);
  a.geo = Geo{d->T, d->Hk, d->Hv, p.N, (d->T + kChunk - 1) / kChunk, d->cu_seqlens, p.varlen ? chunk_off : nullptr};
  a.key_dim = p.key_dim, a.value_dim = p.value_dim, a.conv_dim = p.conv_dim;
  a.x = x, a.w = w, a.state_in = state_in, a.q = q, a.k = k, a.v = v, a.state_out = state_out;
  cudaError_t e;
  if (p.varlen && (e = launch_chunk_offsets(d->cu_seqlens, p.N, chunk_off, st)) != cudaSuccess)
    return capi_cuda(e, "gated delta conv forward", err, errlen);
  if (p.has_empty && state_out &&
      (e = dispatch_empty(d->dtype, d->K, p, d->cu_seqlens, state_in, state_out, st)) != cudaSuccess)
    return capi_cuda(e, "gated delta conv forward", err, errlen);
  if (p.n_chunks == 0) {  // T = 0: the state passes through
    if (state_out) {
      const size_t bytes = (size_t)p.N * (d->K - 1) * p.conv_dim * (d->dtype == QB_DTYPE_BF16 ? 2 : 4);
      e = state_in ? cudaMemcpyAsync(state_out, state_in, bytes, cudaMemcpyDeviceToDevice, st)
                   : cudaMemsetAsync(state_out, 0, bytes, st);
      return capi_cuda(e, "gated delta conv forward", err, errlen);
    }
    return 0;
  }
  const dim3 grid((unsigned)p.n_chunks, (p.conv_dim + NTC * CVF - 1) / (NTC * CVF));
  return capi_cuda(dispatch(d->dtype, 0, d->K, a, grid, 0, st), "gated delta conv forward", err, errlen);
}

int qb_gdn_conv_bwd(const qb_gdn_conv_desc* d, const void* x, const void* w, const void* state_in, const void* dq,
                    const void* dk, const void* dv, const void* dstate_out, void* dx, float* dw, void* dstate_in,
                    void* ws, int64_t ws_bytes, void* stream, char* err, int errlen) {
  ConvPlan p;
  if (check_conv(d, &p, "gated delta conv backward", err, errlen)) return -1;
  if (!x || !w || !dq || !dk || !dv || !dx)
    return capi_fail(err, errlen, "gated delta conv backward: x, w, dq, dk, dv and dx must be non-null");
  if (!vec_aligned(x) || !vec_aligned(dq) || !vec_aligned(dk) || !vec_aligned(dv) || !vec_aligned(dx) ||
      !vec_aligned(state_in) || !vec_aligned(dstate_out) || !vec_aligned(dstate_in))
    return capi_fail(err, errlen, "gated delta conv backward: x, dq, dk, dv, dx and the states need 16-byte alignment");
  const int64_t need = conv_ws(p, d->K, dw != nullptr, nullptr, nullptr, nullptr);
  if (!ws || ws_bytes < need || !capi_aligned(ws, 256))
    return capi_fail(err, errlen, "gated delta conv backward: a 256-byte aligned workspace of %lld bytes is needed",
                     (long long)need);
  cudaStream_t st = (cudaStream_t)stream;
  ConvArgs a{};
  int64_t* chunk_off = nullptr;
  float* part = nullptr;
  conv_ws(p, d->K, dw != nullptr, (char*)ws, &chunk_off, &part);
  a.geo = Geo{d->T, d->Hk, d->Hv, p.N, (d->T + kChunk - 1) / kChunk, d->cu_seqlens, p.varlen ? chunk_off : nullptr};
  a.key_dim = p.key_dim, a.value_dim = p.value_dim, a.conv_dim = p.conv_dim;
  a.x = x, a.w = w, a.state_in = state_in, a.dq = dq, a.dk = dk, a.dv = dv, a.dstate_out = dstate_out;
  a.dx = dx, a.dw_part = part, a.dstate_in = dstate_in;
  cudaError_t e;
  if (p.varlen && (e = launch_chunk_offsets(d->cu_seqlens, p.N, chunk_off, st)) != cudaSuccess)
    return capi_cuda(e, "gated delta conv backward", err, errlen);
  if (p.has_empty && dstate_in &&
      (e = dispatch_empty(d->dtype, d->K, p, d->cu_seqlens, dstate_out, dstate_in, st)) != cudaSuccess)
    return capi_cuda(e, "gated delta conv backward", err, errlen);
  if (p.n_chunks == 0) {
    const size_t bytes = (size_t)p.N * (d->K - 1) * p.conv_dim * (d->dtype == QB_DTYPE_BF16 ? 2 : 4);
    if (dstate_in) {
      e = dstate_out ? cudaMemcpyAsync(dstate_in, dstate_out, bytes, cudaMemcpyDeviceToDevice, st)
                     : cudaMemsetAsync(dstate_in, 0, bytes, st);
      if (e != cudaSuccess) return capi_cuda(e, "gated delta conv backward", err, errlen);
    }
    if (dw) return capi_cuda(cudaMemsetAsync(dw, 0, (size_t)p.conv_dim * d->K * 4, st), "gated delta conv backward",
                             err, errlen);
    return 0;
  }
  const dim3 grid((unsigned)p.n_chunks, (p.conv_dim + NTC * CVB - 1) / (NTC * CVB));
  if ((e = dispatch(d->dtype, 1, d->K, a, grid, 0, st)) != cudaSuccess)
    return capi_cuda(e, "gated delta conv backward", err, errlen);
  if (dw) {
    const int64_t per = (int64_t)p.conv_dim * d->K;
    gdn_conv_dw_sum<<<(unsigned)((per + 31) / 32), 256, 0, st>>>(part, p.n_chunks, per, dw);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return capi_cuda(e, "gated delta conv backward", err, errlen);
  }
  return 0;
}

int qb_gdn_conv_verify(const qb_gdn_conv_desc* d, const void* x, const void* w, const void* state_in, void* q, void* k,
                       void* v, void* states, void* stream, char* err, int errlen) {
  ConvPlan p;
  if (check_conv(d, &p, "gated delta conv verify", err, errlen)) return -1;
  if (p.varlen) return capi_fail(err, errlen, "gated delta conv verify: B sequences of T drafted tokens, no cu_seqlens");
  if (!x || !w || !state_in || !q || !k || !v || !states)
    return capi_fail(err, errlen, "gated delta conv verify: every pointer must be non-null");
  if (!vec_aligned(x) || !vec_aligned(q) || !vec_aligned(k) || !vec_aligned(v) || !vec_aligned(state_in) ||
      !vec_aligned(states))
    return capi_fail(err, errlen, "gated delta conv verify: x, q, k, v and the states need 16-byte alignment");
  if (d->T == 0) return 0;
  ConvArgs a{};
  a.key_dim = p.key_dim, a.value_dim = p.value_dim, a.conv_dim = p.conv_dim;
  a.x = x, a.w = w, a.state_in = state_in, a.q = q, a.k = k, a.v = v, a.state_out = states;
  const dim3 grid(p.N, (p.conv_dim + NTC * CV - 1) / (NTC * CV));
  return capi_cuda(dispatch(d->dtype, 2, d->K, a, grid, d->T, (cudaStream_t)stream), "gated delta conv verify", err,
                   errlen);
}

int qb_gdn_keep_conv_rows(int32_t N, int32_t V, int32_t K, int32_t conv_dim, int32_t dtype, const void* states,
                          const int32_t* keep, void* state_out, int32_t* status, void* stream, char* err, int errlen) {
  if (N < 0 || V < 1 || K < 2 || K > 4 || conv_dim < 1 || conv_dim % CV || (dtype != QB_DTYPE_F32 && dtype != QB_DTYPE_BF16))
    return capi_fail(err, errlen, "gated delta keep_conv_rows: bad arguments (N %d, V %d, K %d, conv_dim %d, dtype %d)",
                     N, V, K, conv_dim, dtype);
  if (!states || !keep || !state_out) return capi_fail(err, errlen, "gated delta keep_conv_rows: null pointer");
  if (!capi_aligned(states, 16) || !capi_aligned(state_out, 16))
    return capi_fail(err, errlen, "gated delta keep_conv_rows: the states need 16-byte alignment");
  if (N == 0) return 0;
  // the rows are copied as raw 16-byte words: (K - 1) conv_dim elements per row, a multiple of 16 bytes
  const int64_t words = (int64_t)(K - 1) * conv_dim * (dtype == QB_DTYPE_BF16 ? 2 : 4) / 4;
  return capi_cuda(launch_keep_rows(N, V, words, (const float*)states, keep, (float*)state_out, status,
                                    (cudaStream_t)stream),
                   "gated delta keep_conv_rows", err, errlen);
}

}  // extern "C"
