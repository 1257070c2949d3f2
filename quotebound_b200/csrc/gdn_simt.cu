// Row-parallel (SIMT) kernels of the Gated DeltaNet recurrence, for any Dk in {32, 64, 128, 256}
// and any Dv.  One warp owns one state row S[r, :] of one (sequence, value head); lane l holds the
// Dk/32 columns [l*NPT, l*NPT + NPT).
//
//  * gdn_seq_fwd     — the forward over T steps (the generic path of qb_gdn_fwd, and the kernel
//                      whose rounding the one-token step and the verify rows reproduce bit for bit).
//  * gdn_step        — one decode token (qb_gdn_step).
//  * gdn_verify      — V tokens run as V steps, every row's state kept (qb_gdn_verify).
// The generic backward is the CUDA-core chunked one of gdn_cc.cu.
#include "gdn_common.cuh"
#include "gdn_simt.cuh"
#include "launch_count.cuh"

namespace qbgdn {

struct SeqRange {
  int64_t b, t0, t1;
};

__device__ __forceinline__ SeqRange seq_range(const int32_t* cu, int n, int T) {
  if (cu) return {0, cu[n], cu[n + 1]};
  return {n, 0, T};
}

// ------------------------------------------------------------------------------------------------
template <int NPT, typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gdn_seq_fwd(SimtArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = blockIdx.x * a.rows_per_block + warp;
  const int hv = blockIdx.y, n = blockIdx.z;
  if (r >= a.Dv) return;
  const int hk = hv / (a.Hv / a.Hk);
  const SeqRange sr = seq_range(a.cu, n, a.T);
  const Tin* __restrict__ q = static_cast<const Tin*>(a.q);
  const Tin* __restrict__ k = static_cast<const Tin*>(a.k);
  const Tin* __restrict__ v = static_cast<const Tin*>(a.v);
  Tout* __restrict__ y = static_cast<Tout*>(a.y);
  const int c0 = lane * NPT;
  const size_t srow = ((size_t)n * a.Hv + hv) * a.Dv + r;
  float s[NPT];
  if (a.h0) {
    load_vec<NPT>(a.h0 + srow * a.Dk + c0, s);
  } else {
#pragma unroll
    for (int i = 0; i < NPT; ++i) s[i] = 0.f;
  }
  const int64_t chunk_base = a.chunk_off ? a.chunk_off[n] : (int64_t)n * ((a.T + kChunk - 1) / kChunk);
  for (int64_t t = sr.t0; t < sr.t1; ++t) {
    if (a.ckpt && ((t - sr.t0) % kChunk) == 0) {
      const int64_t c = chunk_base + (t - sr.t0) / kChunk;
      store_vec<NPT>(a.ckpt + ((c * a.Hv + hv) * a.Dv + r) * (size_t)a.Dk + c0, s);
    }
    const size_t tok = (size_t)sr.b * a.T + t;
    float kk[NPT], qq[NPT];
    load_vec<NPT>(k + (tok * a.Hk + hk) * a.Dk + c0, kk);
    load_vec<NPT>(q + (tok * a.Hk + hk) * a.Dk + c0, qq);
    const size_t gb = tok * a.Hv + hv;
    const float vt = to_f(v[gb * a.Dv + r]);
    const float o = row_step<NPT>(s, kk, qq, vt, a.g[gb], a.beta[gb]);
    if (lane == 0) y[gb * a.Dv + r] = from_f<Tout>(o);
  }
  if (a.hT) store_vec<NPT>(a.hT + srow * a.Dk + c0, s);
}

// One token for N sequences; N plays the role of the sequence index, T = 1.
template <int NPT, typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gdn_step(SimtArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = blockIdx.x * a.rows_per_block + warp;
  const int hv = blockIdx.y, n = blockIdx.z;
  if (r >= a.Dv) return;
  const int hk = hv / (a.Hv / a.Hk);
  const int c0 = lane * NPT;
  const size_t srow = ((size_t)n * a.Hv + hv) * a.Dv + r;
  float s[NPT], kk[NPT], qq[NPT];
  load_vec<NPT>(a.h0 + srow * a.Dk + c0, s);
  load_vec<NPT>(static_cast<const Tin*>(a.k) + ((size_t)n * a.Hk + hk) * a.Dk + c0, kk);
  load_vec<NPT>(static_cast<const Tin*>(a.q) + ((size_t)n * a.Hk + hk) * a.Dk + c0, qq);
  const size_t gb = (size_t)n * a.Hv + hv;
  const float vt = to_f(static_cast<const Tin*>(a.v)[gb * a.Dv + r]);
  const float o = row_step<NPT>(s, kk, qq, vt, a.g[gb], a.beta[gb]);
  if (lane == 0) static_cast<Tout*>(a.y)[gb * a.Dv + r] = from_f<Tout>(o);
  store_vec<NPT>(a.hT + srow * a.Dk + c0, s);
}

// V tokens of N sequences, inputs [N, V, ...]; the state after token j goes to states[n, j].
template <int NPT, typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gdn_verify(SimtArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = blockIdx.x * a.rows_per_block + warp;
  const int hv = blockIdx.y, n = blockIdx.z;
  if (r >= a.Dv) return;
  const int hk = hv / (a.Hv / a.Hk);
  const int c0 = lane * NPT;
  const int V = a.T;
  float s[NPT];
  load_vec<NPT>(a.h0 + (((size_t)n * a.Hv + hv) * a.Dv + r) * a.Dk + c0, s);
  for (int j = 0; j < V; ++j) {
    const size_t tok = (size_t)n * V + j;
    float kk[NPT], qq[NPT];
    load_vec<NPT>(static_cast<const Tin*>(a.k) + (tok * a.Hk + hk) * a.Dk + c0, kk);
    load_vec<NPT>(static_cast<const Tin*>(a.q) + (tok * a.Hk + hk) * a.Dk + c0, qq);
    const size_t gb = tok * a.Hv + hv;
    const float vt = to_f(static_cast<const Tin*>(a.v)[gb * a.Dv + r]);
    const float o = row_step<NPT>(s, kk, qq, vt, a.g[gb], a.beta[gb]);
    if (lane == 0) static_cast<Tout*>(a.y)[gb * a.Dv + r] = from_f<Tout>(o);
    store_vec<NPT>(a.ckpt + ((tok * a.Hv + hv) * a.Dv + r) * (size_t)a.Dk + c0, s);
  }
}

// chunk_off[n] = sum over sequences m < n of ceil(len_m / 64); one thread (n is small).
__global__ void gdn_chunk_offsets(const int32_t* cu, int N, int64_t* chunk_off) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    int64_t acc = 0;
    for (int n = 0; n < N; ++n) {
      chunk_off[n] = acc;
      acc += (cu[n + 1] - cu[n] + kChunk - 1) / kChunk;
    }
    chunk_off[N] = acc;
  }
}

// keep_rows (src/exact.cpp:151-159): state_out[n] = states[n, keep[n] - 1], float4 copies.
__global__ void gdn_keep_rows(int V, int64_t E4, const float4* __restrict__ states, const int32_t* __restrict__ keep,
                              float4* __restrict__ out, int32_t* status) {
  const int n = blockIdx.y;
  const int kn = keep[n];
  if (kn < 1 || kn > V) {
    if (status && blockIdx.x == 0 && threadIdx.x == 0) status[0] = 1;
    return;
  }
  const float4* src = states + ((int64_t)n * V + (kn - 1)) * E4;
  float4* dst = out + (int64_t)n * E4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < E4; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// ------------------------------------------------------------------------------------------------
// Host-side launchers (called by the C ABI after validation).
template <int NPT, typename Tin, typename Tout>
static cudaError_t launch_kind(SimtKind kind, const SimtArgs& a, dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st) {
  switch (kind) {
    case SimtKind::Fwd:
      gdn_seq_fwd<NPT, Tin, Tout><<<grid, block, 0, st>>>(a);
      note_launch();
      break;
    case SimtKind::Step:
      gdn_step<NPT, Tin, Tout><<<grid, block, 0, st>>>(a);
      note_launch();
      break;
    case SimtKind::Verify:
      gdn_verify<NPT, Tin, Tout><<<grid, block, 0, st>>>(a);
      note_launch();
      break;
  }
  return cudaGetLastError();
}

template <typename Tin, typename Tout>
static cudaError_t launch_npt(SimtKind kind, const SimtArgs& a, dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st) {
  switch (a.Dk / 32) {
    case 1: return launch_kind<1, Tin, Tout>(kind, a, grid, block, smem, st);
    case 2: return launch_kind<2, Tin, Tout>(kind, a, grid, block, smem, st);
    case 4: return launch_kind<4, Tin, Tout>(kind, a, grid, block, smem, st);
    case 8: return launch_kind<8, Tin, Tout>(kind, a, grid, block, smem, st);
  }
  return cudaErrorInvalidValue;
}

int simt_rows_per_block(int Dv) {
  int r = 8;
  while (r > 1 && Dv % r) r /= 2;
  return r;
}

cudaError_t simt_launch(SimtKind kind, const SimtArgs& a, int n_seqs, int in_bf16, int out_bf16,
                        cudaStream_t st) {
  const int RPB = a.rows_per_block;
  dim3 grid((a.Dv + RPB - 1) / RPB, a.Hv, n_seqs), block(32 * RPB);
  const size_t smem = 0;
  if (in_bf16 && out_bf16) return launch_npt<__nv_bfloat16, __nv_bfloat16>(kind, a, grid, block, smem, st);
  if (in_bf16) return launch_npt<__nv_bfloat16, float>(kind, a, grid, block, smem, st);
  if (out_bf16) return launch_npt<float, __nv_bfloat16>(kind, a, grid, block, smem, st);
  return launch_npt<float, float>(kind, a, grid, block, smem, st);
}

cudaError_t launch_chunk_offsets(const int32_t* cu, int N, int64_t* chunk_off, cudaStream_t st) {
  gdn_chunk_offsets<<<1, 32, 0, st>>>(cu, N, chunk_off);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_keep_rows(int N, int V, int64_t per_seq, const float* states, const int32_t* keep, float* out,
                             int32_t* status, cudaStream_t st) {
  const int64_t E4 = per_seq / 4;
  const unsigned bx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((E4 + 255) / 256, 64));
  gdn_keep_rows<<<dim3(bx, N), 256, 0, st>>>(V, E4, reinterpret_cast<const float4*>(states), keep,
                                             reinterpret_cast<float4*>(out), status);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
