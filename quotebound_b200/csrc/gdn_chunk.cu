// Tensor-core chunked path of the Gated DeltaNet recurrence (Dk = Dv = 128, bf16 activations),
// sm_100a: TMA tile loads, tcgen05 MMAs with TMEM accumulators, chunk C = 64.
//
// Per value head and chunk (local steps i, j < C; b = inclusive cumsum of log g inside the chunk,
// gamma = exp(b), Gamma_ij = exp(b_i - b_j), lambda_i = exp(b_C - b_i); rows past the sequence end
// carry beta = 0, log g = 0 and zero v / dy):
//   L  = strict-lower(beta_i Gamma_ij (K K^T)_ij),   T = (I + L)^-1
//   P  = lower(Gamma_ij (Q K^T)_ij)
//   E  = diag(beta) (V - diag(gamma) K S^T)                  (S: the chunk-start state, Dv x Dk)
//   D  = T E                                                  (the chunk's delta rows)
//   O  = diag(gamma) Q S^T + P D
//   S' = gamma_C S + (diag(lambda) D)^T K
// the recurrence of src/delta_grad.cpp:13-14 (S~ = g S; u = S~ k; delta = beta (v - u);
// S = S~ + delta k^T; y = S q) over 64 steps at once (the WY / UT form).  Its backward, with dS the
// cotangent of S' and dO that of O:
//   dD  = P^T dO + diag(lambda) K dS^T,   F = T^T dD
//   dS_start = gamma_C dS + (diag(gamma) dO)^T Q - (diag(beta gamma) F)^T K,   dV = diag(beta) F
//   dQ  = diag(gamma) dO S + dP^ K,   dP^ = lower(Gamma (dO D^T))
//   dK  = dP^^T Q + diag(lambda) D dS - diag(beta gamma) F S + dKK K + dKK^T K,
//         dKK = strict-lower(beta_i Gamma_ij (-F D^T)_ij)
//   d b_i (log-gate cumsum) from every Gamma, gamma and lambda above; d log g = reverse cumsum of d b.
//
// Kernels:
//   gdn_chunk_prep       (chunks, Hk): K K^T and Q K^T on the tensor cores, then per value head of the
//                        key head T by forward substitution; writes the T, P and [K; Q] operand images
//                        and the gates.  Fully parallel.
//   gdn_chunk_fwd_state  (Dv/32, Hv, sequences): the chunks of a sequence in order, 32 state rows in
//                        registers; three tcgen05 rounds per chunk (K S^T, Q S^T | T E | P D, K^T D~).
//                        Writes y and, for training, the chunk-start states.
//   gdn_chunk_bwd_state  (Dv/32, Hv, sequences): the chunks in reverse with 32 rows of dS; three rounds
//                        (K dS^T, P^T dO | T^T dD | Q^T (gamma dO), K^T H).  Writes dv, dS per chunk, dh0.
//   gdn_chunk_bwd_grad   (chunks, Hk): everything else per chunk, the value heads of a key head in turn
//                        so dq and dk are summed over the group in TMEM in a fixed order; K K^T is
//                        recomputed there from the [K; Q] image (one MMA per CTA).
// Operand precision: input x input products in bf16 (exact); input x computed with the computed tile
// split into bf16 hi + lo (about 16 mantissa bits); computed x computed in tf32 (round to nearest).
#include <cuda.h>
#include <cuda_bf16.h>

#include "gdn_chunk.cuh"
#include "gdn_common.cuh"
#include "gdn_simt.cuh"
#include "launch_count.cuh"
#include "tc_sm100.cuh"

namespace qbgdn {

namespace {

constexpr int C = kChunk;   // 64
constexpr int DK = 128;
constexpr int DV = 128;
constexpr int DVT = 32;     // value rows of the state per CTA in the walks; the dv slice in the gradient kernel

// fp32 to the nearest tf32 (10 mantissa bits), ties away from zero: add half of the 13 dropped bits'
// weight to the bit pattern and clear them (a carry into the exponent is the correct rounding up;
// infinities keep their pattern).
__device__ __forceinline__ float tf32_rna(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

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
    tok0 = (int64_t)n * g.T + (int64_t)j * C;
    L = min(C, g.T - j * C);
    return;
  }
  int lo = 0, hi = g.N - 1;  // last n with chunk_off[n] <= c
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.chunk_off[mid] <= c) lo = mid; else hi = mid - 1;
  }
  n = lo;
  tok0 = g.cu[n] + (c - g.chunk_off[n]) * C;
  L = (int)min((int64_t)C, (int64_t)g.cu[n + 1] - tok0);
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

// Inclusive prefix sum over 64 values held by threads 0..63 (warps 0 and 1); result in out[64].
__device__ __forceinline__ void scan64(float x, float* out, float* tmp) {
  const int tid = threadIdx.x, lane = tid & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (tid == 31) tmp[0] = x;
  __syncthreads();
  if (tid >= 32 && tid < 64) x += tmp[0];
  if (tid < 64) out[tid] = x;
}

template <typename Tout>
__device__ __forceinline__ void store_row32(Tout* p, const float (&v)[32]);
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(p + 8 * q) =
        make_uint4(tc::pack_bf16(v[8 * q], v[8 * q + 1]), tc::pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                   tc::pack_bf16(v[8 * q + 4], v[8 * q + 5]), tc::pack_bf16(v[8 * q + 6], v[8 * q + 7]));
}
template <>
__device__ __forceinline__ void store_row32<float>(float* p, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) *reinterpret_cast<float4*>(p + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// 16-wide versions (half of a 32-column slice).
struct Row16 {
  uint4 w[2];
};
__device__ __forceinline__ void cvt_row16(const Row16& r, float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint32_t w[4] = {r.w[q].x, r.w[q].y, r.w[q].z, r.w[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
      v[8 * q + 2 * e] = __low2float(h);
      v[8 * q + 2 * e + 1] = __high2float(h);
    }
  }
}
template <typename Tout>
__device__ __forceinline__ void store_row16(Tout* p, const float (&v)[16]);
template <>
__device__ __forceinline__ void store_row16<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q)
    *reinterpret_cast<uint4*>(p + 8 * q) =
        make_uint4(tc::pack_bf16(v[8 * q], v[8 * q + 1]), tc::pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                   tc::pack_bf16(v[8 * q + 4], v[8 * q + 5]), tc::pack_bf16(v[8 * q + 6], v[8 * q + 7]));
}
template <>
__device__ __forceinline__ void store_row16<float>(float* p, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) *reinterpret_cast<float4*>(p + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

__device__ __forceinline__ float softplus_f(float x) { return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x))); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

// Row of chunk row i (0..63) in a stacked [hi; lo] operand image of 128 rows: groups of 16 rows
// alternate hi, lo, so that an M = 128 accumulator holds row i's hi product in lane 32w + l and its lo
// product in lane 32w + 16 + l (i = 16w + l), the lanes of one warp.
__device__ __forceinline__ int img_row(int i) { return 32 * (i >> 4) + (i & 15); }

__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity, int* err, int code) {
  return __syncthreads_and(tc::mbar_wait(bar, parity, err, code)) != 0;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Per (chunk, key head): the [K; Q] image; per value head of the group T, P and the gates of the chunk.
struct PrepArgs {
  Geo geo;
  const float *g, *beta;
  // layer mode (g, beta null): the raw gate inputs and the raw q, k rows normalised here
  const float *a_raw, *b_raw, *A_log, *dt_bias;
  uint8_t* Timg;    // [chunks, Hv] x 16 KB: T as the stacked bf16 [T_hi; T_lo] operand image
  uint8_t* Pimg;    // [chunks, Hv] x 16 KB: P likewise
  uint8_t* KQimg;   // [chunks, Hk] x 32 KB: the walk's [K; Q] operand (16-row groups interleaved)
  float* gates;     // [chunks, Hv, 2, 64]:  b then beta
  int* err;
};

__global__ void __launch_bounds__(128, 4) gdn_chunk_prep(const __grid_constant__ CUtensorMap kmap,
                                                      const __grid_constant__ CUtensorMap qmap, PrepArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // 32 KB in all, so that several CTAs share an SM: the K and Q tiles, then (once the products have
  // read them) T transposed in the K tile and L transposed, then L10 T00, in the Q tile
  uint8_t* ktile = smem;                                   // 16 KB bf16
  uint8_t* qtile = smem + 16384;                           // 16 KB bf16
  __shared__ float sb[64], sbeta[64], stmp[2];
  __shared__ __align__(16) float sX[2][16][16];  // the inverse's 16 x 16 intermediate products
  __shared__ uint64_t bar_tma, bar_mma;
  __shared__ uint32_t tmem_slot;
  constexpr int LS = 64;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t c = blockIdx.x;
  const int hk = blockIdx.y, ratio = a.geo.Hv / a.geo.Hk;
  int n, L;
  int64_t tok0;
  chunk_info(a.geo, c, n, tok0, L);

  if (warp == 0) tc::tmem_alloc(&tmem_slot, 64);
  if (tid == 0) {
    tc::mbar_init(&bar_tma, 1);
    tc::mbar_init(&bar_mma, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  if (tid == 0) {
    tc::mbar_arrive_expect_tx(&bar_tma, 32768);
    tc::tma_load_3d(ktile, &kmap, &bar_tma, 0, hk, (int)tok0);
    tc::tma_load_3d(ktile + 8192, &kmap, &bar_tma, 64, hk, (int)tok0);
    tc::tma_load_3d(qtile, &qmap, &bar_tma, 0, hk, (int)tok0);
    tc::tma_load_3d(qtile + 8192, &qmap, &bar_tma, 64, hk, (int)tok0);
  }
  const bool layer = a.g == nullptr;
  // a value head's raw gate inputs (loaded one head ahead, so that their latency hides behind the
  // previous head's work), then log g and beta from them
  auto gate_load = [&](int hv, float (&gr)[4]) {
    gr[0] = gr[1] = gr[2] = gr[3] = 0.f;
    if (tid < 64 && tid < L) {
      const int64_t gi = (tok0 + tid) * a.geo.Hv + hv;
      if (layer) {
        gr[0] = a.a_raw[gi], gr[1] = a.b_raw[gi], gr[2] = a.A_log[hv], gr[3] = a.dt_bias[hv];
      } else {
        gr[0] = a.g[gi], gr[1] = a.beta[gi];
      }
    }
  };
  auto gate_eval = [&](const float (&gr)[4], float& lg, float& bt) {
    lg = 0.f, bt = 0.f;
    if (tid < 64 && tid < L) {
      if (layer) {  // log g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (src/deltanet.cpp:22-33, :99)
        lg = -expf(gr[2]) * softplus_f(gr[0] + gr[3]);
        bt = sigmoid_f(gr[1]);
      } else {
        lg = fmaxf(logf(gr[0]), -88.f);
        bt = gr[1];
      }
    }
  };
  float gr[4];
  gate_load(hk * ratio, gr);

  bool ok = wait_all(&bar_tma, 0, a.err, 1);
  if (ok && layer) {
    // q and k rows normalised in place as the model does (src/deltanet.cpp:94-97): rms_norm in fp32,
    // rounded to bf16, times the bf16 scalar 1/Dk (q) or 1/sqrt(Dk) (k), rounded again.  Thread t
    // owns half a row (one 128-byte slab row of 64 elements); the order inside a row does not matter,
    // so step c touches chunk c ^ (row & 7): eight consecutive rows then hit eight different banks.
    const int row = tid >> 1, half = tid & 1, rx = row & 7;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      uint8_t* tile = m == 0 ? ktile : qtile;
      uint4* r16 = reinterpret_cast<uint4*>(tile + half * 8192 + row * 128);
      uint4 w[8];
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        w[c] = r16[c ^ rx];
        const uint32_t u[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
          ss = fmaf(__low2float(h), __low2float(h), ss);
          ss = fmaf(__high2float(h), __high2float(h), ss);
        }
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float r = rsqrtf(ss / DK + 1e-6f);
      const float sc = m == 0 ? __bfloat162float(__float2bfloat16_rn(rsqrtf((float)DK))) : 1.f / DK;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t u[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
          const float x0 = __bfloat162float(__float2bfloat16_rn(__low2float(h) * r)) * sc;
          const float x1 = __bfloat162float(__float2bfloat16_rn(__high2float(h) * r)) * sc;
          u[e] = tc::pack_bf16(x0, x1);
        }
        r16[c ^ rx] = make_uint4(u[0], u[1], u[2], u[3]);
      }
    }
    tc::fence_async_smem();
    __syncthreads();
  }
  if (ok && tid == 0) {
    tc::fence_after_sync();
    const uint32_t kt = tc::smem_u32(ktile), qt = tc::smem_u32(qtile);
    // K K^T into the lower half-lanes and Q K^T into the upper half-lanes of the same 64 columns, so
    // that all 128 threads own one row of one product
    tc::mma_tile<tc::kBF16>(tmem, kt, false, 64, kt, false, 64, 64, 64, DK, false);
    tc::mma_tile<tc::kBF16>(tmem + (16u << 16), qt, false, 64, kt, false, 64, 64, 64, DK, false);
    tc::mma_commit(&bar_mma);
  }
  if (ok) {
    // the [K; Q] image of this chunk and key head: per 64-column slab, 2 KB row groups K 0-15, Q 0-15,
    // K 16-31, ... (the swizzle is address-relative within 1 KB, so whole groups move unchanged)
    uint4* dst = reinterpret_cast<uint4*>(a.KQimg + (size_t)(c * a.geo.Hk + hk) * 32768);
#pragma unroll 4
    for (int u = 0; u < 16; ++u) {
      const int idx = tid + 128 * u, o = idx * 16;
      const int sl = o >> 14, g = (o >> 12) & 3, part = (o >> 11) & 1, rem = o & 2047;
      dst[idx] = *reinterpret_cast<const uint4*>((part ? qtile : ktile) + sl * 8192 + g * 2048 + rem);
    }
  }
  ok = __syncthreads_and(ok && tc::mbar_wait(&bar_mma, 0, a.err, 2)) != 0;
  tc::fence_after_sync();
  // The products are the same for every value head of the key head; the gates are not.  Each value
  // head in turn: its gated L and P, T, the images.
  for (int r = 0; r < ratio && ok; ++r) {
  const int hv = hk * ratio + r;
  float lg, bt;
  gate_eval(gr, lg, bt);
  if (r + 1 < ratio) gate_load(hv + 1, gr);
  if (tid < 64) sbeta[tid] = bt;
  scan64(lg, sb, stmp);
  __syncthreads();
  const size_t mat = (size_t)(c * a.geo.Hv + hv) * 4096;
  // the images go straight to global memory, 16-byte chunks in the tile's swizzled order
  uint8_t* pimg = a.Pimg + mat * 4;
  float* Lm = reinterpret_cast<float*>(qtile);  // free once the products above completed
  float* Lt = Lm;  // transposed: Lt[j * LS + i] = beta_i Gamma_ij (K K^T)_ij for j < i
  if (ok) {
    const int i = 16 * warp + (lane & 15);
    const bool kkside = lane < 16;  // lower lanes: K K^T row i; upper lanes: Q K^T row i
    const float bi = sb[i], be = sbeta[i];
    float v[32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, 32 * h), v);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int j = 32 * h + jj;
        const float gam = __expf(bi - sb[j]);  // Gamma_ij (only j <= i is used)
        v[jj] = (kkside ? j < i : j <= i) ? gam * v[jj] : 0.f;
      }
      // one instruction stream for the lane pair: the K K^T lane writes columns 0-15 of L and of P, the
      // Q K^T lane columns 16-31 of both (each sends the other the half it does not write)
      float x[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) x[jj] = __shfl_xor_sync(0xffffffffu, kkside ? v[16 + jj] : v[jj], 16);
      const int c0 = kkside ? 0 : 16;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) Lt[(32 * h + c0 + jj) * LS + i] = be * (kkside ? v[jj] : x[jj]);
      {
        const int r = img_row(i);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int jj = 8 * cc + 2 * e;
            const float p0 = kkside ? x[jj] : v[16 + jj], p1 = kkside ? x[jj + 1] : v[17 + jj];
            const __nv_bfloat162 hh = __floats2bfloat162_rn(p0, p1);
            hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
            lw[e] = tc::pack_bf16(p0 - __low2float(hh), p1 - __high2float(hh));
          }
          const int off = r * 128 + (((4 * h + (kkside ? 0 : 2) + cc) ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(pimg + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(pimg + 2048 + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  // T = (I + L)^-1 in 2 x 2 blocks of 32, each 32 x 32 diagonal block itself in 2 x 2 blocks of 16:
  // the four 16 x 16 diagonal blocks A_b = (I + L_bb)^-1 by column sweep (thread (b, c) < 64 owns column
  // c of A_b in registers: t_j is final once the columns before it have been swept, and sweeping column
  // j updates the rows below it independently), then C = -A_(2m+1) (L_(2m+1, 2m) A_2m) completes the
  // 32 x 32 block T_mm, then T10 = -T11 (L10 T00) as two 32 x 32 products over all 128 threads.
  // Tt[col * 64 + row] holds T transposed (in the K tile, free now).
  float* Tt = reinterpret_cast<float*>(ktile);
  if (ok && tid < 64) {
    const int b = tid >> 4, cc = tid & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = i == cc ? 1.f : 0.f;
#pragma unroll
    for (int j = 0; j < 15; ++j) {
      const float tj = t[j];
      const float* Lj = Lt + (16 * b + j) * LS + 16 * b;
#pragma unroll
      for (int i4 = (j + 1) & ~3; i4 < 16; i4 += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(Lj + i4);
        if (i4 + 0 > j) t[i4 + 0] = fmaf(-l4.x, tj, t[i4 + 0]);
        if (i4 + 1 > j) t[i4 + 1] = fmaf(-l4.y, tj, t[i4 + 1]);
        if (i4 + 2 > j) t[i4 + 2] = fmaf(-l4.z, tj, t[i4 + 2]);
        t[i4 + 3] = fmaf(-l4.w, tj, t[i4 + 3]);
      }
    }
    // column 16 b + cc: rows 16 b .. + 15 are A_b's column; for odd b the rows 16 (b - 1) .. + 15 above
    // it in the same 32 x 32 block are zero, and for b >= 2 so are rows 0 .. 31 (T01 = 0)
    float* col = Tt + (16 * b + cc) * 64;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<float4*>(col + 16 * b)[q] = make_float4(t[4 * q], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
    if (b & 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) reinterpret_cast<float4*>(col + 16 * (b - 1))[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (b >= 2) {
#pragma unroll
      for (int q = 0; q < 8; ++q) reinterpret_cast<float4*>(col)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float* gd = a.gates + (c * a.geo.Hv + hv) * 128;
    gd[tid] = sb[tid];
    gd[64 + tid] = sbeta[tid];
  }
  __syncthreads();
  {
    // thread (m, r, cg): row r of the 16 x 16 off-diagonal block of T_mm, columns 4 cg .. 4 cg + 3
    const int m = tid >> 6, r = tid & 15, cg = (tid >> 4) & 3, o = 32 * m;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {  // X' = L_(2m+1, 2m) A_2m  (A_2m[k][c] = 0 for k < c)
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float l = Lt[(o + k) * LS + o + 16 + r];  // L[o + 16 + r][o + k]
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = fmaf(l, Tt[(o + 4 * cg + e) * 64 + o + k], x[e]);
      }
      reinterpret_cast<float4*>(sX[m][r])[cg] = make_float4(x[0], x[1], x[2], x[3]);
    }
    __syncthreads();
    if (ok) {  // C = -A_(2m+1) X'  (A_(2m+1)[r][k] = 0 for k > r)
      float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float ak = Tt[(o + 16 + k) * 64 + o + 16 + r];
        const float4 xk = reinterpret_cast<const float4*>(sX[m][k])[cg];
        y[0] = fmaf(-ak, xk.x, y[0]);
        y[1] = fmaf(-ak, xk.y, y[1]);
        y[2] = fmaf(-ak, xk.z, y[2]);
        y[3] = fmaf(-ak, xk.w, y[3]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) Tt[(o + 4 * cg + e) * 64 + o + 16 + r] = y[e];
    }
  }
  __syncthreads();
  float* Xs = Lm;  // X = L10 T00 [32][32], where L was (once the products have read it)
  {
    const int r = tid & 31, cg = tid >> 5;  // row r of the block, columns 8 cg .. 8 cg + 7
    float x[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) x[q] = 0.f;
    if (ok) {
#pragma unroll 2
      for (int k4 = 0; k4 < 8; ++k4) {
        float l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) l[e] = Lt[(4 * k4 + e) * LS + 32 + r];  // L[32 + r][k]
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 tq = *reinterpret_cast<const float4*>(Tt + (8 * cg + q) * 64 + 4 * k4);  // T00[k][c]
          x[q] = fmaf(l[0], tq.x, fmaf(l[1], tq.y, fmaf(l[2], tq.z, fmaf(l[3], tq.w, x[q]))));
        }
      }
    }
    __syncthreads();
    reinterpret_cast<float4*>(Xs + r * 32 + 8 * cg)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(Xs + r * 32 + 8 * cg)[1] = make_float4(x[4], x[5], x[6], x[7]);
    __syncthreads();
    float y[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) y[q] = 0.f;
    if (ok) {
#pragma unroll 4
      for (int k = 0; k < 32; ++k) {
        const float tk = Tt[(32 + k) * 64 + 32 + r];  // T11[r][k] (zero for k > r)
        const float4 x0 = reinterpret_cast<const float4*>(Xs + k * 32 + 8 * cg)[0];
        const float4 x1 = reinterpret_cast<const float4*>(Xs + k * 32 + 8 * cg)[1];
        y[0] = fmaf(-tk, x0.x, y[0]);
        y[1] = fmaf(-tk, x0.y, y[1]);
        y[2] = fmaf(-tk, x0.z, y[2]);
        y[3] = fmaf(-tk, x0.w, y[3]);
        y[4] = fmaf(-tk, x1.x, y[4]);
        y[5] = fmaf(-tk, x1.y, y[5]);
        y[6] = fmaf(-tk, x1.z, y[6]);
        y[7] = fmaf(-tk, x1.w, y[7]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) Tt[(8 * cg + q) * 64 + 32 + r] = y[q];  // T10[r][c]
    }
  }
  __syncthreads();
  // the T image: thread (row i, half) converts columns 32 half .. + 31 of row i
  if (ok) {
    const int i = tid & 63, h = tid >> 6;
    float v[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) v[jj] = Tt[(32 * h + jj) * 64 + i];
    uint8_t* timg = a.Timg + mat * 4;
    tc::st_row_bf16x2_32(timg, timg + 2048, img_row(i), v, 4 * h);
  }
  __syncthreads();  // the shared buffers and the gate scan are reused by the next value head
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------------------------------------------
// 8 floats as the bf16 [hi | lo] pair of a 128-byte-swizzled operand row r: hi into chunk hc, lo into
// chunk hc + 4 (columns 8 (hc & 3) .. + 7 of each 32-wide half).
__device__ __forceinline__ void st_hilo8(uint8_t* tile, int r, const float (&v)[8], int hc) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    h[e] = *reinterpret_cast<const uint32_t*>(&hh);
    l[e] = tc::pack_bf16(v[2 * e] - __low2float(hh), v[2 * e + 1] - __high2float(hh));
  }
  uint8_t* row = tile + r * 128;
  *reinterpret_cast<uint4*>(row + ((hc ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(row + (((hc + 4) ^ (r & 7)) << 4)) = make_uint4(l[0], l[1], l[2], l[3]);
}
// 8 floats into 16-byte chunks q0, q0 + 1 of row r of a 128-byte-row fp32 tile swizzled by r & 7.
__device__ __forceinline__ void st8_f32_sw(uint8_t* tile, int r, int q0, const float (&v)[8]) {
#pragma unroll
  for (int q = 0; q < 2; ++q)
    *reinterpret_cast<float4*>(tile + r * 128 + (((q0 + q) ^ (r & 7)) << 4)) =
        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}
template <typename Tout>
__device__ __forceinline__ void store_row8(Tout* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store_row8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]),
                                            tc::pack_bf16(v[4], v[5]), tc::pack_bf16(v[6], v[7]));
}
template <>
__device__ __forceinline__ void store_row8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// The forward state walk.  One CTA per (32 value rows, value head, sequence); thread t holds column t
// of the 32 state rows (S^T[t][0..31]) in registers.
struct StateArgs {
  Geo geo;
  const void* v;          // [B*T, Hv, Dv] bf16
  const float* gates;     // [chunks, Hv, 2, 64]
  const float* h0;        // [N, Hv, Dv, Dk] or null
  void* y;                // [B*T, Hv, Dv]
  float* hT;              // or null
  float* ckpt;            // [chunks, Hv, Dv, Dk] chunk-start states, or null
  const uint8_t* Timg;    // [chunks, Hv] x 16 KB operand images from the prep
  const uint8_t* Pimg;
  const uint8_t* KQimg;   // [chunks, Hk] x 32 KB
  // training: D = T E for the backward (or null), fp32 tiles [chunks, Hv, Dv / 32 slices][64 rows][32]
  float* Ds;
  int* err;
};

// Store 16 floats (4 x 16 bytes).
__device__ __forceinline__ void st16_f32(float* p, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) reinterpret_cast<float4*>(p)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// 16 floats of row r of a [64][32] fp32 tile whose 16-byte chunks are swizzled by r & 7 (chunks
// 4 half .. 4 half + 3): conflict-free when the lanes of a warp own consecutive rows.
__device__ __forceinline__ void st16_f32_sw(uint8_t* tile, int r, int half, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<float4*>(tile + r * 128 + (((4 * half + q) ^ (r & 7)) << 4)) =
        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}
__device__ __forceinline__ void ld16_f32_sw(const uint8_t* tile, int r, int half, float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = *reinterpret_cast<const float4*>(tile + r * 128 + (((4 * half + q) ^ (r & 7)) << 4));
    v[4 * q] = x.x, v[4 * q + 1] = x.y, v[4 * q + 2] = x.z, v[4 * q + 3] = x.w;
  }
}

// Shared memory of the forward walk (bytes from a 1024-aligned base).
constexpr int FW_KQ = 0;           // 2 x 32 KB bf16 [K; Q] tile, 16-row groups interleaved (TMA)
constexpr int FW_T = 65536;        // 2 x 16 KB bf16 [T_hi; T_lo] image (bulk copy)
constexpr int FW_P = 98304;        // 2 x 16 KB bf16 [P_hi; P_lo] image (bulk copy)
constexpr int FW_S = 131072;       // 16 KB bf16 state [hi | lo], MN-major [128 dk][64]
constexpr int FW_E = 147456;       // 8 KB bf16 E [hi | lo], MN-major [64][64]
constexpr int FW_D = 155648;       // 8 KB bf16 D [hi | lo]
constexpr int FW_DT = 163840;      // 8 KB bf16 D~ = diag(lambda) D [hi | lo]
constexpr int FW_CK = 172032;      // 16 KB fp32 chunk-start state staging [32 dv][128 dk] (bulk store)
constexpr int FW_V = 188416;       // 2 x 4 KB bf16 value rows [64][32] (TMA)
constexpr int FW_DS = 196608;      // 2 x 8 KB fp32 D rows [64][32] staging (bulk store, training)
constexpr int FW_Y = 212992;       // 8 KB output rows [64][32] staging (TMA store of full chunks)
constexpr int FW_SMEM = 221184 + 1024;

// Descriptors of the stacked operands.  The [K; Q] tile holds, per 64-column slab (16 KB), the row
// groups K 0-15, Q 0-15, K 16-31, Q 16-31, ... (2 KB each).
// K-step ks of K^T (or Q^T with part = 1) as the M = 128 (dk) MN-major A operand; chunk rows are K.
__device__ __forceinline__ uint64_t desc_kq_t(uint32_t kq, int part, int ks) {
  return tc::sdesc(kq + part * 2048 + ks * 4096, 16384, 1024, 2);
}
// K-step ks of an N = 64 MN-major [hi | lo] operand (128-byte rows, one per K index).
__device__ __forceinline__ uint64_t desc_hl(uint32_t tile, int ks) { return tc::sdesc(tile + ks * 2048, 8192, 1024, 2); }

// A operand forms of mma_run: the M = 128 K-major tiles ([K; Q] and the [hi; lo] images), K^T, Q^T.
enum AForm { kKmaj128 = 0, kKT = 1, kQT = 2 };
// D (+)= A B over KSTEPS bf16 K-steps of 16, B an N = 64 [hi | lo] MN-major tile.
template <int KSTEPS, int AFORM>
__device__ __forceinline__ void mma_run(uint32_t d, uint32_t id, uint32_t a, uint32_t b, bool accumulate) {
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    const uint64_t ad = AFORM == kKmaj128 ? tc::desc_kmajor(a, 128, ks) : desc_kq_t(a, AFORM == kQT ? 1 : 0, ks);
    tc::mma_bf16(d, ad, desc_hl(b, ks), id, (accumulate || ks > 0) ? 1u : 0u);
  }
}

// This thread's 16 columns (16 half ..) of both N halves of a [hi | lo] accumulator, summed (both
// loads in flight together).
__device__ __forceinline__ void tmem_ld_hl16(uint32_t taddr, int half, float (&x)[16]) {
  uint32_t a[16], b[16];
  tc::tmem_ld16_nw(taddr + 16 * half, a);
  tc::tmem_ld16_nw(taddr + 32 + 16 * half, b);
  tc::tmem_wait_ld();
  tc::reg_fence(a);
  tc::reg_fence(b);
#pragma unroll
  for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(a[j]) + __uint_as_float(b[j]);
}
// Two such [hi | lo] sums, four loads in flight together.
__device__ __forceinline__ void tmem_ld_hl16x2(uint32_t ta, uint32_t tb, int half, float (&x)[16], float (&y)[16]) {
  uint32_t a0[16], a1[16], b0[16], b1[16];
  tc::tmem_ld16_nw(ta + 16 * half, a0);
  tc::tmem_ld16_nw(ta + 32 + 16 * half, a1);
  tc::tmem_ld16_nw(tb + 16 * half, b0);
  tc::tmem_ld16_nw(tb + 32 + 16 * half, b1);
  tc::tmem_wait_ld();
  tc::reg_fence(a0);
  tc::reg_fence(a1);
  tc::reg_fence(b0);
  tc::reg_fence(b1);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    x[j] = __uint_as_float(a0[j]) + __uint_as_float(a1[j]);
    y[j] = __uint_as_float(b0[j]) + __uint_as_float(b1[j]);
  }
}
// The same, then the hi-row and lo-row products of lanes l and l + 16 summed (both lanes get the sum).
__device__ __forceinline__ void tmem_ld_hl16_pair(uint32_t taddr, int half, float (&x)[16]) {
  tmem_ld_hl16(taddr, half, x);
#pragma unroll
  for (int j = 0; j < 16; ++j) x[j] += __shfl_xor_sync(0xffffffffu, x[j], 16);
}

// 256 threads: warp w reads TMEM lanes 32 (w & 3) .. + 31 and handles the value columns
// 16 (w >> 2) .. + 15 of the CTA's 32; thread t holds S[dv0 + 16 (w >> 2) + j][t & 127].
template <typename Tout>
__global__ void __launch_bounds__(256, 1) gdn_chunk_fwd_state(const __grid_constant__ CUtensorMap vmap,
                                                              const __grid_constant__ CUtensorMap ymap, StateArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float sg[2][128];
  __shared__ uint64_t bar_tma[2], bar_mma;
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2, dk = tid & 127;
  const int dv0 = blockIdx.x * DVT, hv = blockIdx.y, n = blockIdx.z;
  const int Hv = a.geo.Hv, hk = hv / (Hv / a.geo.Hk);
  int64_t c_first, nchunks, seq0, seq1;
  seq_chunks(a.geo, n, c_first, nchunks, seq0, seq1);

  // TMEM: [K; Q] S^T 0, D 64, S update 128, P D 192 (64 columns each: hi and lo halves)
  const uint32_t cA = 0, cD = 64, cS = 128, cO = 192;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 256);
  if (tid == 0) {
    tc::mbar_init(&bar_tma[0], 1);
    tc::mbar_init(&bar_tma[1], 1);
    tc::mbar_init(&bar_mma, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tl = tc::taddr(tmem, 32 * quad, 0);  // this warp's lanes

  float s[16];  // s[j] = S[dv0 + 16 half + j][dk]
  {
    const size_t base = (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
    for (int j = 0; j < 16; ++j) s[j] = a.h0 ? a.h0[base + (size_t)j * DK] : 0.f;
  }

  // One thread of warp 1 moves everything a chunk reads (the [K; Q], T and P images, the gates and the
  // value rows) and the checkpoint, so that warp 0's thread issues the MMAs meanwhile and no thread
  // waits on a global load inside the walk.
  auto issue_loads = [&](int64_t jc, int buf) {
    const int64_t cg = c_first + jc;
    tc::mbar_arrive_expect_tx(&bar_tma[buf], 32768 + 2 * 16384 + 512 + 4096);
    tc::bulk_load(smem + FW_KQ + buf * 32768, a.KQimg + (size_t)(cg * a.geo.Hk + hk) * 32768, 32768, &bar_tma[buf]);
    tc::bulk_load(smem + FW_T + buf * 16384, a.Timg + (size_t)(cg * Hv + hv) * 16384, 16384, &bar_tma[buf]);
    tc::bulk_load(smem + FW_P + buf * 16384, a.Pimg + (size_t)(cg * Hv + hv) * 16384, 16384, &bar_tma[buf]);
    tc::bulk_load(sg[buf], a.gates + (cg * Hv + hv) * 128, 512, &bar_tma[buf]);
    tc::tma_load_3d(smem + FW_V + buf * 4096, &vmap, &bar_tma[buf], dv0, hv, (int)(seq0 + jc * C));
  };

  // Lane l < 16 owns chunk row i = 16 quad + l for the K-side products (E, D) and lane l + 16 the same
  // row for the Q-side ones (Y, D~, y).
  const int i_row = 16 * quad + (lane & 15);
  const bool kside = lane < 16;
  if (nchunks > 0 && tid == 32) {
    tc::prefetch_tmap(&vmap);
    issue_loads(0, 0);
  }
  uint32_t ph = 0;
  bool ok = true;
  const uint32_t idA = tc::idesc(tc::kBF16, 128, 64, false, true);
  const uint32_t idT = tc::idesc(tc::kBF16, 128, 64, true, true);
  int64_t ystage_tok = -1;  // first token of the full chunk whose output rows wait in the staging tile

  // The waits for an MMA round are per thread (the TMEM results are ready for every thread once it has
  // seen the commit); their outcome joins the chunk's next barrier, where every thread breaks alike.
  for (int64_t jc = 0; jc < nchunks; ++jc) {
    const int buf = (int)(jc & 1);
    const int64_t cg = c_first + jc;
    const int64_t tok0 = seq0 + jc * C;
    const int L = (int)min((int64_t)C, seq1 - tok0);

    // 1. the chunk-start state: staged for the bulk store of the checkpoint, and as the [hi | lo]
    //    operand row dk
    if (a.ckpt) {  // rounded to tf32: its one reader takes it as a tf32 operand
      float* ck = reinterpret_cast<float*>(smem + FW_CK) + 16 * half * DK + dk;
#pragma unroll
      for (int j = 0; j < 16; ++j) ck[j * DK] = tf32_rna(s[j]);
    }
    tc::st_row_hilo16(smem + FW_S, dk, s, half);
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok && tc::mbar_wait(&bar_tma[buf], (uint32_t)((jc >> 1) & 1), a.err, 10)) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    const uint32_t kq = tc::smem_u32(smem + FW_KQ + buf * 32768);
    // 2. [K; Q] S^T in one pass (M = 128, N = 64: the state's hi and lo halves)
    if (tid == 0) {
      mma_run<8, kKmaj128>(tmem + cA, idA, kq, tc::smem_u32(smem + FW_S), false);
      tc::mma_commit(&bar_mma);
    }
    if (tid == 32) {
      if (a.ckpt) tc::bulk_store(a.ckpt + ((cg * Hv + hv) * DV + dv0) * (size_t)DK, smem + FW_CK, DVT * DK * 4);
      if (ystage_tok >= 0) tc::tma_store_3d(&ymap, smem + FW_Y, dv0, hv, (int)ystage_tok);  // last chunk's y
      tc::bulk_commit();
      if (jc + 1 < nchunks) issue_loads(jc + 1, buf ^ 1);  // the next chunk's tiles
    }
    const float* gb = sg[buf];
    const float bi = gb[i_row], be = gb[64 + i_row], gi = __expf(bi), bC = gb[63];
    float vr[16];  // this row's values (rows past the sequence's end read as zero)
    {
      Row16 raw;
      const uint4* vp = reinterpret_cast<const uint4*>(smem + FW_V + buf * 4096 + i_row * 64 + 32 * half);
      raw.w[0] = i_row < L ? vp[0] : make_uint4(0, 0, 0, 0);
      raw.w[1] = i_row < L ? vp[1] : make_uint4(0, 0, 0, 0);
      cvt_row16(raw, vr);
    }
    ok = ok && tc::mbar_wait(&bar_mma, ph, a.err, 11);
    ph ^= 1;
    tc::fence_after_sync();
    // 3. K side: E = diag(beta) (V - diag(gamma) K S^T) as the [hi | lo] operand; Q side: gamma Q S^T
    float yp[16];
    const size_t ptile = ((size_t)(cg * Hv + hv) * (DV / DVT) + blockIdx.x) * 2048;  // this CTA's tile
    {
      // one instruction stream for the lane pair: the K-side lane forms E's columns 0-7 from its K S^T
      // row, the Q-side lane columns 8-15 from the K-side lane's; the Q-side lane keeps gamma Q S^T
      tmem_ld_hl16(tl + cA, half, yp);
      float e8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float ks = __shfl_xor_sync(0xffffffffu, yp[8 + j], 16);
        e8[j] = be * ((kside ? vr[j] : vr[8 + j]) - gi * (kside ? yp[j] : ks));
      }
      st_hilo8(smem + FW_E, i_row, e8, 2 * half + (kside ? 0 : 1));
#pragma unroll
      for (int j = 0; j < 16; ++j) yp[j] *= gi;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 4. D = T E  ([T_hi; T_lo] stacked: row i's two products in lanes l and l + 16)
    if (tid == 0) {
      mma_run<4, kKmaj128>(tmem + cD, idA, tc::smem_u32(smem + FW_T + buf * 16384), tc::smem_u32(smem + FW_E), false);
      tc::mma_commit(&bar_mma);
    }

    ok = ok && tc::mbar_wait(&bar_mma, ph, a.err, 12);
    ph ^= 1;
    tc::fence_after_sync();
    {
      // both lanes of the pair hold row i of D; one instruction stream for both: the K-side lane writes
      // D as the [hi | lo] operand of P D and columns 0-7 of the tf32 copy, the Q-side lane
      // D~ = diag(lambda) D for the state update and columns 8-15 of the copy
      float d[16];
      tmem_ld_hl16_pair(tl + cD, half, d);
      // (the other staging buffer's store was read before the last chunk's final barrier)
      if (a.Ds) {  // tf32-rounded: the gradient kernel's tf32 operand, loaded as is
        uint8_t* row = smem + FW_DS + buf * 8192 + i_row * 128;
        const int q0 = 4 * half + (kside ? 0 : 2);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float x[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] = tf32_rna(kside ? d[4 * q + e] : d[8 + 4 * q + e]);
          *reinterpret_cast<float4*>(row + (((q0 + q) ^ (i_row & 7)) << 4)) = make_float4(x[0], x[1], x[2], x[3]);
        }
      }
      const float sc = kside ? 1.f : __expf(bC - bi);
#pragma unroll
      for (int j = 0; j < 16; ++j) d[j] *= sc;
      tc::st_row_hilo16(smem + (kside ? FW_D : FW_DT), i_row, d, half);
    }
    if (tid == 32) tc::bulk_wait_read();  // the staging buffers are rewritten below and next chunk
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 5. S update^T = K^T D~ (M = 128 dk rows);  O2 = P D ([P_hi; P_lo] stacked)
    if (tid == 0) {
      mma_run<4, kKT>(tmem + cS, idT, kq, tc::smem_u32(smem + FW_DT), false);
      mma_run<4, kKmaj128>(tmem + cO, idA, tc::smem_u32(smem + FW_P + buf * 16384), tc::smem_u32(smem + FW_D), false);
      tc::mma_commit(&bar_mma);
    }
    if (tid == 32 && a.Ds) {
      tc::bulk_store(a.Ds + ptile, smem + FW_DS + buf * 8192, 8192);
      tc::bulk_commit();
    }
    ok = ok && tc::mbar_wait(&bar_mma, ph, a.err, 13);
    ph ^= 1;
    tc::fence_after_sync();
    {
      float u[16], o2[16];
      tmem_ld_hl16x2(tl + cS, tl + cO, half, u, o2);
      const float gC = __expf(bC);
#pragma unroll
      for (int j = 0; j < 16; ++j) s[j] = fmaf(gC, s[j], u[j]);
#pragma unroll
      for (int j = 0; j < 16; ++j) u[j] = o2[j] + __shfl_xor_sync(0xffffffffu, o2[j], 16);
      // both lanes hold P D's row; the K-side lane writes columns 0-7 (with the Q-side lane's gamma Q S^T),
      // the Q-side lane columns 8-15
      const int hc = kside ? 0 : 1;
      float y8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float qy = __shfl_xor_sync(0xffffffffu, yp[j], 16);
        y8[j] = kside ? u[j] + qy : u[8 + j] + yp[8 + j];
      }
      if (L == C)  // a full chunk goes out by one TMA store after the next barrier
        store_row8<Tout>(reinterpret_cast<Tout*>(smem + FW_Y) + i_row * DVT + 16 * half + 8 * hc, y8);
      else if (i_row < L)  // the rows after a sequence's end belong to the next sequence: not written
        store_row8<Tout>(static_cast<Tout*>(a.y) + ((tok0 + i_row) * Hv + hv) * (size_t)DV + dv0 + 16 * half + 8 * hc, y8);
    }
    ystage_tok = L == C ? tok0 : -1;
    tc::fence_async_smem();
    tc::fence_before_sync();
  }
  ok = __syncthreads_and(ok) != 0;  // (the last round's waits were per thread)
  if (ok && ystage_tok >= 0 && tid == 32) {  // the last chunk's output rows
    tc::tma_store_3d(&ymap, smem + FW_Y, dv0, hv, (int)ystage_tok);
    tc::bulk_commit();
  }
  if (tid == 32) tc::bulk_wait();
  if (ok && a.hT) {
    float* dst = a.hT + (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[(size_t)j * DK] = s[j];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------------------------------------
// The backward state walk: chunks in reverse, 32 rows of dS per CTA (thread t holds dS[dv0+j][t]).
struct BwdStateArgs {
  Geo geo;
  const void* dy;         // [B*T, Hv, Dv] bf16
  const float* gates;
  const float* dhT;       // [N, Hv, Dv, Dk] or null
  void* dv;               // [B*T, Hv, Dv]
  float* dh0;             // or null
  float* dsbuf;           // [chunks, Hv, Dv, Dk]: cotangent of each chunk's end state
  const uint8_t* Timg;    // the forward's operand images
  const uint8_t* Pimg;
  const uint8_t* KQimg;
  // the gradient kernel's A operand [dO; F] (F = T^T dD), tf32, as the 128-row K-major image with
  // 16-row groups interleaved: [chunks, Hv, Dv / 32] x 16 KB
  uint8_t* Aimg;
  int* err;
};

constexpr int BW_KQ = 0;           // 2 x 32 KB bf16 [K; Q] image
constexpr int BW_T = 65536;        // 16 KB bf16 [T_hi; T_lo] image (reloaded once the chunk's F is done)
constexpr int BW_P = 81920;        // 16 KB bf16 [P_hi; P_lo] image (reloaded once P^T dO is done)
constexpr int BW_S = 98304;        // 16 KB bf16 dS [hi | lo], MN-major [128 dk][64]
constexpr int BW_DO = 114688;      // 8 KB bf16 dO, MN-major [64][32] (128-byte rows, half used)
constexpr int BW_GD = 122880;      // 8 KB bf16 gamma dO [hi | lo]
constexpr int BW_DD = 131072;      // 8 KB bf16 dD [hi | lo]
constexpr int BW_H = 139264;       // 8 KB bf16 H = -beta gamma F [hi | lo]
constexpr int BW_CK = 147456;      // 16 KB fp32 dS staging [32 dv][128 dk] (bulk store)
constexpr int BW_V = 163840;       // 2 x 4 KB bf16 dO rows [64][32] (TMA)
constexpr int BW_FS = 172032;      // 2 x 16 KB [dO; F] operand image staging (bulk store)
constexpr int BW_DV = 204800;      // 8 KB dv rows [64][32] staging (TMA store of full chunks)
constexpr int BW_SMEM = 212992 + 1024;

// K-step ks of the transpose of one half (part 0 = hi, 1 = lo) of a [hi; lo] image as the M = 64
// MN-major A operand: the image's rows (chunk steps) are K.
__device__ __forceinline__ uint64_t desc_img_t(uint32_t img, int part, int ks) {
  return tc::sdesc(img + part * 2048 + ks * 4096, 8192, 1024, 2);
}

// Load 16 fp32 of a shared row.
__device__ __forceinline__ void ld16_f32(const uint8_t* p, float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = reinterpret_cast<const float4*>(p)[q];
    v[4 * q] = x.x, v[4 * q + 1] = x.y, v[4 * q + 2] = x.z, v[4 * q + 3] = x.w;
  }
}
// 16 bf16 of a shared row as floats, zero unless valid.
__device__ __forceinline__ void ld16_bf16(const uint8_t* p, bool valid, float (&v)[16]) {
  Row16 r;
  const uint4 z = make_uint4(0, 0, 0, 0);
  r.w[0] = valid ? reinterpret_cast<const uint4*>(p)[0] : z;
  r.w[1] = valid ? reinterpret_cast<const uint4*>(p)[1] : z;
  cvt_row16(r, v);
}

// The backward state walk: chunks in reverse, 32 rows of dS per CTA, 256 threads as in the forward walk
// (thread t holds dS[dv0 + 16 (w >> 2) + j][t & 127]).  Besides dv, the per-chunk dS and dh0 it leaves
// the gradient kernel F = T^T dD.
template <typename Tout>
__global__ void __launch_bounds__(256, 1) gdn_chunk_bwd_state(const __grid_constant__ CUtensorMap dmap,
                                                              const __grid_constant__ CUtensorMap dvmap,
                                                              BwdStateArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float sg[2][128];
  __shared__ uint64_t bar_tma[2], bar_t, bar_p, bar_mma;
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2, dk = tid & 127;
  const int dv0 = blockIdx.x * DVT, hv = blockIdx.y, n = blockIdx.z;
  const int Hv = a.geo.Hv, hk = hv / (Hv / a.geo.Hk);
  int64_t c_first, nchunks, seq0, seq1;
  seq_chunks(a.geo, n, c_first, nchunks, seq0, seq1);

  // TMEM: [K; Q] dS^T 0 (64), P^T dO 64 (32), F 128 (64), U 192 (64)
  const uint32_t cX = 0, cG = 64, cF = 128, cU = 192;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 256);
  if (tid == 0) {
    tc::mbar_init(&bar_tma[0], 1);
    tc::mbar_init(&bar_tma[1], 1);
    tc::mbar_init(&bar_t, 1);
    tc::mbar_init(&bar_p, 1);
    tc::mbar_init(&bar_mma, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tl = tc::taddr(tmem, 32 * quad, 0);

  float ds[16];  // ds[j] = dS[dv0 + 16 half + j][dk]
  {
    const size_t base = (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
    for (int j = 0; j < 16; ++j) ds[j] = a.dhT ? a.dhT[base + (size_t)j * DK] : 0.f;
  }

  // one thread of warp 1 issues every copy; the T and P images have one buffer each, refilled as soon
  // as the chunk's last product with them has completed
  auto issue_main = [&](int64_t jc, int buf) {
    const int64_t cg = c_first + jc;
    tc::mbar_arrive_expect_tx(&bar_tma[buf], 32768 + 512 + 4096);
    tc::bulk_load(smem + BW_KQ + buf * 32768, a.KQimg + (size_t)(cg * a.geo.Hk + hk) * 32768, 32768, &bar_tma[buf]);
    tc::bulk_load(sg[buf], a.gates + (cg * Hv + hv) * 128, 512, &bar_tma[buf]);
    tc::tma_load_3d(smem + BW_V + buf * 4096, &dmap, &bar_tma[buf], dv0, hv, (int)(seq0 + jc * C));
  };
  auto issue_t = [&](int64_t jc) {
    tc::mbar_arrive_expect_tx(&bar_t, 16384);
    tc::bulk_load(smem + BW_T, a.Timg + (size_t)((c_first + jc) * Hv + hv) * 16384, 16384, &bar_t);
  };
  auto issue_p = [&](int64_t jc) {
    tc::mbar_arrive_expect_tx(&bar_p, 16384);
    tc::bulk_load(smem + BW_P, a.Pimg + (size_t)((c_first + jc) * Hv + hv) * 16384, 16384, &bar_p);
  };
  const int i_row = 16 * quad + (lane & 15);
  const bool kside = lane < 16;
  if (nchunks > 0 && tid == 32) {
    tc::prefetch_tmap(&dmap);
    issue_main(nchunks - 1, 0);
    issue_t(nchunks - 1);
    issue_p(nchunks - 1);
  }
  uint32_t ph = 0;
  bool ok = true;
  const uint32_t idX = tc::idesc(tc::kBF16, 128, 64, false, true);  // [K; Q] x [hi | lo]
  const uint32_t idG = tc::idesc(tc::kBF16, 64, 32, true, true);    // P^T x dO
  const uint32_t idF = tc::idesc(tc::kBF16, 64, 64, true, true);    // T^T x [hi | lo]
  const uint32_t idU = tc::idesc(tc::kBF16, 128, 64, true, true);   // Q^T, K^T x [hi | lo]

  // MMA-round waits per thread, joined at the chunk's next barrier (as in the forward walk)
  for (int64_t it = 0; it < nchunks; ++it) {
    const int64_t jc = nchunks - 1 - it;
    const int buf = (int)(it & 1);
    const int64_t cg = c_first + jc;
    const int64_t tok0 = seq0 + jc * C;
    const int L = (int)min((int64_t)C, seq1 - tok0);

    // 1. dS of this chunk's end: staged for the gradient kernel, and as the [hi | lo] operand row dk
    {  // rounded to tf32: its one reader takes it as a tf32 operand
      float* ck = reinterpret_cast<float*>(smem + BW_CK) + 16 * half * DK + dk;
#pragma unroll
      for (int j = 0; j < 16; ++j) ck[j * DK] = tf32_rna(ds[j]);
    }
    tc::st_row_hilo16(smem + BW_S, dk, ds, half);
    // (each thread waits for the chunk's rows and gates itself: steps 1 and 2 share one barrier)
    bool okw = ok && tc::mbar_wait(&bar_tma[buf], (uint32_t)((it >> 1) & 1), a.err, 20);
    const float* gb = sg[buf];
    const float bi = gb[i_row], be = gb[64 + i_row], gi = __expf(bi), bC = gb[63];
    // 2. dO row i (zero past the end) as the plain bf16 operand of P^T dO, as gamma dO [hi | lo] and, exact
    //    in tf32, into the gradient kernel's image (lower row of the pair; the other staging buffer's
    //    store was read before the last chunk's step-4 barrier).  One instruction stream for the lane
    //    pair: the K-side lane takes columns 0-7 of the thread's 16, the Q-side lane columns 8-15.
    {
      const int hc = kside ? 0 : 1;
      const uint4 w = i_row < L ? reinterpret_cast<const uint4*>(smem + BW_V + buf * 4096 + i_row * 64 + 32 * half)[hc]
                                : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(smem + BW_DO + i_row * 128 + (((2 * half + hc) ^ (i_row & 7)) << 4)) = w;
      float d[8];
      {
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
          d[2 * e] = __low2float(h2);
          d[2 * e + 1] = __high2float(h2);
        }
      }
      st8_f32_sw(smem + BW_FS + buf * 16384, img_row(i_row), 4 * half + 2 * hc, d);
#pragma unroll
      for (int j = 0; j < 8; ++j) d[j] *= gi;
      st_hilo8(smem + BW_GD, i_row, d, 2 * half + hc);
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    okw = okw && tc::mbar_wait(&bar_t, (uint32_t)(it & 1), a.err, 25) && tc::mbar_wait(&bar_p, (uint32_t)(it & 1), a.err, 26);
    ok = __syncthreads_and(okw) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    const uint32_t kq = tc::smem_u32(smem + BW_KQ + buf * 32768);
    const uint32_t pimg = tc::smem_u32(smem + BW_P), timg = tc::smem_u32(smem + BW_T);
    // 3. [K; Q] dS^T (the K rows are X1 = K dS^T) and G = P^T dO (P_hi^T and P_lo^T accumulated)
    if (tid == 0) {
      mma_run<8, kKmaj128>(tmem + cX, idX, kq, tc::smem_u32(smem + BW_S), false);
      const uint32_t dO = tc::smem_u32(smem + BW_DO);
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + cG, desc_img_t(pimg, part, ks), desc_hl(dO, ks), idG, (part | ks) ? 1u : 0u);
      tc::mma_commit(&bar_mma);
      // U's first half Q^T (gamma dO) needs no result of this chunk: it runs during the next epilogue,
      // and step 6 adds K^T H to it
      mma_run<4, kQT>(tmem + cU, idU, kq, tc::smem_u32(smem + BW_GD), false);
    }
    if (tid == 32) {  // while the products run: this chunk's dS out, the previous chunk's tiles in
      tc::bulk_store(a.dsbuf + ((cg * Hv + hv) * DV + dv0) * (size_t)DK, smem + BW_CK, DVT * DK * 4);
      tc::bulk_commit();
      if (jc > 0) issue_main(jc - 1, buf ^ 1);  // the previous chunk's [K; Q], gates and dO rows
    }
    ok = ok && tc::mbar_wait(&bar_mma, ph, a.err, 21);
    ph ^= 1;
    tc::fence_after_sync();
    if (ok && tid == 32 && jc > 0) issue_p(jc - 1);  // P's last reader has completed
    // 4. dD = diag(lambda) K dS^T + P^T dO (K side), as the [hi | lo] operand.  tcgen05.ld is a
    //    warp-wide aligned instruction: every lane executes the same loads, outside the branch.
    {
      float x[16], g[16];
      {
        uint32_t a0[16], a1[16], b0[16];
        tc::tmem_ld16_nw(tl + cX + 16 * half, a0);
        tc::tmem_ld16_nw(tl + cX + 32 + 16 * half, a1);
        tc::tmem_ld16_nw(tl + cG + 16 * half, b0);
        tc::tmem_wait_ld();
        tc::reg_fence(a0);
        tc::reg_fence(a1);
        tc::reg_fence(b0);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          x[j] = __uint_as_float(a0[j]) + __uint_as_float(a1[j]);
          g[j] = __uint_as_float(b0[j]);
        }
      }
      // the K-side lane forms dD; the Q-side lane takes its columns 8-15 and stores them
      const float lam = __expf(bC - bi);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = fmaf(lam, x[j], g[j]);
      float d8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = __shfl_xor_sync(0xffffffffu, x[8 + j], 16);
        d8[j] = kside ? x[j] : y;
      }
      st_hilo8(smem + BW_DD, i_row, d8, 2 * half + (kside ? 0 : 1));
    }
    if (tid == 32) tc::bulk_wait_read();  // the staging buffer is rewritten next chunk
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 5. F = T^T dD (T_hi^T and T_lo^T accumulated; M = 64: row j in the K-side lanes)
    if (tid == 0) {
      const uint32_t dd = tc::smem_u32(smem + BW_DD);
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + cF, desc_img_t(timg, part, ks), desc_hl(dd, ks), idF, (part | ks) ? 1u : 0u);
      tc::mma_commit(&bar_mma);
    }
    ok = ok && tc::mbar_wait(&bar_mma, ph, a.err, 22);
    ph ^= 1;
    tc::fence_after_sync();
    if (ok && tid == 32 && jc > 0) issue_t(jc - 1);  // T's last reader has completed
    {
      float f[16];
      tmem_ld_hl16(tl + cF, half, f);
      // F's row i is in the K-side lane; the Q-side lane takes its columns 8-15, and both lanes write
      // their 8 columns of the three outputs with one instruction stream
      const int hc = kside ? 0 : 1;
      float f8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = __shfl_xor_sync(0xffffffffu, f[8 + j], 16);
        f8[j] = kside ? f[j] : y;
      }
      {  // F, tf32-rounded, into the image's upper row of the pair
        float fr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) fr[j] = tf32_rna(f8[j]);
        st8_f32_sw(smem + BW_FS + buf * 16384, img_row(i_row) + 16, 4 * half + 2 * hc, fr);
      }
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = be * f8[j];
      if (L == C)  // a full chunk goes out by one TMA store after the barrier below
        store_row8<Tout>(reinterpret_cast<Tout*>(smem + BW_DV) + i_row * DVT + 16 * half + 8 * hc, o);
      else if (i_row < L)  // the rows after a sequence's end belong to the next sequence: not written
        store_row8<Tout>(static_cast<Tout*>(a.dv) + ((tok0 + i_row) * Hv + hv) * (size_t)DV + dv0 + 16 * half + 8 * hc, o);
      const float h = -be * gi;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = h * f8[j];
      st_hilo8(smem + BW_H, i_row, o, 2 * half + hc);
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 6. U = Q^T (gamma dO) (issued in step 3) + K^T H (M = 128 dk rows)
    if (tid == 0) {
      mma_run<4, kKT>(tmem + cU, idU, kq, tc::smem_u32(smem + BW_H), true);
      tc::mma_commit(&bar_mma);
    }
    if (tid == 32) {
      tc::bulk_store(a.Aimg + ((size_t)(cg * Hv + hv) * (DV / DVT) + blockIdx.x) * 16384, smem + BW_FS + buf * 16384,
                     16384);
      if (L == C) tc::tma_store_3d(&dvmap, smem + BW_DV, dv0, hv, (int)tok0);
      tc::bulk_commit();
    }
    ok = ok && tc::mbar_wait(&bar_mma, ph, a.err, 23);
    ph ^= 1;
    tc::fence_after_sync();
    {
      float u[16];
      tmem_ld_hl16(tl + cU, half, u);
      const float gC = __expf(bC);
#pragma unroll
      for (int j = 0; j < 16; ++j) ds[j] = fmaf(gC, ds[j], u[j]);
    }
    tc::fence_before_sync();
  }
  ok = __syncthreads_and(ok) != 0;  // (the last round's waits were per thread)
  if (tid == 32) tc::bulk_wait();
  if (ok && a.dh0) {
    float* dst = a.dh0 + (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[(size_t)j * DK] = ds[j];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------------------------------------
// Per-chunk gradients: one CTA per (chunk, key head); its value heads in turn, Dv in four slices of 32.
// D comes from the forward walk and F from the reverse walk.  Per value head this kernel accumulates
// over the value rows dO S, F S, D dS (unscaled) and dO D^T, F D^T; the finalize takes the per-row
// terms of d log g from them -- Q_i . (dO S)_i = dO_i . Y_i, K_i . (F S)_i = F_i . R_i,
// K_i . (D dS)_i = D_i . (K dS^T)_i -- and adds gamma dO S, -beta gamma F S + lambda D dS and the
// Gamma-masked products into dQ and dK.
struct GradArgs {
  Geo geo;
  const float* g;           // [B*T, Hv] (dg = d log g / g); null in layer mode
  const float* gates;       // [chunks, Hv, 2, 64]
  const uint8_t *Pimg, *KQimg;  // the forward's operand images
  const float* Ds;          // D (tf32-rounded), fp32 tiles [chunks, Hv, Dv / 32][64][32], rows swizzled
  const uint8_t* Aimg;      // [dO; F] operand images [chunks, Hv, Dv / 32] x 16 KB
  void *dq, *dk;            // [B*T, Hk, Dk]
  float *dg, *dbeta;        // [B*T, Hv]; layer mode: da, db
  int* err;
  // layer mode: raw inputs for the norm and gate chain rule, per-chunk head sums of dA_log, ddt_bias
  const __nv_bfloat16 *q_raw, *k_raw;
  const float *a_raw, *b_raw, *A_log, *dt_bias;
  float* head_part;         // [chunks, Hv, 2]
  float *dA_log, *ddt_bias; // [Hv]: the sums over all chunks, written by the CTA that finishes last
  unsigned* done;           // CTAs finished (zero when the kernel starts)
};

// Shared memory of the gradient kernel.
constexpr int GR_KQ = 0;           // 32 KB bf16 [K; Q] image
constexpr int GR_P = 32768;        // 16 KB bf16 [P_hi; P_lo] image of the value head
constexpr int GR_BUF = 49152;      // 2 x 60 KB slice buffers: S, dS (tf32, MN-major [32 dv][128 dk], +0, +16 KB),
constexpr int GR_BS = 61440;       //   the [dO; F] image (+32 KB), D (K-major [64][32], +48 KB), V rows (+56 KB)
constexpr int GR_KO = 172032;      // 16 KB bf16 K rows alone (K-major): the B operand of K K^T
constexpr int GR_RAW = 188416;     // 32 KB layer mode: the raw q (rows 0-63) and k (rows 64-127) rows, 256 B each
constexpr int GR_SMEM = 221184 + 1024;
// The value head's finalize reuses the second slice buffer (its last slice is an odd one): the
// [dP^; dKK] images and a column-sum scratch; meanwhile the next value head's first slice arrives in
// the first buffer.
constexpr int GR_FHI = GR_BUF + GR_BS, GR_FLO = GR_BUF + GR_BS + 16384, GR_SCR = GR_BUF + GR_BS + 32768;
static_assert((DV / DVT) % 2 == 0, "a value head's last slice must use the second buffer");
static_assert(32768 + (64 * 65 + 4 * 64) * 4 <= GR_BS, "finalize scratch exceeds a slice buffer");

// 16 bytes global -> shared by the non-bulk asynchronous copy; the issuing thread waits for its own.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 16 floats into chunks 4 half .. 4 half + 3 of row r of a K-major fp32 128-byte-swizzled slab.
__device__ __forceinline__ void st_row_k_f32_16(uint8_t* slab, int r, const float (&v)[16], int half) {
  uint8_t* row = slab + r * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<float4*>(row + (((4 * half + c) ^ (r & 7)) << 4)) =
        make_float4(tf32_rna(v[4 * c]), tf32_rna(v[4 * c + 1]), tf32_rna(v[4 * c + 2]), tf32_rna(v[4 * c + 3]));
}
// 16 floats as bf16 hi (into hi_img) and lo (into lo_img), row r, 16-byte chunks c0 and c0 + 1 of a
// 128-byte-swizzled tile.
__device__ __forceinline__ void st_hilo16_chunks(uint8_t* hi_img, uint8_t* lo_img, int r, const float (&v)[16], int c0) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = v[8 * c + 2 * e], y = v[8 * c + 2 * e + 1];
      const __nv_bfloat162 hh = __floats2bfloat162_rn(x, y);
      h[e] = *reinterpret_cast<const uint32_t*>(&hh);
      l[e] = tc::pack_bf16(x - __low2float(hh), y - __high2float(hh));
    }
    const int off = r * 128 + (((c0 + c) ^ (r & 7)) << 4);
    *reinterpret_cast<uint4*>(hi_img + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_img + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}
// 32 bf16 of row r of a K-major bf16 image slab (128-byte swizzle), columns 32 m .. 32 m + 31.
__device__ __forceinline__ void ld_img_row32(const uint8_t* slab, int r, int m, float (&v)[32]) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const uint4 w = *reinterpret_cast<const uint4*>(slab + r * 128 + (((4 * m + cc) ^ (r & 7)) << 4));
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
      v[8 * cc + 2 * e] = __low2float(h);
      v[8 * cc + 2 * e + 1] = __high2float(h);
    }
  }
}

// 256 threads.  Warp w reads TMEM lanes 32 (w & 3) .. + 31 and handles columns 16 (w >> 2) .. + 15 of a
// 32-wide slice (32 (w >> 2) .. of the 64-wide finalize, 64 (w >> 2) .. of the 128-wide dk).  The
// stacked accumulators hold chunk row i = 16 (w & 3) + l in lane l ("lower": dQ, dO S, dP) and in lane
// l + 16 ("upper": dK, F S, D dS, F D^T).
template <typename Tout>
__global__ void __launch_bounds__(256, 1) gdn_chunk_bwd_grad(const __grid_constant__ CUtensorMap smap_mn,
                                                             const __grid_constant__ CUtensorMap dmap_mn,
                                                             const __grid_constant__ CUtensorMap vmap, GradArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float sgt[2][128];  // the value heads' gates: b[64], beta[64] (double-buffered)
  __shared__ float srow[6][2][64];           // per-row partial sums from both column halves
  __shared__ float sdb[65], sred[16];
  __shared__ float snorm[2][2][128];
  __shared__ uint64_t bar_kq, bar_h, bar_kk, bar_s[2], bar_mma;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int64_t c = blockIdx.x;
  const int hk = blockIdx.y, Hv = a.geo.Hv, ratio = Hv / a.geo.Hk;
  int n, L;
  int64_t tok0;
  chunk_info(a.geo, c, n, tok0, L);
  const int i_row = 16 * quad + (lane & 15);
  const bool lower = lane < 16;
  const bool rvalid = i_row < L;

  // TMEM: dQ | dK 0 (128), dO S | F S 128 (128), D dS 256 (upper lanes, 128), dP | F D^T 384 (64),
  // K K^T 448 (64, lower lanes; the upper lanes get Q K^T, unused)
  const uint32_t cQK = 0, cA1 = 128, cA2 = 256, cPF = 384, cKK = 448;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 512);
  if (tid == 0) {
    tc::mbar_init(&bar_kq, 1);
    tc::mbar_init(&bar_h, 1);
    tc::mbar_init(&bar_kk, 1);
    tc::mbar_init(&bar_s[0], 1);
    tc::mbar_init(&bar_s[1], 1);
    tc::mbar_init(&bar_mma, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tl = tc::taddr(tmem, 32 * quad, 0);
  constexpr int NSL = DV / DVT;
  // layer mode: this thread's half row of raw q (lower lanes) or k (upper lanes) for the norm chain rule
  // at the end, fetched now; 16-byte chunks swizzled by the row
  const size_t rowoff = ((tok0 + i_row) * a.geo.Hk + hk) * (size_t)DK + 64 * half;
  uint8_t* rawrow = smem + GR_RAW + ((lower ? 0 : 64) + i_row) * 256 + 128 * half;
  if (!a.g && rvalid) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>((lower ? a.q_raw : a.k_raw) + rowoff);
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) cp_async16(rawrow + ((cc ^ (i_row & 7)) << 4), src + 16 * cc);
  }

  // slice q = r * NSL + sl of this CTA: S, dS slices, D and F tiles, dO and value rows, into buffer q & 1
  auto issue_slice = [&](int q) {
    const int r = q / NSL, sl = q - r * NSL, hv = hk * ratio + r, bs = q & 1;
    uint8_t* buf = smem + GR_BUF + bs * GR_BS;
    const int srow_ = (int)((c * Hv + hv) * DV + sl * DVT);
    const size_t tile = (size_t)(c * Hv + hv) * NSL + sl;
    tc::mbar_arrive_expect_tx(&bar_s[bs], 3 * 16384 + 8192 + 4096);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      tc::tma_load_2d(buf + 4096 * b, &smap_mn, &bar_s[bs], 32 * b, srow_);
      tc::tma_load_2d(buf + 16384 + 4096 * b, &dmap_mn, &bar_s[bs], 32 * b, srow_);
    }
    tc::bulk_load(buf + 32768, a.Aimg + tile * 16384, 16384, &bar_s[bs]);
    tc::bulk_load(buf + 49152, a.Ds + tile * 2048, 8192, &bar_s[bs]);
    tc::tma_load_3d(buf + 57344, &vmap, &bar_s[bs], sl * DVT, hv, (int)tok0);
  };
  auto issue_head = [&](int r) {
    const int hv = hk * ratio + r;
    tc::mbar_arrive_expect_tx(&bar_h, 16384 + 512);
    tc::bulk_load(smem + GR_P, a.Pimg + (size_t)(c * Hv + hv) * 16384, 16384, &bar_h);
    tc::bulk_load(sgt[r & 1], a.gates + (c * Hv + hv) * 128, 512, &bar_h);
  };
  if (tid == 32) {
    tc::prefetch_tmap(&smap_mn);
    tc::prefetch_tmap(&dmap_mn);
    tc::prefetch_tmap(&vmap);
    tc::mbar_arrive_expect_tx(&bar_kq, 32768);
    tc::bulk_load(smem + GR_KQ, a.KQimg + (size_t)(c * a.geo.Hk + hk) * 32768, 32768, &bar_kq);
    issue_head(0);
    issue_slice(0);
  }
  uint32_t ph_mma = 0;
  bool ok = wait_all(&bar_kq, 0, a.err, 30);
  const uint32_t kq = tc::smem_u32(smem + GR_KQ);
  // K K^T (the same for every value head of the group): the image's K row groups (2 KB each) copied
  // unchanged into a K-only tile (the swizzle is relative to 1 KB, so whole groups keep it), then
  // [K; Q] K^T in eight MMAs; consumed by the finalizes
  if (ok) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int o = (tid + 256 * u) * 16, sl = o >> 13, g = (o >> 11) & 3, rem = o & 2047;
      *reinterpret_cast<uint4*>(smem + GR_KO + o) =
          *reinterpret_cast<const uint4*>(smem + GR_KQ + sl * 16384 + g * 4096 + rem);
    }
  }
  tc::fence_async_smem();
  ok = __syncthreads_and(ok) != 0;
  if (ok && tid == 0) {
    tc::fence_after_sync();
    const uint32_t ko = tc::smem_u32(smem + GR_KO), idK = tc::idesc(tc::kBF16, 128, 64, false, false);
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks)
      tc::mma_bf16(tmem + cKK, tc::desc_kmajor(kq, 128, ks), tc::desc_kmajor(ko, 64, ks), idK, ks > 0 ? 1u : 0u);
    tc::mma_commit(&bar_kk);
  }
  const uint32_t idC1 = tc::idesc(tc::kTF32, 128, 128, false, true);
  const uint32_t idC2 = tc::idesc(tc::kTF32, 64, 128, false, true);
  const uint32_t idC3 = tc::idesc(tc::kTF32, 128, 64, false, false);
  const uint32_t idF1 = tc::idesc(tc::kBF16, 128, 128, false, true);
  const uint32_t idF2 = tc::idesc(tc::kBF16, 64, 128, true, true);

  for (int r = 0; r < ratio && ok; ++r) {
    const int hv = hk * ratio + r;
    ok = wait_all(&bar_h, (uint32_t)(r & 1), a.err, 31);
    if (!ok) break;
    const float* sg = sgt[r & 1];
    const float bi = sg[i_row], be = sg[64 + i_row], gi = __expf(bi), bC = sg[63], lam = __expf(bC - bi);
    float t5 = 0.f;   // sum of S (.) dS over this thread's elements
    float fv = 0.f;   // lower lanes: F_i . V_i over this thread's value rows
    // the finalize's per-row inputs of the gate chain rule, loaded now (consumed at the end of the head)
    float in0 = 0.f, in1 = 0.f, eA = 0.f, dtb = 0.f;
    if (tid < 64 && tid < L) {
      const int64_t gi_idx = (tok0 + tid) * Hv + hv;
      if (a.g) {
        in0 = __ldg(a.g + gi_idx);
      } else {
        in0 = __ldg(a.a_raw + gi_idx);
        in1 = __ldg(a.b_raw + gi_idx);
        eA = __ldg(a.A_log + hv);
        dtb = __ldg(a.dt_bias + hv);
      }
    }

    for (int sl = 0; sl < NSL && ok; ++sl) {
      const int q = r * NSL + sl, bs = q & 1;
      uint8_t* buf = smem + GR_BUF + bs * GR_BS;
      // each thread waits for the slice's data itself; the barrier at the end of the slice keeps the
      // buffers' reuse ordered and makes a failed wait everyone's
      ok = ok && tc::mbar_wait(&bar_s[bs], (uint32_t)((q >> 1) & 1), a.err, 37);
      // the other buffer's last reader has finished (the finalize uses the second buffer, so the next
      // value head's first slice goes out during this head's last slice)
      if (ok && tid == 32 && q + 1 < ratio * NSL) issue_slice(q + 1);
      // a. over the slice's value rows (tf32, K = 32; every operand arrives in its final form): [dO; F] S,
      //    D dS (M = 64 in the upper lanes), [dO; F] D^T -- issued at once
      if (tid == 0 && ok) {
        tc::fence_after_sync();
        const uint32_t s32 = tc::smem_u32(buf), d32 = tc::smem_u32(buf + 16384);
        const uint32_t aa = tc::smem_u32(buf + 32768), dt = tc::smem_u32(buf + 49152);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_tf32(tmem + cA1, tc::desc_kmajor(aa, 128, ks), tc::desc_mnmajor(s32, DVT, ks, 8), idC1,
                       (sl > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_tf32(tmem + cA2 + (16u << 16), tc::desc_kmajor(dt, 64, ks), tc::desc_mnmajor(d32, DVT, ks, 8), idC2,
                       (sl > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_tf32(tmem + cPF, tc::desc_kmajor(aa, 128, ks), tc::desc_kmajor(dt, 64, ks), idC3,
                       (sl > 0 || ks > 0) ? 1u : 0u);
        tc::mma_commit(&bar_mma);
      }
      // b. meanwhile: t5 = S (.) dS, and F_i . V_i (lower lanes)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = tid + 256 * u;
        const float4 sv = reinterpret_cast<const float4*>(buf)[idx];
        const float4 dvv = reinterpret_cast<const float4*>(buf + 16384)[idx];
        t5 += sv.x * dvv.x + sv.y * dvv.y + sv.z * dvv.z + sv.w * dvv.w;
      }
      {  // the lower lane of the pair takes columns 0-7, the upper one 8-15 (summed in the finalize)
        const int hc = lower ? 0 : 1, r = img_row(i_row) + 16;
        const uint8_t* frow = buf + 32768 + r * 128;
        const float4 f0 = *reinterpret_cast<const float4*>(frow + (((4 * half + 2 * hc) ^ (r & 7)) << 4));
        const float4 f1 = *reinterpret_cast<const float4*>(frow + (((4 * half + 2 * hc + 1) ^ (r & 7)) << 4));
        const uint4 w = rvalid ? reinterpret_cast<const uint4*>(buf + 57344 + i_row * 64 + 32 * half)[hc]
                               : make_uint4(0, 0, 0, 0);
        const float f[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        const uint32_t u4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&u4[e]);
          fv = fmaf(f[2 * e], __low2float(h2), fv);
          fv = fmaf(f[2 * e + 1], __high2float(h2), fv);
        }
      }
      ok = __syncthreads_and(ok && tc::mbar_wait(&bar_mma, ph_mma, a.err, 34)) != 0;
      ph_mma ^= 1;
      tc::fence_after_sync();
    }
    if (!ok) break;

    // e. finalize this value head
    // e1. the row terms from the unscaled products, and their scaled sum into dQ (lower lanes) and dK
    //     (upper lanes), 64 columns per thread in two passes of 32
    {
      float ta = 0.f, tb = 0.f;  // lower: Q . dO S; upper: K . F S and K . D dS
      const float wa = lower ? gi : -be * gi;
#pragma unroll 1
      for (int m = 0; m < 2; ++m) {
        const int col = 64 * half + 32 * m;
        float x1[32], x2[32], kqr[32];
        tc::tmem_ld32(tl + cA1 + col, x1);
        tc::tmem_ld32(tl + cA2 + col, x2);
        ld_img_row32(smem + GR_KQ + half * 16384, img_row(i_row) + (lower ? 16 : 0), m, kqr);
        float q0[32];
        if (r > 0) tc::tmem_ld32(tl + cQK + col, q0);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          ta = fmaf(kqr[j], x1[j], ta);
          tb = fmaf(kqr[j], x2[j], tb);
          const float w = wa * x1[j] + (lower ? 0.f : lam * x2[j]);
          q0[j] = r > 0 ? q0[j] + w : w;
        }
        tc::tmem_st32(tl + cQK + col, q0);
      }
      tc::tmem_wait_st();
      fv += __shfl_xor_sync(0xffffffffu, fv, 16);
      if (lower) {
        srow[0][half][i_row] = ta;   // t3
        srow[1][half][i_row] = fv;   // F . V
      } else {
        srow[2][half][i_row] = ta;   // t2
        srow[3][half][i_row] = tb;   // t4
      }
    }
    ok = wait_all(&bar_kk, 0u, a.err, 35);
    if (!ok) break;
    tc::fence_after_sync();
    float* scratch = reinterpret_cast<float*>(smem + GR_SCR);  // [64][65], then 4 x 64 column partials
    float rsum = 0.f, dbl = 0.f;
    {
      // Lane l holds dP[i][32 half + 0..31], lane l + 16 holds F D^T there; one exchange leaves each
      // lane both for 16 columns: j0 = 32 half (lower lane), 32 half + 16 (upper lane).  K K^T row i
      // is in lane l alone; its second 16 columns go to lane l + 16.
      float v[32], kk32[32], dp[16], fd[16], kk[16];
      tc::tmem_ld32(tl + cPF + 32 * half, v);
      tc::tmem_ld32(tl + cKK + 32 * half, kk32);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float x = __shfl_xor_sync(0xffffffffu, lower ? v[16 + k] : v[k], 16);
        const float y = __shfl_xor_sync(0xffffffffu, kk32[16 + k], 16);
        dp[k] = lower ? v[k] : x;
        fd[k] = lower ? x : v[16 + k];
        kk[k] = lower ? kk32[k] : y;
      }
      const int j0 = 32 * half + (lower ? 0 : 16);
      // this row's P (hi + lo from the image) for the 16 columns, loaded up front
      float pv[16];
      {
        const int rr = img_row(i_row);
        const uint8_t* prow = smem + GR_P + rr * 128;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int ch = (j0 >> 3) + cc;
          const uint4 hi = *reinterpret_cast<const uint4*>(prow + ((ch ^ (rr & 7)) << 4));
          const uint4 lo = *reinterpret_cast<const uint4*>(prow + 2048 + ((ch ^ (rr & 7)) << 4));
          const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w}, lw[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&hw[e]);
            const __nv_bfloat162 l2 = *reinterpret_cast<const __nv_bfloat162*>(&lw[e]);
            pv[8 * cc + 2 * e] = __low2float(h2) + __low2float(l2);
            pv[8 * cc + 2 * e + 1] = __high2float(h2) + __high2float(l2);
          }
        }
      }
      float ph[16], kh[16], xs[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int j = j0 + k;
        const float gam = j <= i_row ? __expf(bi - sg[j]) : 0.f;
        const float xp = j <= i_row ? dp[k] * pv[k] : 0.f;
        const float dl = j < i_row ? -fd[k] : 0.f;
        const float lv = gam * kk[k];  // L_ij / beta_i = Gamma_ij (K K^T)_ij
        const float xl = dl * be * lv;
        dbl = fmaf(dl, lv, dbl);
        xs[k] = xp + xl;
        rsum += xs[k];
        ph[k] = dp[k] * gam;        // dP^
        kh[k] = dl * be * gam;      // dKK
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) scratch[i_row * 65 + j0 + k] = xs[k];
      const int rr = img_row(i_row), c0 = j0 >> 3;
      st_hilo16_chunks(smem + GR_FHI, smem + GR_FLO, rr, ph, c0);
      st_hilo16_chunks(smem + GR_FHI, smem + GR_FLO, rr + 16, kh, c0);
    }
    {  // the row sums of both lanes of the pair, per column half
      const float rs = rsum + __shfl_xor_sync(0xffffffffu, rsum, 16);
      const float db2 = dbl + __shfl_xor_sync(0xffffffffu, dbl, 16);
      if (lower) {
        srow[4][half][i_row] = rs;
        srow[5][half][i_row] = db2;
      }
    }
    {
      float t5w = t5;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t5w += __shfl_xor_sync(0xffffffffu, t5w, o);
      if (lane == 0) sred[warp] = t5w;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // the P image has been read: the next value head's P and gates (into the other gate buffer)
    if (tid == 32 && r + 1 < ratio) issue_head(r + 1);
    if (tid == 0) {
      // dQ | dK += [dP^; dKK] K (hi then lo);  dK += dP^^T Q + dKK^T K  (M = 64, upper lanes)
      const uint32_t fhi = tc::smem_u32(smem + GR_FHI), flo = tc::smem_u32(smem + GR_FLO);
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const uint32_t f = m ? flo : fhi;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + cQK, tc::desc_kmajor(f, 128, ks), desc_kq_t(kq, 0, ks), idF1, 1u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + cQK + (16u << 16), desc_img_t(f, 0, ks), desc_kq_t(kq, 1, ks), idF2, 1u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + cQK + (16u << 16), desc_img_t(f, 1, ks), desc_kq_t(kq, 0, ks), idF2, 1u);
      }
      tc::mma_commit(&bar_mma);
    }
    // column sums of the Gamma terms (fixed order: four 16-row partials, then their sum); row totals; d b
    {
      const int col = tid & 63, part = tid >> 6;
      float cs = 0.f;
#pragma unroll 4
      for (int i = 16 * part; i < 16 * part + 16; ++i) cs += scratch[i * 65 + col];
      scratch[64 * 65 + part * 64 + col] = cs;
    }
    __syncthreads();
    float lt4 = 0.f, dbv = 0.f;
    if (tid < 64) {
      const int i = tid;
      const float* cp = scratch + 64 * 65;
      const float csum = (cp[i] + cp[64 + i]) + (cp[128 + i] + cp[192 + i]);
      const float bi_ = sg[i], be_ = sg[64 + i], gi_ = __expf(bi_), lam_ = __expf(bC - bi_);
      const float t3_ = srow[0][0][i] + srow[0][1][i];
      const float t2_ = srow[2][0][i] + srow[2][1][i];
      const float t4_ = srow[3][0][i] + srow[3][1][i];
      const float rs = srow[4][0][i] + srow[4][1][i];
      dbv = rs - csum + gi_ * t3_ - be_ * gi_ * t2_ - lam_ * t4_;
      lt4 = lam_ * t4_;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lt4 += __shfl_xor_sync(0xffffffffu, lt4, o);
    if (lane == 0 && warp < 2) sred[8 + warp] = lt4;
    __syncthreads();
    if (tid == 63) {
      float st5 = 0.f;
      for (int w = 0; w < 8; ++w) st5 += sred[w];
      dbv += (sred[8] + sred[9]) + __expf(bC) * st5;
    }
    // d log g_i = sum over rows i' >= i of d b_i': a suffix scan over the 64 rows (two warps)
    if (tid < 64) {
      float x = dbv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, x, o);
        if (lane + o < 32) x += y;
      }
      if (tid == 32) sdb[0] = x;  // the upper warp's total (rows 32..63)
      sdb[1 + tid] = x;
    }
    __syncthreads();
    float pa = 0.f, pd = 0.f;  // layer mode: this row's share of the head's dA_log, ddt_bias
    if (tid < 64 && tid < L) {
      const int i = tid;
      const float dl = sdb[1 + i] + (i < 32 ? sdb[0] : 0.f);  // d log g_i
      const int64_t gi_idx = (tok0 + i) * Hv + hv;
      // d beta = F . (V - gamma R) + the L terms;  F . R = K . (F S) = t2
      const float gi_ = __expf(sg[i]);
      const float t1_ = (srow[1][0][i] + srow[1][1][i]) - gi_ * (srow[2][0][i] + srow[2][1][i]);
      const float dbe = t1_ + srow[5][0][i] + srow[5][1][i];
      if (a.g) {
        // dg = d log g / g; a gate of exactly 0 (log g clamped) gets 0, which keeps g * dg = 0 exact
        a.dg[gi_idx] = in0 > 0.f ? dl / in0 : 0.f;
        a.dbeta[gi_idx] = dbe;
      } else {
        // log g = -e^A softplus(x), x = a + dt_bias: da = d log g * (-e^A sigmoid(x)); beta = sigmoid(b)
        const float ea = expf(eA), x = in0 + dtb;
        const float da = dl * (-ea * sigmoid_f(x));
        const float sb_ = sigmoid_f(in1);
        a.dg[gi_idx] = da;
        a.dbeta[gi_idx] = dbe * sb_ * (1.f - sb_);
        pa = dl * (-ea * softplus_f(x));
        pd = da;
      }
    }
    if (!a.g) {  // fixed-order block sums of the head parameters' gradients for this chunk
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        pa += __shfl_xor_sync(0xffffffffu, pa, o);
        pd += __shfl_xor_sync(0xffffffffu, pd, o);
      }
      if (lane == 0 && warp < 2) {
        sred[12 + warp] = pa;
        sred[14 + warp] = pd;
      }
      __syncthreads();
      if (tid == 0) {
        a.head_part[(c * Hv + hv) * 2] = sred[12] + sred[13];
        a.head_part[(c * Hv + hv) * 2 + 1] = sred[14] + sred[15];
      }
    }
    tc::fence_async_smem();  // the scratch writes before the next TMA into this buffer
    ok = wait_all(&bar_mma, ph_mma, a.err, 36);
    ph_mma ^= 1;
    tc::fence_after_sync();
  }
  // f. dq (lower lanes) and dk (upper lanes) rows of this key head, 64 columns per thread (layer mode:
  //    through the norms to the raw q, k)
  if (!a.g) cp_async_wait_all();
  if (ok) {
    Tout* out = static_cast<Tout*>(lower ? a.dq : a.dk) + rowoff;
    float v0[32], v1[32];
    tc::tmem_ld32(tl + cQK + 64 * half, v0);
    tc::tmem_ld32(tl + cQK + 64 * half + 32, v1);
    if (!a.g) {
      // x^ = s bf16(x r), r = rsqrt(mean(x^2) + eps):  dx = s r (dx^ - r^2 (x . dx^) x / Dk)
      float x0[32], x1[32];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 w = make_uint4(0, 0, 0, 0);
        if (rvalid) w = *reinterpret_cast<const uint4*>(rawrow + ((cc ^ (i_row & 7)) << 4));
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
        float* xd = cc < 4 ? x0 + 8 * cc : x1 + 8 * (cc - 4);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
          xd[2 * e] = __low2float(h);
          xd[2 * e + 1] = __high2float(h);
        }
      }
      float ss = 0.f, dot = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        ss = fmaf(x0[j], x0[j], fmaf(x1[j], x1[j], ss));
        dot = fmaf(x0[j], v0[j], fmaf(x1[j], v1[j], dot));
      }
      const int ln = 32 * quad + lane;
      snorm[0][half][ln] = ss;
      snorm[1][half][ln] = dot;
      __syncthreads();
      ss += snorm[0][half ^ 1][ln];
      dot += snorm[1][half ^ 1][ln];
      const float rn = rsqrtf(ss / DK + 1e-6f);
      const float sc = lower ? 1.f / DK : __bfloat162float(__float2bfloat16_rn(rsqrtf((float)DK)));
      const float c2 = rn * rn * dot / DK;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v0[j] = sc * rn * (v0[j] - c2 * x0[j]);
        v1[j] = sc * rn * (v1[j] - c2 * x1[j]);
      }
    }
    if (rvalid) {
      store_row32<Tout>(out, v0);
      store_row32<Tout>(out + 32, v1);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
  if (!a.g) {
    // layer mode: the CTA that finishes last sums every chunk's head terms, in chunk order (the same
    // result whichever CTA it is):  dA_log[h], ddt_bias[h] = sum over chunks of head_part[c][h][0 | 1]
    if (tid == 0) {
      __threadfence();
      s_last = atomicAdd(a.done, 1u) == gridDim.x * gridDim.y - 1;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int64_t nc = gridDim.x;
      for (int j = tid; j < 2 * Hv; j += blockDim.x) {
        const float* p = a.head_part + j;  // head j >> 1, term j & 1
        float s = 0.f;
        int64_t cc = 0;
        for (; cc + 8 <= nc; cc += 8) {
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = __ldcg(p + (cc + e) * Hv * 2);
#pragma unroll
          for (int e = 0; e < 8; ++e) s += x[e];
        }
        for (; cc < nc; ++cc) s += __ldcg(p + cc * Hv * 2);
        ((j & 1) ? a.ddt_bias : a.dA_log)[j >> 1] = s;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Host side.
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// [rows, heads, dim] bf16 activations; box = 64 columns x 1 head x 64 rows, 128-byte swizzle.
bool map_act(CUtensorMap* m, const void* base, int64_t rows, int heads, int dim, int box_rows = 64) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)dim * 2, (cuuint64_t)heads * dim * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 rows [rows, heads, dim] read as unswizzled boxes of box_cols x box_rows of one head (the
// value or output-gradient rows of a chunk); rows past the end read as zero.
bool map_rows(CUtensorMap* m, const void* base, int64_t rows, int heads, int dim, int box_cols, int box_rows,
              bool f32 = false) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  const cuuint64_t eb = f32 ? 4 : 2;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)dim * eb, (cuuint64_t)heads * dim * eb};
  cuuint32_t box[3] = {(cuuint32_t)box_cols, 1, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  return f(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
           dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// State rows [rows, 128] fp32 (a chunk-state buffer); box = 32 columns x 32 rows in the 32-byte-atom
// swizzle: four boxes make the MN-major tf32 operand of a 32-row slice.
bool map_state_mn(CUtensorMap* m, const void* base, int64_t rows) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  cuuint64_t strides[1] = {128 * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t a256(int64_t x) { return (x + 255) & ~int64_t(255); }

// The chunk intermediates: [ckpt][gates] fp32, the forward's T, P and [K; Q] operand images and its
// tf32-rounded D tiles.
struct Saved {
  float *ckpt, *gates;
  uint8_t *Timg, *Pimg, *KQimg;
  float* Ds;
};

int64_t saved_layout(int Hv, int Hk, int64_t n_chunks, char* base, Saved* s) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* at = base ? base + off : nullptr;
    off += a256(bytes);
    return at;
  };
  Saved x;
  x.ckpt = (float*)take(n_chunks * Hv * (int64_t)DV * DK * 4);
  x.gates = (float*)take(n_chunks * Hv * 128 * 4);
  x.Timg = (uint8_t*)take(n_chunks * Hv * 16384);
  x.Pimg = (uint8_t*)take(n_chunks * Hv * 16384);
  x.KQimg = (uint8_t*)take(n_chunks * Hk * 32768);
  x.Ds = (float*)take(n_chunks * Hv * 64 * DV * 4);
  if (s) *s = x;
  return off;
}

// Workspace: [chunk_off][err][fwd: T, P and [K; Q] images, gates when nothing is saved | bwd: dS per
// chunk, per-chunk head sums (layer mode), and a saved buffer plus forward workspace when the backward
// recomputes].
struct Ws {
  int64_t* chunk_off;
  int* err;          // 4 words, zeroed by each call: [0] the error code, [2] the gradient kernel's CTA count
  uint8_t *Timg, *Pimg, *KQimg;
  float* gates;
  float* dsbuf;
  uint8_t* Aimg;     // [dO; F] operand images from the reverse walk, [chunks, Hv, 4] x 16 KB
  float* head_part;
  char* saved;
  char* fwd_ws;
};

int64_t ws_layout(int Hv, int Hk, int N, int64_t n_chunks, bool layer, bool varlen, int op, bool with_saved,
                  char* base, Ws* w) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* at = base ? base + off : nullptr;
    off += a256(bytes);
    return at;
  };
  Ws x{};
  x.chunk_off = (int64_t*)take(varlen ? (int64_t)(N + 1) * 8 : 0);
  x.err = (int*)take(16);
  if (op == 0) {
    x.Timg = (uint8_t*)take(n_chunks * Hv * 16384);
    x.Pimg = (uint8_t*)take(n_chunks * Hv * 16384);
    x.KQimg = (uint8_t*)take(n_chunks * Hk * 32768);
    x.gates = (float*)take(n_chunks * Hv * 128 * 4);
  } else {
    x.dsbuf = (float*)take(n_chunks * Hv * (int64_t)DV * DK * 4);
    x.Aimg = (uint8_t*)take(n_chunks * Hv * (DV / DVT) * 16384);
    x.head_part = (float*)take(layer ? n_chunks * Hv * 2 * 4 : 0);
    if (with_saved) {
      x.saved = take(saved_layout(Hv, Hk, n_chunks, nullptr, nullptr));
      x.fwd_ws = take(ws_layout(Hv, Hk, N, n_chunks, layer, varlen, 0, false, nullptr, nullptr));
    }
  }
  if (w) *w = x;
  return off;
}

}  // namespace

bool chunked_supported(int Dk, int Dv) { return Dk == DK && Dv == DV && encode_fn() != nullptr; }
bool chunked_bwd_ready() { return true; }

int64_t chunked_saved_bytes(int Hv, int Hk, int64_t n_chunks, int64_t tokens, bool layer) {
  return saved_layout(Hv, Hk, n_chunks, nullptr, nullptr);
}

int64_t chunked_ws_bytes(int Hv, int Hk, int N, int64_t n_chunks, int64_t tokens, bool varlen, int op, bool with_saved,
                         bool layer) {
  return ws_layout(Hv, Hk, N, n_chunks, layer, varlen, op, with_saved, nullptr, nullptr);
}

cudaError_t chunked_fwd(const ChunkFwdArgs& a, void* ws, cudaStream_t st) {
  if (!a.in_bf16) return cudaErrorInvalidValue;
  const bool layer = a.g == nullptr;
  const int64_t rows = (int64_t)a.B * a.T;
  Ws w;
  ws_layout(a.Hv, a.Hk, a.N, a.n_chunks, layer, a.cu != nullptr, 0, false, (char*)ws, &w);
  Saved sv{};
  float *gates = w.gates, *ckpt = nullptr;
  uint8_t *Ti = w.Timg, *Pi = w.Pimg, *KQi = w.KQimg;
  if (a.saved) {
    saved_layout(a.Hv, a.Hk, a.n_chunks, (char*)a.saved, &sv);
    gates = sv.gates, ckpt = sv.ckpt;
    Ti = sv.Timg, Pi = sv.Pimg, KQi = sv.KQimg;
  }
  cudaError_t e;
  if ((e = cudaMemsetAsync(w.err, 0, 16, st)) != cudaSuccess) return e;
  if (a.cu && (e = launch_chunk_offsets(a.cu, a.N, w.chunk_off, st)) != cudaSuccess) return e;
  CUtensorMap kmap, qmap;
  if (!map_act(&kmap, a.k, rows, a.Hk, a.Dk) || !map_act(&qmap, a.q, rows, a.Hk, a.Dk)) return cudaErrorInvalidValue;
  Geo geo{a.T, a.Hk, a.Hv, a.N, (a.T + C - 1) / C, a.cu, a.cu ? w.chunk_off : nullptr};
  if (a.n_chunks > 0) {
    PrepArgs pa{geo, a.g, a.beta, a.a_raw, a.b_raw, a.A_log, a.dt_bias, Ti, Pi, KQi, gates, w.err};
    const int prep_smem = 1024 + 32768;
    if ((e = cudaFuncSetAttribute(gdn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem)) !=
        cudaSuccess)
      return e;
    gdn_chunk_prep<<<dim3((unsigned)a.n_chunks, a.Hk), 128, prep_smem, st>>>(kmap, qmap, pa);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  CUtensorMap vmap, ymap;
  if (!map_rows(&vmap, a.v, rows, a.Hv, a.Dv, DVT, C) || !map_rows(&ymap, a.y, rows, a.Hv, a.Dv, DVT, C, !a.out_bf16))
    return cudaErrorInvalidValue;
  StateArgs sa{geo, a.v, gates, a.h0, a.y, a.hT, ckpt, Ti, Pi, KQi, a.saved ? sv.Ds : nullptr, w.err};
  auto kern = a.out_bf16 ? gdn_chunk_fwd_state<__nv_bfloat16> : gdn_chunk_fwd_state<float>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FW_SMEM)) != cudaSuccess) return e;
  kern<<<dim3(DV / DVT, a.Hv, a.N), 256, FW_SMEM, st>>>(vmap, ymap, sa);
  note_launch();
  return cudaGetLastError();
}

cudaError_t chunked_bwd(const ChunkBwdArgs& a, void* ws, cudaStream_t st) {
  if (!a.in_bf16) return cudaErrorInvalidValue;
  const bool layer = a.g == nullptr;
  const int64_t rows = (int64_t)a.B * a.T;
  Ws w;
  ws_layout(a.Hv, a.Hk, a.N, a.n_chunks, layer, a.cu != nullptr, 1, a.saved == nullptr, (char*)ws, &w);
  cudaError_t e;
  const void* saved = a.saved;
  if (!saved) {  // recompute the forward's intermediates with the same forward (y is discarded into dv)
    ChunkFwdArgs f{};
    f.B = a.B, f.T = a.T, f.Hk = a.Hk, f.Hv = a.Hv, f.Dk = a.Dk, f.Dv = a.Dv, f.N = a.N, f.n_chunks = a.n_chunks;
    f.cu = a.cu, f.q = a.q, f.k = a.k, f.v = a.v, f.g = a.g, f.beta = a.beta, f.h0 = a.h0, f.y = a.dv;
    f.saved = w.saved, f.in_bf16 = a.in_bf16, f.out_bf16 = a.out_bf16;
    f.a_raw = a.a_raw, f.b_raw = a.b_raw, f.A_log = a.A_log, f.dt_bias = a.dt_bias;
    if ((e = chunked_fwd(f, w.fwd_ws, st)) != cudaSuccess) return e;
    saved = w.saved;
  }
  Saved sv;
  saved_layout(a.Hv, a.Hk, a.n_chunks, (char*)saved, &sv);
  if ((e = cudaMemsetAsync(w.err, 0, 16, st)) != cudaSuccess) return e;
  if (a.cu && (e = launch_chunk_offsets(a.cu, a.N, w.chunk_off, st)) != cudaSuccess) return e;
  Geo geo{a.T, a.Hk, a.Hv, a.N, (a.T + C - 1) / C, a.cu, a.cu ? w.chunk_off : nullptr};
  CUtensorMap dmap, vmap, dvmap;
  if (!map_rows(&dmap, a.dy, rows, a.Hv, a.Dv, DVT, C) || !map_rows(&vmap, a.v, rows, a.Hv, a.Dv, DVT, C) ||
      !map_rows(&dvmap, a.dv, rows, a.Hv, a.Dv, DVT, C, !a.out_bf16))
    return cudaErrorInvalidValue;
  BwdStateArgs ba{geo, a.dy, sv.gates, a.dhT, a.dv, a.dh0, w.dsbuf, sv.Timg, sv.Pimg, sv.KQimg, w.Aimg, w.err};
  auto k1 = a.out_bf16 ? gdn_chunk_bwd_state<__nv_bfloat16> : gdn_chunk_bwd_state<float>;
  if ((e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM)) != cudaSuccess) return e;
  k1<<<dim3(DV / DVT, a.Hv, a.N), 256, BW_SMEM, st>>>(dmap, dvmap, ba);
  note_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (a.n_chunks == 0) {
    if (layer) {
      if ((e = cudaMemsetAsync(a.dA_log, 0, a.Hv * 4, st)) != cudaSuccess) return e;
      if ((e = cudaMemsetAsync(a.ddt_bias, 0, a.Hv * 4, st)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  CUtensorMap smap_mn, dmap_mn;
  if (!map_state_mn(&smap_mn, sv.ckpt, a.n_chunks * a.Hv * (int64_t)DV) ||
      !map_state_mn(&dmap_mn, w.dsbuf, a.n_chunks * a.Hv * (int64_t)DV))
    return cudaErrorInvalidValue;
  GradArgs ga{geo, a.g, sv.gates, sv.Pimg, sv.KQimg, sv.Ds, w.Aimg, a.dq, a.dk, a.dg, a.dbeta, w.err,
              static_cast<const __nv_bfloat16*>(a.q), static_cast<const __nv_bfloat16*>(a.k),
              a.a_raw, a.b_raw, a.A_log, a.dt_bias, w.head_part, a.dA_log, a.ddt_bias,
              reinterpret_cast<unsigned*>(w.err + 2)};
  auto k2 = a.out_bf16 ? gdn_chunk_bwd_grad<__nv_bfloat16> : gdn_chunk_bwd_grad<float>;
  if ((e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, GR_SMEM)) != cudaSuccess) return e;
  k2<<<dim3((unsigned)a.n_chunks, a.Hk), 256, GR_SMEM, st>>>(smap_mn, dmap_mn, vmap, ga);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
