// Tensor-core chunked path of the Gated DeltaNet recurrence (Dk = Dv = 128, bf16 activations),
// sm_100a: TMA tile loads, tcgen05 MMAs with TMEM accumulators, chunk C = 64.
//
// Per value head and chunk (local steps i, j < C; b = inclusive cumsum of log g inside the chunk,
// gamma = exp(b); rows past the sequence end carry k = q = v = 0, beta = 0, log g = 0):
//   L  = strictly-lower(beta_i exp(b_i - b_j) (K K^T)_ij),   T = (I + L)^-1
//   P  = lower-incl(exp(b_i - b_j) (Q K^T)_ij)
//   E  = diag(beta) (V - diag(gamma) K S^T)                  (S: the chunk-start state, Dv x Dk)
//   D  = T E                                                  (the chunk's delta rows)
//   O  = diag(gamma) Q S^T + P D
//   S' = gamma_C S + (diag(exp(b_C - b)) D)^T K
// This is the recurrence of src/delta_grad.cpp:13-14 (S~ = g S; u = S~ k; delta = beta (v - u);
// S = S~ + delta k^T; y = S q) applied to 64 steps at once (the WY / UT form).
//
// Kernels:
//   gdn_chunk_prep       grid (chunks, Hv): K K^T on the tensor cores, the triangular inverse T by
//                        forward substitution, the chunk's cumulative log gates.  Fully parallel.
//   gdn_chunk_fwd_state  grid (Dv/32, Hv, sequences): walks the chunks of a sequence in order with a
//                        32-row slice of the state in registers; per chunk three tcgen05 rounds
//                        (K S^T, Q S^T, Q K^T | T E | P D, K^T D~).  Writes y and, for training, the
//                        chunk-start states (the reference's ckpt, src/delta_grad.cpp:172-181).
// Operand precision: products of two inputs (K K^T, Q K^T) in bf16 (exact); an input times a computed
// tile with the computed tile split into bf16 hi + lo (about 16 mantissa bits); two computed tiles
// in tf32 (round-to-nearest).
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
constexpr int DVT = 32;     // value rows of the state per CTA in the state walk

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
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

}  // namespace

// ------------------------------------------------------------------------------------------------
// Per (chunk, value head): T = (I + L)^-1 and the gates (b, beta) of the chunk.
struct PrepArgs {
  Geo geo;
  const float *g, *beta;
  float* Tbuf;      // [chunks, Hv, 64, 64]
  float* gates;     // [chunks, Hv, 2, 64]: b then beta
  int* err;
};

__global__ void __launch_bounds__(128) gdn_chunk_prep(const __grid_constant__ CUtensorMap kmap, PrepArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ktile = smem;                                   // 16 KB bf16, two 64-column slabs
  float* Lm = reinterpret_cast<float*>(smem + 16384);      // [64][68]
  __shared__ float sb[64], sbeta[64], stmp[2];
  __shared__ uint64_t bar_tma, bar_mma;
  __shared__ uint32_t tmem_slot;
  constexpr int LS = 68;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t c = blockIdx.x;
  const int hv = blockIdx.y, hk = hv / (a.geo.Hv / a.geo.Hk);
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
    tc::mbar_arrive_expect_tx(&bar_tma, 16384);
    tc::tma_load_3d(ktile, &kmap, &bar_tma, 0, hk, (int)tok0);
    tc::tma_load_3d(ktile + 8192, &kmap, &bar_tma, 64, hk, (int)tok0);
  }
  float lg = 0.f, bt = 0.f;
  if (tid < 64 && tid < L) {
    const int64_t gi = (tok0 + tid) * a.geo.Hv + hv;
    lg = fmaxf(logf(a.g[gi]), -88.f);
    bt = a.beta[gi];
  }
  if (tid < 64) sbeta[tid] = bt;
  scan64(lg, sb, stmp);

  bool ok = __syncthreads_and(tc::mbar_wait(&bar_tma, 0, a.err, 1)) != 0;
  if (ok && tid == 0) {
    tc::fence_after_sync();
    tc::mma_tile<tc::kBF16>(tmem, tc::smem_u32(ktile), false, 64, tc::smem_u32(ktile), false, 64, 64, 64, DK, false);
    tc::mma_commit(&bar_mma);
  }
  ok = __syncthreads_and(ok && tc::mbar_wait(&bar_mma, 0, a.err, 2)) != 0;
  tc::fence_after_sync();
  if (ok) {
    const int i = 16 * warp + (lane & 15);
    float v[32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, 32 * h), v);
      if (lane < 16) {
        const float bi = sb[i], be = sbeta[i];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * h + jj;
          Lm[i * LS + j] = j < i ? be * __expf(bi - sb[j]) * v[jj] : 0.f;
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (ok && tid < 64) {
    // column `col` of T = (I + L)^-1 by forward substitution, kept in registers
    const int col = tid;
    float t[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      float s = (i == col) ? 1.f : 0.f;
      const float* Li = Lm + i * LS;
#pragma unroll
      for (int j = 0; j < i; ++j) s = fmaf(-Li[j], t[j], s);
      t[i] = s;
    }
    // the state walk feeds T to tf32 MMAs: round to nearest here rather than let the operand read drop bits
#pragma unroll
    for (int i = 0; i < 64; ++i) t[i] = tf32_rna(t[i]);
    float* dst = a.Tbuf + ((c * a.geo.Hv + hv) * 64) * 64;
#pragma unroll
    for (int i = 0; i < 64; ++i) dst[i * 64 + col] = t[i];
    float* gd = a.gates + (c * a.geo.Hv + hv) * 128;
    gd[tid] = sb[tid];
    gd[64 + tid] = sbeta[tid];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------------------------------------------
// The state walk.  One CTA per (32 value rows, value head, sequence); thread t holds column t of
// the 32 state rows (S^T[t][0..31]) in registers.
struct StateArgs {
  Geo geo;
  const void* v;          // [B*T, Hv, Dv] bf16
  const float* gates;     // [chunks, Hv, 2, 64]
  const float* h0;        // [N, Hv, Dv, Dk] or null
  void* y;                // [B*T, Hv, Dv] (bf16 or fp32)
  float* hT;              // or null
  float* ckpt;            // [chunks, Hv, Dv, Dk] chunk-start states, or null
  int out_bf16;
  int* err;
};

// Shared-memory plan of the state walk (bytes from a 1024-aligned base).
constexpr int SM_K = 0;            // 2 x 16 KB bf16 K tiles (TMA)
constexpr int SM_Q = 32768;        // 2 x 16 KB bf16 Q tiles (TMA)
constexpr int SM_T = 65536;        // 2 x 16 KB fp32 T tiles (TMA)
constexpr int SM_SHI = 98304;      // 8 KB bf16 state hi, K-major [32][128]
constexpr int SM_SLO = 106496;     // 8 KB bf16 state lo
constexpr int SM_E = 114688;       // 8 KB fp32 E, MN-major [64][32]
constexpr int SM_P = 122880;       // 16 KB fp32 P, K-major [64][64]
constexpr int SM_D = 139264;       // 8 KB fp32 D, MN-major [64][32]
constexpr int SM_DHI = 147456;     // 8 KB bf16 D~ hi, MN-major [64][32]
constexpr int SM_DLO = 155648;     // 8 KB bf16 D~ lo
constexpr int SM_STATE_BYTES = 163840;
constexpr int STATE_SMEM = SM_STATE_BYTES + 1024;

template <bool OUT_BF16>
__global__ void __launch_bounds__(128, 1) gdn_chunk_fwd_state(const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap tmap,
                                                              StateArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ float sg[2][128];
  __shared__ uint64_t bar_tma[2], bar_mma;
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dv0 = blockIdx.x * DVT, hv = blockIdx.y, n = blockIdx.z;
  const int Hv = a.geo.Hv, hk = hv / (Hv / a.geo.Hk);
  int64_t c_first, nchunks;
  if (a.geo.cu) {
    c_first = a.geo.chunk_off[n];
    nchunks = a.geo.chunk_off[n + 1] - c_first;
  } else {
    c_first = (int64_t)n * a.geo.ncs;
    nchunks = a.geo.ncs;
  }
  const int64_t seq0 = a.geo.cu ? a.geo.cu[n] : (int64_t)n * a.geo.T;
  const int64_t seq1 = a.geo.cu ? a.geo.cu[n + 1] : (int64_t)n * a.geo.T + a.geo.T;

  // TMEM columns
  const uint32_t cR = 0, cY = 32, cQK = 64, cD = 128, cO = 160, cS = 192;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 256);
  if (tid == 0) {
    tc::mbar_init(&bar_tma[0], 1);
    tc::mbar_init(&bar_tma[1], 1);
    tc::mbar_init(&bar_mma, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&kmap);
    tc::prefetch_tmap(&qmap);
    tc::prefetch_tmap(&tmap);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;

  // state slice: s[j] = S[dv0 + j][tid]
  float s[DVT];
  {
    const size_t base = ((size_t)n * Hv + hv) * DV * DK;
#pragma unroll
    for (int j = 0; j < DVT; ++j) s[j] = a.h0 ? a.h0[base + (size_t)(dv0 + j) * DK + tid] : 0.f;
  }

  auto issue_loads = [&](int64_t jc, int buf) {
    const int64_t tok = seq0 + jc * C;
    const int64_t cg = c_first + jc;
    tc::mbar_arrive_expect_tx(&bar_tma[buf], 16384 * 3);
    tc::tma_load_3d(smem + SM_K + buf * 16384, &kmap, &bar_tma[buf], 0, hk, (int)tok);
    tc::tma_load_3d(smem + SM_K + buf * 16384 + 8192, &kmap, &bar_tma[buf], 64, hk, (int)tok);
    tc::tma_load_3d(smem + SM_Q + buf * 16384, &qmap, &bar_tma[buf], 0, hk, (int)tok);
    tc::tma_load_3d(smem + SM_Q + buf * 16384 + 8192, &qmap, &bar_tma[buf], 64, hk, (int)tok);
    const int trow = (int)((cg * Hv + hv) * 64);
    tc::tma_load_2d(smem + SM_T + buf * 16384, &tmap, &bar_tma[buf], 0, trow);
    tc::tma_load_2d(smem + SM_T + buf * 16384 + 8192, &tmap, &bar_tma[buf], 32, trow);
  };

  if (nchunks > 0) {
    if (tid == 0) issue_loads(0, 0);
    sg[0][tid] = a.gates[(c_first * Hv + hv) * 128 + tid];
  }
  uint32_t mma_phase = 0;
  bool ok = true;
  const int i_row = 16 * warp + (lane & 15);  // row of the M = 64 accumulators this thread reads
  const bool row_owner = lane < 16;

  for (int64_t jc = 0; jc < nchunks && ok; ++jc) {
    const int buf = (int)(jc & 1);
    const int64_t cg = c_first + jc;
    const int64_t tok0 = seq0 + jc * C;
    const int L = (int)min((int64_t)C, seq1 - tok0);

    // 1. the chunk-start state: saved for the backward, and split into the bf16 hi/lo operand
    if (a.ckpt) {
      float* dst = a.ckpt + ((cg * Hv + hv) * DV + dv0) * (size_t)DK + tid;
#pragma unroll
      for (int j = 0; j < DVT; ++j) dst[(size_t)j * DK] = s[j];
    }
#pragma unroll
    for (int j = 0; j < DVT; ++j) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(s[j]);
      const __nv_bfloat16 lo = __float2bfloat16_rn(s[j] - __bfloat162float(hi));
      const uint32_t o = tc::off_kmajor(j, tid, DVT, 2);
      *reinterpret_cast<__nv_bfloat16*>(smem + SM_SHI + o) = hi;
      *reinterpret_cast<__nv_bfloat16*>(smem + SM_SLO + o) = lo;
    }
    // 2. this thread's value row (rows past the end read as zero)
    float vr[DVT];
    if (row_owner && i_row < L) {
      const __nv_bfloat16* vp =
          static_cast<const __nv_bfloat16*>(a.v) + ((tok0 + i_row) * Hv + hv) * (size_t)DV + dv0;
#pragma unroll
      for (int q4 = 0; q4 < DVT / 8; ++q4) {
        float t8[8];
        load_vec<8>(vp + 8 * q4, t8);
#pragma unroll
        for (int e = 0; e < 8; ++e) vr[8 * q4 + e] = t8[e];
      }
    } else {
#pragma unroll
      for (int j = 0; j < DVT; ++j) vr[j] = 0.f;
    }
    // 3. tiles of this chunk
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(tc::mbar_wait(&bar_tma[buf], (uint32_t)((jc >> 1) & 1), a.err, 10)) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // prefetch the next chunk into the other buffer (its last readers finished last iteration)
    if (jc + 1 < nchunks) {
      if (tid == 0) issue_loads(jc + 1, buf ^ 1);
      sg[buf ^ 1][tid] = a.gates[((cg + 1) * Hv + hv) * 128 + tid];
    }
    const uint32_t kt = tc::smem_u32(smem + SM_K + buf * 16384);
    const uint32_t qt = tc::smem_u32(smem + SM_Q + buf * 16384);
    const uint32_t tt = tc::smem_u32(smem + SM_T + buf * 16384);
    // 4. R = K S^T, Y = Q S^T (S split hi + lo), QK = Q K^T
    if (tid == 0) {
      const uint32_t shi = tc::smem_u32(smem + SM_SHI), slo = tc::smem_u32(smem + SM_SLO);
      tc::mma_tile<tc::kBF16>(tmem + cR, kt, false, 64, shi, false, DVT, 64, DVT, DK, false);
      tc::mma_tile<tc::kBF16>(tmem + cR, kt, false, 64, slo, false, DVT, 64, DVT, DK, true);
      tc::mma_tile<tc::kBF16>(tmem + cY, qt, false, 64, shi, false, DVT, 64, DVT, DK, false);
      tc::mma_tile<tc::kBF16>(tmem + cY, qt, false, 64, slo, false, DVT, 64, DVT, DK, true);
      tc::mma_tile<tc::kBF16>(tmem + cQK, qt, false, 64, kt, false, 64, 64, 64, DK, false);
      tc::mma_commit(&bar_mma);
    }
    ok = __syncthreads_and(tc::mbar_wait(&bar_mma, mma_phase, a.err, 11)) != 0;
    mma_phase ^= 1;
    tc::fence_after_sync();
    if (!ok) break;
    const float* gb = sg[buf];
    const float bi = gb[i_row], be = gb[64 + i_row], gi = __expf(bi);
    float yp[DVT];
    {
      float r[32];
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, cR), r);
      if (row_owner) {
#pragma unroll
        for (int j = 0; j < DVT; ++j) {
          const float e = be * (vr[j] - gi * r[j]);
          *reinterpret_cast<float*>(smem + SM_E + tc::off_mnmajor(i_row, j, 64, 4)) = tf32_rna(e);
        }
      }
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, cY), r);
#pragma unroll
      for (int j = 0; j < DVT; ++j) yp[j] = gi * r[j];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tc::tmem_ld32(tc::taddr(tmem, 32 * warp, cQK + 32 * h), r);
        if (row_owner) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int j = 32 * h + jj;
            const float p = j <= i_row ? __expf(bi - gb[j]) * r[jj] : 0.f;
            *reinterpret_cast<float*>(smem + SM_P + tc::off_kmajor(i_row, j, 64, 4)) = tf32_rna(p);
          }
        }
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // 5. D = T E
    if (tid == 0) {
      tc::mma_tile<tc::kTF32>(tmem + cD, tt, false, 64, tc::smem_u32(smem + SM_E), true, 64, 64, DVT, C, false);
      tc::mma_commit(&bar_mma);
    }
    ok = __syncthreads_and(tc::mbar_wait(&bar_mma, mma_phase, a.err, 12)) != 0;
    mma_phase ^= 1;
    tc::fence_after_sync();
    if (!ok) break;
    const float bC = gb[63];
    {
      float d[32];
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, cD), d);
      if (row_owner) {
        const float sc = __expf(bC - bi);
#pragma unroll
        for (int j = 0; j < DVT; ++j) {
          *reinterpret_cast<float*>(smem + SM_D + tc::off_mnmajor(i_row, j, 64, 4)) = tf32_rna(d[j]);
          const float dt = sc * d[j];
          const __nv_bfloat16 hi = __float2bfloat16_rn(dt);
          const __nv_bfloat16 lo = __float2bfloat16_rn(dt - __bfloat162float(hi));
          const uint32_t o = tc::off_mnmajor(i_row, j, 64, 2);
          *reinterpret_cast<__nv_bfloat16*>(smem + SM_DHI + o) = hi;
          *reinterpret_cast<__nv_bfloat16*>(smem + SM_DLO + o) = lo;
        }
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // 6. O2 = P D;  S_upd^T = K^T D~ (K as the MN-major A operand: Dk rows, chunk steps as K)
    if (tid == 0) {
      tc::mma_tile<tc::kTF32>(tmem + cO, tc::smem_u32(smem + SM_P), false, 64, tc::smem_u32(smem + SM_D), true, 64,
                              64, DVT, C, false);
      tc::mma_tile<tc::kBF16>(tmem + cS, kt, true, 64, tc::smem_u32(smem + SM_DHI), true, 64, 128, DVT, C, false);
      tc::mma_tile<tc::kBF16>(tmem + cS, kt, true, 64, tc::smem_u32(smem + SM_DLO), true, 64, 128, DVT, C, true);
      tc::mma_commit(&bar_mma);
    }
    ok = __syncthreads_and(tc::mbar_wait(&bar_mma, mma_phase, a.err, 13)) != 0;
    mma_phase ^= 1;
    tc::fence_after_sync();
    if (!ok) break;
    {
      float u[32];
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, cS), u);
      const float gC = __expf(bC);
#pragma unroll
      for (int j = 0; j < DVT; ++j) s[j] = fmaf(gC, s[j], u[j]);
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, cO), u);
      if (row_owner && i_row < L) {
        const size_t yo = ((tok0 + i_row) * Hv + hv) * (size_t)DV + dv0;
        if (OUT_BF16) {
          __nv_bfloat16* yp16 = static_cast<__nv_bfloat16*>(a.y) + yo;
#pragma unroll
          for (int q = 0; q < DVT / 8; ++q) {
            uint4 pk;
            uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 h2 =
                  __floats2bfloat162_rn(yp[8 * q + 2 * e] + u[8 * q + 2 * e], yp[8 * q + 2 * e + 1] + u[8 * q + 2 * e + 1]);
              w[e] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(yp16 + 8 * q) = pk;
          }
        } else {
          float* yp32 = static_cast<float*>(a.y) + yo;
#pragma unroll
          for (int j = 0; j < DVT; ++j) yp32[j] = yp[j] + u[j];
        }
      }
    }
    tc::fence_before_sync();
  }
  if (ok && a.hT) {
    float* dst = a.hT + (((size_t)n * Hv + hv) * DV + dv0) * DK + tid;
#pragma unroll
    for (int j = 0; j < DVT; ++j) dst[(size_t)j * DK] = s[j];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
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
bool map_act(CUtensorMap* m, const void* base, int64_t rows, int heads, int dim) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)dim * 2, (cuuint64_t)heads * dim * 2};
  cuuint32_t box[3] = {64, 1, 64};
  cuuint32_t es[3] = {1, 1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, 64] fp32 matrices stacked; box = 32 columns x 64 rows, 128-byte swizzle.
bool map_f32_64(CUtensorMap* m, const void* base, int64_t rows) {
  EncodeTiled f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {64, (cuuint64_t)rows};
  cuuint64_t strides[1] = {64 * 4};
  cuuint32_t box[2] = {32, 64};
  cuuint32_t es[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t a256(int64_t x) { return (x + 255) & ~int64_t(255); }

struct FwdWs {
  int64_t* chunk_off;
  int* err;
  float *Tbuf, *gates;  // used when no saved buffer is given
};

int64_t fwd_ws(int Hv, int N, int64_t n_chunks, bool varlen, char* base, FwdWs* w) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* at = base ? base + off : nullptr;
    off += a256(bytes);
    return at;
  };
  FwdWs x{};
  x.chunk_off = (int64_t*)take(varlen ? (int64_t)(N + 1) * 8 : 0);
  x.err = (int*)take(16);
  x.Tbuf = (float*)take(n_chunks * Hv * 4096 * 4);
  x.gates = (float*)take(n_chunks * Hv * 128 * 4);
  if (w) *w = x;
  return off;
}

}  // namespace

bool chunked_supported(int Dk, int Dv) { return Dk == DK && Dv == DV && encode_fn() != nullptr; }

// saved = [ckpt: chunks x Hv x Dv x Dk][T: chunks x Hv x 64 x 64][gates: chunks x Hv x 128], fp32
int64_t chunked_saved_bytes(int Hv, int Dk, int Dv, int64_t n_chunks, int64_t) {
  return a256(n_chunks * Hv * (int64_t)Dv * Dk * 4) + a256(n_chunks * Hv * 4096 * 4) + a256(n_chunks * Hv * 128 * 4);
}

int64_t chunked_ws_bytes(int Hv, int Hk, int Dk, int Dv, int N, int64_t n_chunks, int64_t tokens, bool varlen, int op,
                         bool with_saved) {
  (void)Hk;
  (void)Dk;
  (void)Dv;
  (void)tokens;
  (void)op;
  (void)with_saved;
  return fwd_ws(Hv, N, n_chunks, varlen, nullptr, nullptr);
}

cudaError_t chunked_fwd(const ChunkFwdArgs& a, void* ws, cudaStream_t st) {
  if (!a.in_bf16) return cudaErrorInvalidValue;
  FwdWs w;
  fwd_ws(a.Hv, a.N, a.n_chunks, a.cu != nullptr, (char*)ws, &w);
  float* ckpt = nullptr;
  float* Tbuf = w.Tbuf;
  float* gates = w.gates;
  if (a.saved) {
    char* sv = (char*)a.saved;
    ckpt = (float*)sv;
    Tbuf = (float*)(sv + a256(a.n_chunks * a.Hv * (int64_t)a.Dv * a.Dk * 4));
    gates = (float*)((char*)Tbuf + a256(a.n_chunks * a.Hv * 4096 * 4));
  }
  cudaError_t e;
  if ((e = cudaMemsetAsync(w.err, 0, 16, st)) != cudaSuccess) return e;
  if (a.cu) {
    if ((e = launch_chunk_offsets(a.cu, a.N, w.chunk_off, st)) != cudaSuccess) return e;
  }
  const int64_t rows = (int64_t)a.B * a.T;
  CUtensorMap kmap, qmap, tmap;
  if (!map_act(&kmap, a.k, rows, a.Hk, a.Dk) || !map_act(&qmap, a.q, rows, a.Hk, a.Dk) ||
      !map_f32_64(&tmap, Tbuf, a.n_chunks * a.Hv * 64))
    return cudaErrorInvalidValue;
  Geo geo{a.T, a.Hk, a.Hv, a.N, (a.T + C - 1) / C, a.cu, a.cu ? w.chunk_off : nullptr};

  PrepArgs pa{geo, a.g, a.beta, Tbuf, gates, w.err};
  const int prep_smem = 1024 + 16384 + 64 * 68 * 4;
  if ((e = cudaFuncSetAttribute(gdn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem)) !=
      cudaSuccess)
    return e;
  if (a.n_chunks > 0) {
    gdn_chunk_prep<<<dim3((unsigned)a.n_chunks, a.Hv), 128, prep_smem, st>>>(kmap, pa);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }

  StateArgs sa{geo, a.v, gates, a.h0, a.y, a.hT, ckpt, a.out_bf16, w.err};
  auto kern = a.out_bf16 ? gdn_chunk_fwd_state<true> : gdn_chunk_fwd_state<false>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, STATE_SMEM)) != cudaSuccess)
    return e;
  kern<<<dim3(DV / DVT, a.Hv, a.N), 128, STATE_SMEM, st>>>(kmap, qmap, tmap, sa);
  note_launch();
  return cudaGetLastError();
}

bool chunked_bwd_ready() { return false; }

cudaError_t chunked_bwd(const ChunkBwdArgs&, void*, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace qbgdn
