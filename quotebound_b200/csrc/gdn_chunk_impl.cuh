// Shared pieces of the tensor-core chunked path (Dk = Dv = 128, bf16 activations, chunk C = 64):
// the chunk geometry, the operand-image and TMEM helpers, each kernel's argument block and shared
// memory map, and the launchers the host side calls.  The kernels themselves live one per file:
//   gdn_chunk_prep.cu   gdn_chunk_prep       per (chunk, key head): K K^T, Q K^T, T, P and the images
//   gdn_chunk_fwd.cu    gdn_chunk_fwd_state  the forward walk over a sequence's chunks
//   gdn_chunk_bwd.cu    gdn_chunk_bwd_state  the reverse walk (dS across chunks)
//   gdn_chunk_grad.cu   gdn_chunk_bwd_grad   the per-chunk gradients
//   gdn_chunk_host.cu   layouts, tensor maps and the two orchestrations chunked_fwd / chunked_bwd
//
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
//                        on the chain (K dS^T | T^T dD | K^T H), with P^T dO (a chunk ahead) and
//                        Q^T (gamma dO) beside it.  Writes dv, dS per chunk, dh0.
//   gdn_chunk_bwd_grad   (chunks, Hk): everything else per chunk, the value heads of a key head in turn
//                        so dq and dk are summed over the group in TMEM in a fixed order; K K^T is
//                        recomputed there from the [K; Q] image (one MMA per CTA).
// Operand precision: input x input products in bf16 (exact); input x computed with the computed tile
// split into bf16 hi + lo (about 16 mantissa bits); computed x computed in tf32 (round to nearest).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>

#include "gdn_chunk.cuh"
#include "gdn_common.cuh"
#include "gdn_simt.cuh"
#include "launch_count.cuh"
#include "status.cuh"
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

// Every thread waits for the phase (a wait that gives up drains it, tc::mbar_wait_or_drain); the
// CTA-wide outcome.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity, int* err, int code, const int* hook) {
  return __syncthreads_and(tc::mbar_wait_or_drain(bar, parity, err, code, hook)) != 0;
}


// ---- the forward walk's helpers ------------------------------------------------------------------
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
constexpr int FW_V = 172032;       // 2 x 4 KB bf16 value rows [64][32] (TMA)
constexpr int FW_Y = 180224;       // 8 KB output rows [64][32] staging (TMA store of full chunks)
constexpr int FW_CK = 188416;      // 16 KB fp32 chunk-start state staging [32 dv][128 dk] (bulk store)
constexpr int FW_SMEM = 204800 + 1024;

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

// ---- the reverse walk's helpers ------------------------------------------------------------------
constexpr int BW_KQ = 0;           // 2 x 32 KB bf16 [K; Q] image
constexpr int BW_T = 65536;        // 2 x 16 KB bf16 [T_hi; T_lo] image
constexpr int BW_P = 98304;        // 2 x 16 KB bf16 [P_hi; P_lo] image
constexpr int BW_S = 131072;       // 16 KB bf16 dS [hi | lo], MN-major [128 dk][64]
constexpr int BW_GD = 147456;      // 8 KB bf16 gamma dO [hi | lo]
constexpr int BW_DD = 155648;      // 8 KB bf16 dD [hi | lo]
constexpr int BW_H = 163840;       // 8 KB bf16 H = -beta gamma F [hi | lo]
constexpr int BW_V = 172032;       // 2 x 4 KB bf16 dO rows [64][32], 64-byte swizzle (TMA)
constexpr int BW_FS = 180224;      // 2 x 16 KB [dO; F] operand image staging (bulk store)
constexpr int BW_DV = 212992;      // 8 KB dv rows [64][32] staging (TMA store of full chunks)
constexpr int BW_SMEM = 221184 + 1024;

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

// ---- the gradient kernel's helpers ---------------------------------------------------------------
// Shared memory of the gradient kernel.
constexpr int GR_KQ = 0;           // 32 KB bf16 [K; Q] image
constexpr int GR_FREE = 32768;     // 16 KB unused
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

}  // namespace

// ---- argument blocks --------------------------------------------------------------------------------
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
  // recompute mode (non-null): every chunk on its own, its start state read from these chunk-start states
  // [chunks, Hv, Dv, Dk]; D is written, y, the final state and the checkpoint are not
  const float* ckpt_in;
  int64_t geo_chunks;  // the number of chunks (the grid's z extent in recompute mode)
};

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
  const uint8_t* KQimg;     // the forward's [K; Q] operand image
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

// ---- launchers (one per kernel file) -----------------------------------------------------------------
cudaError_t launch_chunk_prep(const CUtensorMap& kmap, const CUtensorMap& qmap, const PrepArgs& a, int64_t n_chunks,
                              int Hk, cudaStream_t st);
cudaError_t launch_chunk_fwd_state(const CUtensorMap& vmap, const CUtensorMap& ymap, const StateArgs& a, int Hv, int N,
                                   bool out_bf16, cudaStream_t st);
cudaError_t launch_chunk_bwd_state(const CUtensorMap& dmap, const CUtensorMap& dvmap, const BwdStateArgs& a, int Hv,
                                   int N, bool out_bf16, cudaStream_t st);
cudaError_t launch_chunk_bwd_grad(const CUtensorMap& smap_mn, const CUtensorMap& dmap_mn, const CUtensorMap& vmap,
                                  const CUtensorMap& dqmap, const CUtensorMap& dkmap, const GradArgs& a,
                                  int64_t n_chunks, int Hk, bool out_bf16, cudaStream_t st);

}  // namespace qbgdn
