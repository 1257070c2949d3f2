// sm_100a building blocks: mbarriers with bounded waits, TMA tile loads, and tcgen05 tensor-core
// MMAs with TMEM accumulators.  Operand tiles live in shared memory in the 128-byte-swizzled
// canonical layouts the MMA descriptors describe:
//
//  * K-major tile (R rows of M or N, K contiguous): the K extent is cut into 128-byte slabs
//    (64 bf16 or 32 fp32 elements); slab s holds R rows of 128 bytes, row r at r*128, and the
//    16-byte chunk j of row r sits at chunk (j ^ (r & 7)).  Slabs follow each other every R*128
//    bytes.  Descriptor: SBO = 1024 (8 rows), LBO unused; one MMA K-step (32 bytes) advances the
//    start address by 32 bytes inside a slab.
//  * MN-major tile (K rows, M or N contiguous): the MN extent is cut into 128-byte slabs; slab s
//    holds Krows rows of 128 bytes (row = one k).  bf16: 128-byte swizzle, 16-byte chunk j of row k
//    at chunk (j ^ (k & 7)), SBO = 1024 (8 k-rows).  tf32: the 32-byte-atom variant of the 128-byte
//    swizzle (layout type 1), 32-byte granule j of row k at granule (j ^ (k & 3)), SBO = 512
//    (4 k-rows).  LBO = the slab stride (Krows*128); one MMA K-step advances the start by 16 (bf16)
//    or 8 (tf32) rows.
//
// Every slab starts on a 1024-byte boundary, so the hardware's address-based swizzle matches.
// Every CTA loads its own tiles from its own GPU's memory; no load is shared across a cluster.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qbgdn {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarriers ---------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of the same phase (try_wait may suspend the thread for a while before it
// answers no).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity to complete.  Gives up after about one second of
// wall time (checked every 256 polls; each poll may itself suspend briefly) or 2^24 polls, records
// `code` in the status block `err` (the first failure of a call wins) and returns false; the caller
// then skips its remaining work, waits (again bounded, with no code) for the copies and products it
// still has in flight, frees its TMEM and returns.  Never spins forever, never traps.
//
// err points at the status block that opens every workspace (status.cuh), word 0 the code.  hook is
// the kernel's shared-memory copy of the block's test hook (words 4 and 5, read once per CTA by
// load_hook): when hook[0] equals `code`, this wait gives up after hook[1] polls, so that a test can
// make one named wait run out on a normal input.  The first poll does not suspend, so a wait whose
// data is still in flight always reaches the hook.
constexpr uint32_t kMaxPolls = 1u << 24;
constexpr uint64_t kMaxWaitNs = 1000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          const int* hook = nullptr) {
  if (mbar_test_wait(bar, parity)) return true;
  uint32_t limit = kMaxPolls;
  if (hook && code > 0 && hook[0] == code) limit = (uint32_t)hook[1];
  uint64_t t0 = 0;  // the wall clock starts at the 256th poll (a short wait never reads it)
  for (uint32_t i = 1; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > kMaxWaitNs) break;
    }
  }
  if (err) atomicCAS(err, 0, code);
  return false;
}
// The test hook of the status block into shared memory (one thread, before the CTA's first barrier).
__device__ __forceinline__ void load_hook(int* hook, const int* err) {
  hook[0] = err ? err[4] : 0;
  hook[1] = err ? err[5] : 0;
}
// The failure path's wait for work still in flight: the full limits, nothing recorded.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  return mbar_wait(bar, parity, nullptr, 0);
}
// mbar_wait for a phase whose copies or products were issued; when it gives up, the same phase is
// waited for again (mbar_drain), so that they have landed before anything reads or reuses their
// buffers.  Returns whether the first wait succeeded.
__device__ __forceinline__ bool mbar_wait_or_drain(uint64_t* bar, uint32_t parity, int* err, int code,
                                                   const int* hook = nullptr) {
  if (mbar_wait(bar, parity, err, code, hook)) return true;
  mbar_drain(bar, parity);
  return false;
}

// ---- TMA ----------------------------------------------------------------------------------------
// 3-D tiled load into this CTA's shared memory, completing `bytes` on the mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// 3-D tiled store from this CTA's shared memory (bulk async-group; commit and wait like bulk_store).
// Coordinates must not be negative.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- fences -------------------------------------------------------------------------------------
// Generic-proxy writes to shared memory -> visible to the async proxy (MMA operand reads).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- TMEM -----------------------------------------------------------------------------------------
// Executed by one whole warp; the TMEM address lands in *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns into v (this thread's lane).  Then wait::ld.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 consecutive columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Loads without the wait, so that several can be in flight: issue them, then tmem_wait_ld(), then
// reg_fence() on each destination before its first use (the fence ties the registers' uses to a
// point after the wait; the compiler may not hoist them above it).
__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// Store 32 consecutive columns of this thread's lane (warp-wide); tmem_wait_st before the MMAs that
// read them are issued.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column): lane in the high 16 bits.
__device__ __forceinline__ uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ---- descriptors ---------------------------------------------------------------------------------
enum Kind { kBF16 = 1, kTF32 = 2 };

// Instruction descriptor of kind::f16 (bf16 inputs) or kind::tf32, fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc(int kind, int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (uint32_t(kind) << 7) | (uint32_t(kind) << 10)  // A, B formats: bf16 = 1, tf32 = 2
         | (uint32_t(a_mn_major) << 15) | (uint32_t(b_mn_major) << 16) | (uint32_t(N >> 3) << 17) |
         (uint32_t(M >> 4) << 24);
}

// Shared-memory matrix descriptor, sm_100 version field.  layout: 2 = 128-byte swizzle, 1 = 128-byte
// swizzle with 32-byte atoms (the tf32 MN-major layout).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                          uint32_t layout = 2) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(layout) << 61);
}

// Descriptor of MMA K-step `ks` over a K-major tile with R rows (32 bytes per step).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int R, int ks) {
  return sdesc(tile + (ks >> 2) * (R * 128) + (ks & 3) * 32, 16, 1024);
}
// Descriptor of MMA K-step `ks` over an MN-major tile with Krows k-rows; rows_per_step is 16 for
// bf16 and 8 for tf32.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int Krows, int ks, int rows_per_step) {
  return rows_per_step == 16 ? sdesc(tile + ks * 16 * 128, Krows * 128, 1024, 2)
                             : sdesc(tile + ks * 8 * 128, Krows * 128, 512, 1);
}

// Byte offset of element (r, k) in a K-major tile of R rows, element size eb.
__host__ __device__ __forceinline__ uint32_t off_kmajor(int r, int k, int R, int eb) {
  const int E = 128 / eb, slab = k / E, kin = k - slab * E;
  const int chunk = (kin * eb) >> 4, within = (kin * eb) & 15;
  return slab * (R * 128) + r * 128 + ((chunk ^ (r & 7)) << 4) + within;
}
// Byte offset of element (k, r) in an MN-major tile of Krows k-rows (bf16: 16-byte chunks swizzled
// by k & 7; fp32: 32-byte granules swizzled by k & 3).
__host__ __device__ __forceinline__ uint32_t off_mnmajor(int k, int r, int Krows, int eb) {
  const int E = 128 / eb, slab = r / E, rin = r - slab * E;
  const int byte = rin * eb;
  if (eb == 4) return slab * (Krows * 128) + k * 128 + ((((byte >> 5) ^ (k & 3))) << 5) + (byte & 31);
  return slab * (Krows * 128) + k * 128 + ((((byte >> 4) ^ (k & 7))) << 4) + (byte & 15);
}

// ---- MMA issue (one thread) ------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[M x N] (+)= A[M x K] * B[N x K]^T over K / kstep MMA instructions.  Operand tiles as above;
// a_mn / b_mn select MN-major tiles (then a_rows / b_rows are the tile's K row count).
template <int KIND>
__device__ __forceinline__ void mma_tile(uint32_t d_tmem, uint32_t a_tile, bool a_mn, int a_rows, uint32_t b_tile,
                                         bool b_mn, int b_rows, int M, int N, int K, bool accumulate) {
  const uint32_t id = idesc(KIND, M, N, a_mn, b_mn);
  const int kstep = KIND == kBF16 ? 16 : 8;
  for (int ks = 0; ks < K / kstep; ++ks) {
    const uint64_t a = a_mn ? desc_mnmajor(a_tile, a_rows, ks, kstep) : desc_kmajor(a_tile, a_rows, ks);
    const uint64_t b = b_mn ? desc_mnmajor(b_tile, b_rows, ks, kstep) : desc_kmajor(b_tile, b_rows, ks);
    if (KIND == kBF16)
      mma_bf16(d_tmem, a, b, id, (accumulate || ks > 0) ? 1u : 0u);
    else
      mma_tf32(d_tmem, a, b, id, (accumulate || ks > 0) ? 1u : 0u);
  }
}

// ---- vectorised row stores into operand tiles (one thread writes one whole row) ----------------------
// fp32, MN-major tf32 layout (32-byte granules swizzled by k & 3): row k of one 128-byte slab.
__device__ __forceinline__ void st_row_mn_f32(uint8_t* slab, int k, const float (&v)[32]) {
  uint8_t* row = slab + k * 128;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float4* dst = reinterpret_cast<float4*>(row + ((g ^ (k & 3)) << 5));
    dst[0] = make_float4(v[8 * g], v[8 * g + 1], v[8 * g + 2], v[8 * g + 3]);
    dst[1] = make_float4(v[8 * g + 4], v[8 * g + 5], v[8 * g + 6], v[8 * g + 7]);
  }
}
// fp32, K-major 128-byte swizzle (16-byte chunks swizzled by r & 7): row r of one slab (32 floats).
__device__ __forceinline__ void st_row_k_f32(uint8_t* slab, int r, const float (&v)[32]) {
  uint8_t* row = slab + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(row + ((c ^ (r & 7)) << 4)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// Split 32 floats into bf16 hi + lo (hi + lo carries about 16 mantissa bits) and store both rows in
// a bf16 128-byte-swizzled tile (16-byte chunks swizzled by r & 7; 32 elements = chunks 0..3).
// Used for K-major rows and MN-major rows alike: the byte pattern is the same.  c0 = 4 writes the
// elements 32..63 of a 64-wide row.
__device__ __forceinline__ void st_row_bf16x2_32(uint8_t* hi_slab, uint8_t* lo_slab, int r, const float (&v)[32],
                                                 int c0 = 0, int lo_c0 = -1) {
  const int lc0 = lo_c0 < 0 ? c0 : lo_c0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = v[8 * c + 2 * e], b = v[8 * c + 2 * e + 1];
      const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
      h[e] = *reinterpret_cast<const uint32_t*>(&hh);
      l[e] = pack_bf16(a - __low2float(hh), b - __high2float(hh));
    }
    *reinterpret_cast<uint4*>(hi_slab + r * 128 + (((c + c0) ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_slab + r * 128 + (((c + lc0) ^ (r & 7)) << 4)) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// One 128-byte row [hi of 32 | lo of 32]: the N = 64 operand row whose two halves the MMA multiplies
// in one instruction (the halves' products are summed by the reader of the accumulator).
__device__ __forceinline__ void st_row_hilo(uint8_t* tile, int r, const float (&v)[32]) {
  st_row_bf16x2_32(tile, tile, r, v, 0, 4);
}

// Half of such a row: 16 floats (columns 16 half .. 16 half + 15 of each 32-wide half) as hi chunks
// 2 half, 2 half + 1 and lo chunks 4 + 2 half, 5 + 2 half.
__device__ __forceinline__ void st_row_hilo16(uint8_t* tile, int r, const float (&v)[16], int half) {
  uint8_t* row = tile + r * 128;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = v[8 * c + 2 * e], b = v[8 * c + 2 * e + 1];
      const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
      h[e] = *reinterpret_cast<const uint32_t*>(&hh);
      l[e] = pack_bf16(a - __low2float(hh), b - __high2float(hh));
    }
    *reinterpret_cast<uint4*>(row + (((2 * half + c) ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(row + (((4 + 2 * half + c) ^ (r & 7)) << 4)) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// ---- bulk (non-tensor) copies: contiguous bytes, 16-byte aligned addresses and sizes ---------------
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of every committed bulk store have been read
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every committed bulk store has completed
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace tc
}  // namespace qbgdn
