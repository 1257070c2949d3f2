// Test support: one tcgen05 MMA tile D = A * B^T through the same helpers the chunked kernels use
// (quotebound_b200/csrc/tc_sm100.cuh), for every operand majorness and kind the kernels need.
// Built by tests/test_gpu_tc.py into tests/_build/libtcprobe.so.
#include <cuda_bf16.h>

#include "tc_sm100.cuh"

using namespace qbgdn;

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

// Bytes of an R x K operand tile: whole 128-byte slabs along the contiguous dimension.
__host__ __device__ inline int tile_bytes(int R, int K, int eb, int mn_major) {
  const int slabs = mn_major ? (R * eb + 127) / 128 : (K * eb + 127) / 128;
  return slabs * (mn_major ? K : R) * 128;
}

// A logical [M][K], B logical [N][K], D [M][N]; fp32 in global.
__global__ void __launch_bounds__(128) tc_probe_kernel(int M, int N, int K, int kind, int a_mn, int b_mn,
                                                       const float* A, const float* B, float* D, int* err,
                                                       int lane_off) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int eb = kind == tc::kBF16 ? 2 : 4;
  uint8_t* a_tile = smem;
  uint8_t* b_tile = smem + tile_bytes(M, K, eb, a_mn);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int ncols = 32;
  while (ncols < N) ncols <<= 1;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, ncols);
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  for (int i = tid; i < M * K; i += blockDim.x) {
    const int m = i / K, k = i % K;
    const uint32_t o = a_mn ? tc::off_mnmajor(k, m, K, eb) : tc::off_kmajor(m, k, M, eb);
    if (eb == 2)
      *reinterpret_cast<__nv_bfloat16*>(a_tile + o) = __float2bfloat16_rn(A[i]);
    else
      *reinterpret_cast<float*>(a_tile + o) = to_tf32(A[i]);
  }
  for (int i = tid; i < N * K; i += blockDim.x) {
    const int n = i / K, k = i % K;
    const uint32_t o = b_mn ? tc::off_mnmajor(k, n, K, eb) : tc::off_kmajor(n, k, N, eb);
    if (eb == 2)
      *reinterpret_cast<__nv_bfloat16*>(b_tile + o) = __float2bfloat16_rn(B[i]);
    else
      *reinterpret_cast<float*>(b_tile + o) = to_tf32(B[i]);
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  // M = 64 only: lane_off = 16 puts the accumulator in the upper half of each 32-lane subpartition
  const uint32_t dst = tmem + ((uint32_t)lane_off << 16);
  if (tid == 0) {
    if (kind == tc::kBF16)
      tc::mma_tile<tc::kBF16>(dst, tc::smem_u32(a_tile), a_mn, a_mn ? K : M, tc::smem_u32(b_tile), b_mn,
                              b_mn ? K : N, M, N, K, false);
    else
      tc::mma_tile<tc::kTF32>(dst, tc::smem_u32(a_tile), a_mn, a_mn ? K : M, tc::smem_u32(b_tile), b_mn,
                              b_mn ? K : N, M, N, K, false);
    tc::mma_commit(&bar);
  }
  const bool ok = tc::mbar_wait(&bar, 0, err, 1);
  tc::fence_after_sync();
  if (ok) {
    // M = 128: row m in lane m.  M = 64: rows 16w..16w+15 in lanes 32w..32w+15.
    const int row = M == 128 ? 32 * warp + lane : 16 * warp + (lane - lane_off);
    const bool mine = M == 128 || (lane >= lane_off && lane < lane_off + 16);
    for (int c = 0; c < N; c += 16) {
      float v[16];
      tc::tmem_ld16(tc::taddr(tmem, 32 * warp, c), v);
      if (mine)
        for (int j = 0; j < 16 && c + j < N; ++j) D[row * N + c + j] = v[j];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, ncols);
}

extern "C" int tc_probe_gemm(int M, int N, int K, int kind, int a_mn, int b_mn, const float* A, const float* B,
                             float* D, int* err, int lane_off) {
  if ((M != 64 && M != 128) || N < 16 || N > 256 || N % 16 || K < 16 || K > 128 || K % 16) return -1;
  if (lane_off != 0 && (M != 64 || lane_off != 16)) return -1;
  const int eb = kind == tc::kBF16 ? 2 : 4;
  const int smem = 1024 + tile_bytes(M, K, eb, a_mn) + tile_bytes(N, K, eb, b_mn);
  cudaFuncSetAttribute(tc_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  tc_probe_kernel<<<1, 128, smem>>>(M, N, K, kind, a_mn, b_mn, A, B, D, err, lane_off);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// TMA layout probe: one 2-D box of 32 fp32 columns x 64 rows from an [rows][64] fp32 matrix, loaded
// with the given swizzle (3 = 128B, 4 = 128B with 32-byte atoms), copied back raw so the test can
// compare every element's position with the layouts tc_sm100.cuh assumes.
__global__ void __launch_bounds__(128) tc_probe_tma_kernel(const __grid_constant__ CUtensorMap map, int row0,
                                                           int col0, float* out, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t bar;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    tc::mbar_arrive_expect_tx(&bar, 8192);
    tc::tma_load_2d(smem, &map, &bar, col0, row0);
  }
  const bool ok = tc::mbar_wait(&bar, 0, err, 1);
  __syncthreads();
  if (ok)
    for (int i = threadIdx.x; i < 2048; i += blockDim.x) out[i] = reinterpret_cast<float*>(smem)[i];
}

extern "C" int tc_probe_tma(const float* src, int rows, int row0, int col0, int swizzle, float* out, int* err) {
  using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return -3;
  if (rows < 64 || row0 < 0 || row0 + 64 > rows || (col0 != 0 && col0 != 32)) return -1;
  CUtensorMap map;
  cuuint64_t dims[2] = {64, (cuuint64_t)rows};
  cuuint64_t strides[1] = {64 * 4};
  cuuint32_t box[2] = {32, 64};
  cuuint32_t es[2] = {1, 1};
  CUtensorMapSwizzle sw = swizzle == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  if (reinterpret_cast<EncodeTiled>(p)(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(src), dims,
                                       strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                       CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return -4;
  cudaFuncSetAttribute(tc_probe_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 8192 + 1024);
  tc_probe_tma_kernel<<<1, 128, 8192 + 1024>>>(map, row0, col0, out, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
