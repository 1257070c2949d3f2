// The chunk prep of the tensor-core path: per (chunk, key head) K K^T and Q K^T on the tensor cores,
// then per value head of the group the gates, L, P and T = (I + L)^-1, written as operand images.
#include "gdn_chunk_impl.cuh"

namespace qbgdn {

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
  __shared__ int s_hook[2];
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
    tc::load_hook(s_hook, a.err);
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

  bool ok = wait_all(&bar_tma, 0, a.err, 1, s_hook);
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
  ok = __syncthreads_and(ok && tc::mbar_wait_or_drain(&bar_mma, 0, a.err, 2, s_hook)) != 0;
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
      // Gamma_ij = e^(b_i - b_j) for this 32-column half (only j <= i is used): both lanes of the pair
      // need the same row's, so each forms 16 (the exponentials bound this phase) and they swap them
      float gh[16], go[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) gh[k] = __expf(bi - sb[32 * h + (kkside ? 0 : 16) + k]);
#pragma unroll
      for (int k = 0; k < 16; ++k) go[k] = __shfl_xor_sync(0xffffffffu, gh[k], 16);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int j = 32 * h + jj;
        const float gam = ((jj < 16) == kkside) ? gh[jj & 15] : go[jj & 15];
        // (P's rows past the sequence's end are zero: the reverse walk multiplies P^T with the raw rows
        // of the output gradient there, which belong to the next sequence)
        v[jj] = (kkside ? j < i : (j <= i && i < L)) ? gam * v[jj] : 0.f;
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

cudaError_t launch_chunk_prep(const CUtensorMap& kmap, const CUtensorMap& qmap, const PrepArgs& a, int64_t n_chunks,
                              int Hk, cudaStream_t st) {
  const int smem = 1024 + 32768;
  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  gdn_chunk_prep<<<dim3((unsigned)n_chunks, Hk), 128, smem, st>>>(kmap, qmap, a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
