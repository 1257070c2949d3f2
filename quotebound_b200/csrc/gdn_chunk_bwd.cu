// The reverse walk of the tensor-core path: a sequence's chunks backwards, 32 rows of dS per CTA.
#include "gdn_chunk_impl.cuh"

namespace qbgdn {

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
  __shared__ uint64_t bar_tma[2], bar_t, bar_p, bar_mma, bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_hook[2];

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
    tc::mbar_init(&bar_drain, 1);
    tc::load_hook(s_hook, a.err);
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
  // failure path bookkeeping (the issuing thread's): loads issued for iterations [0, *_issued), and
  // the iterations whose load waits this thread ran
  int64_t main_issued = nchunks > 0 ? 1 : 0, t_issued = main_issued, p_issued = main_issued, seen = 0;
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
    const bool waits = ok;
    bool okw = ok && tc::mbar_wait_or_drain(&bar_tma[buf], (uint32_t)((it >> 1) & 1), a.err, 20, s_hook);
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
    if (waits) {  // (the T and P waits run even when the row wait gave up, so that all three have landed)
      const bool okt = tc::mbar_wait_or_drain(&bar_t, (uint32_t)(it & 1), a.err, 25, s_hook);
      const bool okp = tc::mbar_wait_or_drain(&bar_p, (uint32_t)(it & 1), a.err, 26, s_hook);
      okw = okw && okt && okp;
      seen = it + 1;
    }
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
    if (jc > 0) main_issued = it + 2;
    ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 21, s_hook);
    ph ^= 1;
    tc::fence_after_sync();
    if (ok && tid == 32 && jc > 0) {  // P's last reader has completed
      issue_p(jc - 1);
      p_issued = it + 2;
    }
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
    ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 22, s_hook);
    ph ^= 1;
    tc::fence_after_sync();
    if (ok && tid == 32 && jc > 0) {  // T's last reader has completed
      issue_t(jc - 1);
      t_issued = it + 2;
    }
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
    ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 23, s_hook);
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
  if (!ok) {  // a wait gave up: everything still in flight lands before the TMEM and the CTA go
    if (tid == 0) {  // every product this thread issued
      tc::mma_commit(&bar_drain);
      tc::mbar_drain(&bar_drain, 0);
    }
    if (tid == 32) {
      for (int64_t m = seen; m < main_issued; ++m) tc::mbar_drain(&bar_tma[m & 1], (uint32_t)((m >> 1) & 1));
      for (int64_t m = seen; m < t_issued; ++m) tc::mbar_drain(&bar_t, (uint32_t)(m & 1));
      for (int64_t m = seen; m < p_issued; ++m) tc::mbar_drain(&bar_p, (uint32_t)(m & 1));
    }
  }
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

cudaError_t launch_chunk_bwd_state(const CUtensorMap& dmap, const CUtensorMap& dvmap, const BwdStateArgs& a, int Hv,
                                   int N, bool out_bf16, cudaStream_t st) {
  auto kern = out_bf16 ? gdn_chunk_bwd_state<__nv_bfloat16> : gdn_chunk_bwd_state<float>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
  if (e != cudaSuccess) return e;
  kern<<<dim3(DV / DVT, Hv, N), 256, BW_SMEM, st>>>(dmap, dvmap, a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
