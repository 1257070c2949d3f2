// The reverse walk of the tensor-core path: a sequence's chunks backwards, 32 rows of dS per CTA.
#include "gdn_chunk_impl.cuh"

namespace qbgdn {

// The backward state walk: chunks in reverse, 32 rows of dS per CTA.  320 threads: warps 0-7 hold dS
// (thread t < 256 holds dS[dv0 + 16 (w >> 2) + j][t & 127]) and run the epilogues; lane 0 of warp 8
// issues every MMA, lane 0 of warp 9 every copy (issuing either costs the thread hundreds of cycles a
// round, which would otherwise delay an epilogue warp).  Per chunk the chain is
// [K; Q] dS^T -> dD -> F = T^T dD -> H -> K^T H -> dS; the products that need no dS -- G = P^T dO (from
// the value-gradient rows as they land, a chunk ahead) and Q^T (gamma dO) -- run where the tensor pipe
// would idle, and the epilogue work that feeds no product of the chain (the dS copy for the gradient
// kernel, the dO rows' staging) fills the waits for the products.  Besides dv, the per-chunk dS and
// dh0 it leaves the gradient kernel F = T^T dD.
template <typename Tout>
__global__ void __launch_bounds__(320, 1) gdn_chunk_bwd_state(const __grid_constant__ CUtensorMap dmap,
                                                              const __grid_constant__ CUtensorMap dvmap,
                                                              BwdStateArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float sg[2][128];
  __shared__ uint64_t bar_main[2], bar_g[2], bar_mma, bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_hook[2];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // (lanes 1-31 of warps 8 and 9 only join the barriers)
  const bool epi = warp < 8, issuer = tid == 256, copier = tid == 288;
  const int quad = warp & 3, half = (warp >> 2) & 1, dk = tid & 127;
  const int dv0 = blockIdx.x * DVT, hv = blockIdx.y, n = blockIdx.z;
  const int Hv = a.geo.Hv, hk = hv / (Hv / a.geo.Hk);
  int64_t c_first, nchunks, seq0, seq1;
  seq_chunks(a.geo, n, c_first, nchunks, seq0, seq1);

  // TMEM: [K; Q] dS^T 0 (64), P^T dO 64 (32), F 128 (64), U 192 (64)
  const uint32_t cX = 0, cG = 64, cF = 128, cU = 192;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 256);
  if (tid == 0) {
#pragma unroll
    for (int b = 0; b < 2; ++b) tc::mbar_init(&bar_main[b], 1), tc::mbar_init(&bar_g[b], 1);
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

  float ds[16];  // ds[j] = dS[dv0 + 16 half + j][dk] (the epilogue warps)
  if (epi) {
    const size_t base = (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
    for (int j = 0; j < 16; ++j) ds[j] = a.dhT ? a.dhT[base + (size_t)j * DK] : 0.f;
  }

  // The copies of the chunk handled `it` iterations in (jc = nchunks - 1 - it), all into buffer it & 1,
  // in two groups: its [K; Q] and T images and gates (issued a chunk ahead, at its start), and G's
  // operands, its P image and value-gradient rows (64-byte swizzle: the MN-major B operand of P^T dO,
  // read in place), issued two chunks ahead (their last readers finish early in the chunk).  The copies
  // land one to two microseconds after they are issued.
  auto issue_main = [&](int64_t it) {
    const int b = (int)(it & 1);
    const int64_t jc = nchunks - 1 - it, cg = c_first + jc;
    tc::mbar_arrive_expect_tx(&bar_main[b], 32768 + 512 + 16384);
    tc::bulk_load(smem + BW_KQ + b * 32768, a.KQimg + (size_t)(cg * a.geo.Hk + hk) * 32768, 32768, &bar_main[b]);
    tc::bulk_load(sg[b], a.gates + (cg * Hv + hv) * 128, 512, &bar_main[b]);
    tc::bulk_load(smem + BW_T + b * 16384, a.Timg + (size_t)(cg * Hv + hv) * 16384, 16384, &bar_main[b]);
  };
  auto issue_g = [&](int64_t it) {
    const int b = (int)(it & 1);
    const int64_t jc = nchunks - 1 - it, cg = c_first + jc;
    tc::mbar_arrive_expect_tx(&bar_g[b], 16384 + 4096);
    tc::bulk_load(smem + BW_P + b * 16384, a.Pimg + (size_t)(cg * Hv + hv) * 16384, 16384, &bar_g[b]);
    tc::tma_load_3d(smem + BW_V + b * 4096, &dmap, &bar_g[b], dv0, hv, (int)(seq0 + jc * C));
  };
  const uint32_t idX = tc::idesc(tc::kBF16, 128, 64, false, true);  // [K; Q] x [hi | lo]
  const uint32_t idG = tc::idesc(tc::kBF16, 64, 32, true, true);    // P^T x dO
  const uint32_t idF = tc::idesc(tc::kBF16, 64, 64, true, true);    // T^T x [hi | lo]
  const uint32_t idU = tc::idesc(tc::kBF16, 128, 64, true, true);   // Q^T, K^T x [hi | lo]
  // G = P^T dO of iteration it into cG: P_hi^T and P_lo^T accumulated (M = 64), the value-gradient
  // rows as the MN-major N = 32 operand (64-byte rows in the 64-byte swizzle, 512 bytes per 8 rows).
  // P's rows past the sequence's end are zero, so the next sequence's rows there add nothing.
  auto mma_g = [&](int64_t it, int part) {  // part 0: P_hi^T dO (fresh), 1: + P_lo^T dO
    const int b = (int)(it & 1);
    const uint32_t pimg = tc::smem_u32(smem + BW_P + b * 16384), vt = tc::smem_u32(smem + BW_V + b * 4096);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      tc::mma_bf16(tmem + cG, desc_img_t(pimg, part, ks), tc::sdesc(vt + ks * 1024, 4096, 512, 4), idG,
                   (part | ks) ? 1u : 0u);
  };

  bool ok = true;
  int64_t issued = 0, g_issued = 0;  // the copier's counts of iterations whose copies were issued
  if (copier && nchunks > 0) {
    tc::prefetch_tmap(&dmap);
    tc::prefetch_tmap(&dvmap);
    issue_main(0), issued = 1;
    issue_g(0), g_issued = 1;
    if (nchunks > 1) issue_g(1), g_issued = 2;
  }
  if (issuer && nchunks > 0) {
    ok = tc::mbar_wait_or_drain(&bar_g[0], 0, a.err, 26, s_hook);
    if (ok) mma_g(0, 0), mma_g(0, 1);  // completes before the first chunk's round-3 commit
  }
  const int i_row = 16 * quad + (lane & 15);
  const bool kside = lane < 16;
  uint32_t ph = 0;  // the next phase of bar_mma (three per chunk)

  for (int64_t it = 0; it < nchunks; ++it) {
    const int64_t jc = nchunks - 1 - it;
    const int b = (int)(it & 1);
    const int64_t cg = c_first + jc;
    const int64_t tok0 = seq0 + jc * C;
    const int L = (int)min((int64_t)C, seq1 - tok0);

    // 1. dS of this chunk's end as the [hi | lo] operand row dk
    if (epi) tc::st_row_hilo16(smem + BW_S, dk, ds, half);
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    const uint32_t kq = tc::smem_u32(smem + BW_KQ + b * 32768);
    // 3. [K; Q] dS^T (the K rows are X = K dS^T; G is in TMEM since the last chunk); the next chunk's
    //    copies, into the buffers the chunk before has finished with
    if (issuer) {
      ok = tc::mbar_wait_or_drain(&bar_main[b], (uint32_t)((it >> 1) & 1), a.err, 20, s_hook);
      tc::fence_after_sync();
      if (ok) {
        mma_run<8, kKmaj128>(tmem + cX, idX, kq, tc::smem_u32(smem + BW_S), false);
        tc::mma_commit(&bar_mma);
      }
    }
    if (copier) {
      if (it + 1 < nchunks) issue_main(it + 1), issued = it + 2;  // the buffers of the chunk before
      tc::bulk_wait_read();  // the last chunk's image and dv stores: their staging is rewritten below
    }
    float bi = 0.f, be = 0.f, gi = 0.f, bC = 0.f;
    if (epi) {
      // meanwhile the chunk's rows and gates: dO row i (zero past the end) into the gradient kernel's
      // image (exact in tf32, lower row of the pair) and as gamma dO [hi | lo] for Q^T (gamma dO).  One
      // instruction stream for the lane pair: the K-side lane takes columns 0-7 of the thread's 16, the
      // Q-side lane columns 8-15.
      ok = ok && tc::mbar_wait_or_drain(&bar_main[b], (uint32_t)((it >> 1) & 1), a.err, 20, s_hook);
      ok = ok && tc::mbar_wait_or_drain(&bar_g[b], (uint32_t)((it >> 1) & 1), a.err, 26, s_hook);
      const float* gb = sg[b];
      bi = gb[i_row], be = gb[64 + i_row], gi = __expf(bi), bC = gb[63];
      {
        const int hc = kside ? 0 : 1, c16 = 2 * half + hc;
        const uint4 w = i_row < L ? *reinterpret_cast<const uint4*>(smem + BW_V + b * 4096 + i_row * 64 +
                                                                   ((c16 ^ ((i_row >> 1) & 3)) << 4))
                                  : make_uint4(0, 0, 0, 0);
        float d[8];
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&u[e]);
          d[2 * e] = __low2float(h2);
          d[2 * e + 1] = __high2float(h2);
        }
        st8_f32_sw(smem + BW_FS + b * 16384, img_row(i_row), 4 * half + 2 * hc, d);
#pragma unroll
        for (int j = 0; j < 8; ++j) d[j] *= gi;
        st_hilo8(smem + BW_GD, i_row, d, 2 * half + hc);
      }
      // 4. dD = diag(lambda) K dS^T + P^T dO (K side), as the [hi | lo] operand.  tcgen05.ld is a
      //    warp-wide aligned instruction: every lane executes the same loads, outside the branch.
      ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 21, s_hook);
      tc::fence_after_sync();
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
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 5. F = T^T dD (T_hi^T and T_lo^T accumulated; M = 64: row j in the K-side lanes); then Q^T (gamma
    //    dO), U's first half, which runs during the F epilogue.  G's operands of the chunk after next go
    //    into this chunk's buffers (G of this chunk completed before round 3's commit, and the dO rows
    //    were staged before the last barrier).
    if (copier && it + 2 < nchunks) issue_g(it + 2), g_issued = it + 3;
    if (issuer) {
      {
        const uint32_t dd = tc::smem_u32(smem + BW_DD), timg = tc::smem_u32(smem + BW_T + b * 16384);
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_bf16(tmem + cF, desc_img_t(timg, part, ks), desc_hl(dd, ks), idF, (part | ks) ? 1u : 0u);
        tc::mma_commit(&bar_mma);
        mma_run<4, kQT>(tmem + cU, idU, kq, tc::smem_u32(smem + BW_GD), false);
      }
      // G of the next chunk (cG was read in step 4), its first half here (it runs during the F
      // epilogue, ahead of K^T H), the second after K^T H
      if (it + 1 < nchunks) {
        ok = tc::mbar_wait_or_drain(&bar_g[b ^ 1], (uint32_t)(((it + 1) >> 1) & 1), a.err, 26, s_hook);
        if (ok) mma_g(it + 1, 0);
      }
    }
    if (epi) {
      // meanwhile dS (tf32-rounded: its one reader takes it as a tf32 operand) into the gradient
      // kernel's per-chunk dS
      {
        float* dst = a.dsbuf + ((cg * Hv + hv) * DV + dv0 + 16 * half) * (size_t)DK + dk;
#pragma unroll
        for (int j = 0; j < 16; ++j) dst[(size_t)j * DK] = tf32_rna(ds[j]);
      }
      ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph ^ 1, a.err, 22, s_hook);
      tc::fence_after_sync();
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
        st8_f32_sw(smem + BW_FS + b * 16384, img_row(i_row) + 16, 4 * half + 2 * hc, fr);
      }
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = be * f8[j];
      if (L == C)  // a full chunk goes out by one TMA store after the barrier below
        store_row8<Tout>(sizeof(Tout) == 2  // bf16 rows in the 64-byte swizzle of the dv map (spread over the banks)
                             ? reinterpret_cast<Tout*>(smem + BW_DV + i_row * 64 + (((2 * half + hc) ^ ((i_row >> 1) & 3)) << 4))
                             : reinterpret_cast<Tout*>(smem + BW_DV) + i_row * DVT + 16 * half + 8 * hc,
                         o);
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
    // 6. U = Q^T (gamma dO) (issued in step 5) + K^T H (M = 128 dk rows); the stores of this chunk's
    //    image and dv rows
    if (issuer) {
      mma_run<4, kKT>(tmem + cU, idU, kq, tc::smem_u32(smem + BW_H), true);
      tc::mma_commit(&bar_mma);
      if (it + 1 < nchunks) mma_g(it + 1, 1);
    }
    if (copier) {
      tc::bulk_store(a.Aimg + ((size_t)(cg * Hv + hv) * (DV / DVT) + blockIdx.x) * 16384, smem + BW_FS + b * 16384,
                     16384);
      if (L == C) tc::tma_store_3d(&dvmap, smem + BW_DV, dv0, hv, (int)tok0);
      tc::bulk_commit();
    }
    if (epi) {
      ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 23, s_hook);
      tc::fence_after_sync();
      float u[16];
      tmem_ld_hl16(tl + cU, half, u);
      const float gC = __expf(bC);
#pragma unroll
      for (int j = 0; j < 16; ++j) ds[j] = fmaf(gC, ds[j], u[j]);
    }
    ph ^= 1;  // three phases: the chunk's last wait had the parity of its first
    tc::fence_before_sync();
  }
  ok = __syncthreads_and(ok) != 0;  // (the last round's waits were per thread)
  if (!ok) {  // a wait gave up: everything still in flight lands before the TMEM and the CTA go
    if (issuer) {
      tc::mma_commit(&bar_drain);  // every product this thread issued
      tc::mbar_drain(&bar_drain, 0);
    }
    if (copier) {  // each buffer's latest copies (the earlier ones have landed)
      for (int64_t m = issued > 2 ? issued - 2 : 0; m < issued; ++m)
        tc::mbar_drain(&bar_main[m & 1], (uint32_t)((m >> 1) & 1));
      for (int64_t m = g_issued > 2 ? g_issued - 2 : 0; m < g_issued; ++m)
        tc::mbar_drain(&bar_g[m & 1], (uint32_t)((m >> 1) & 1));
    }
  }
  if (copier) tc::bulk_wait();
  if (ok && epi && a.dh0) {
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
  kern<<<dim3(DV / DVT, Hv, N), 320, BW_SMEM, st>>>(dmap, dvmap, a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
