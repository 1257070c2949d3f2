// The forward walk of the tensor-core path: a sequence's chunks in order, 32 state rows per CTA.
#include "gdn_chunk_impl.cuh"

namespace qbgdn {

// 320 threads.  Warps 0-7 hold the state and run the epilogues: warp w reads TMEM lanes 32 (w & 3) .. + 31
// and handles the value columns 16 (w >> 2) .. + 15 of the CTA's 32; thread t < 256 holds
// S[dv0 + 16 (w >> 2) + j][t & 127].  Lane 0 of warp 8 issues every MMA, lane 0 of warp 9 every copy:
// issuing costs a thread hundreds of cycles a round, which would otherwise delay an epilogue warp.  Per
// chunk the chain is [K; Q] S^T -> E -> D = T E -> D~ -> K^T D~ -> S; the output product P D runs after
// the state update and its rows are read out during the next chunk, and the copies for the gradient
// kernel (the chunk-start state, D) are written while the epilogue warps wait for a product.
template <typename Tout>
__global__ void __launch_bounds__(320, 1) gdn_chunk_fwd_state(const __grid_constant__ CUtensorMap vmap,
                                                              const __grid_constant__ CUtensorMap ymap, StateArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float sg[2][128];
  __shared__ uint64_t bar_tma[2], bar_p[2], bar_mma, bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_hook[2];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // (lanes 1-31 of warps 8 and 9 only join the barriers)
  const bool epi = warp < 8, issuer = tid == 256, copier = tid == 288;
  const int quad = warp & 3, half = (warp >> 2) & 1, dk = tid & 127;
  const int dv0 = blockIdx.x * DVT, hv = blockIdx.y, n = blockIdx.z;
  const int Hv = a.geo.Hv, hk = hv / (Hv / a.geo.Hk);
  // recompute mode: this CTA's one chunk (blockIdx.z), its start state from the checkpoint; D is the product
  const bool outputs = a.ckpt_in == nullptr;
  int64_t c_first, nchunks, seq0, seq1;
  if (!outputs) {
    int nn, Lc;
    int64_t t0;
    c_first = blockIdx.z;
    chunk_info(a.geo, c_first, nn, t0, Lc);
    nchunks = 1, seq0 = t0, seq1 = t0 + Lc;
  } else {
    seq_chunks(a.geo, n, c_first, nchunks, seq0, seq1);
  }

  // TMEM: [K; Q] S^T 0, D 64, S update 128, P D 192 (64 columns each: hi and lo halves)
  const uint32_t cA = 0, cD = 64, cS = 128, cO = 192;
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 256);
  if (tid == 0) {
#pragma unroll
    for (int b = 0; b < 2; ++b) tc::mbar_init(&bar_tma[b], 1), tc::mbar_init(&bar_p[b], 1);
    tc::mbar_init(&bar_mma, 1);
    tc::mbar_init(&bar_drain, 1);
    tc::load_hook(s_hook, a.err);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tl = tc::taddr(tmem, 32 * quad, 0);  // this warp's lanes

  float s[16];  // s[j] = S[dv0 + 16 half + j][dk] (the epilogue warps)
  if (epi) {
    if (outputs) {
      const size_t base = (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
      for (int j = 0; j < 16; ++j) s[j] = a.h0 ? a.h0[base + (size_t)j * DK] : 0.f;
    } else {
      const float* ck = a.ckpt_in + (((size_t)c_first * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
      for (int j = 0; j < 16; ++j) s[j] = ck[(size_t)j * DK];
    }
  }

  // Everything a chunk reads (the [K; Q] and T images, the gates and the value rows on one barrier, the
  // P image on another), by one copy each into buffer jc & 1, so that no thread waits on a global load
  // inside the walk.  The copies land a chunk or more after they are issued, so each goes out as soon
  // as its buffer's last reader is done: P once the P D of two chunks back has completed, the rest at
  // the start of the chunk before.
  auto issue_loads = [&](int64_t jc) {
    const int buf = (int)(jc & 1);
    const int64_t cg = c_first + jc;
    tc::mbar_arrive_expect_tx(&bar_tma[buf], 32768 + 16384 + 512 + 4096);
    tc::bulk_load(smem + FW_KQ + buf * 32768, a.KQimg + (size_t)(cg * a.geo.Hk + hk) * 32768, 32768, &bar_tma[buf]);
    tc::bulk_load(smem + FW_T + buf * 16384, a.Timg + (size_t)(cg * Hv + hv) * 16384, 16384, &bar_tma[buf]);
    tc::bulk_load(sg[buf], a.gates + (cg * Hv + hv) * 128, 512, &bar_tma[buf]);
    tc::tma_load_3d(smem + FW_V + buf * 4096, &vmap, &bar_tma[buf], dv0, hv, (int)(seq0 + jc * C));
  };
  auto issue_p = [&](int64_t jc) {
    const int buf = (int)(jc & 1);
    tc::mbar_arrive_expect_tx(&bar_p[buf], 16384);
    tc::bulk_load(smem + FW_P + buf * 16384, a.Pimg + (size_t)((c_first + jc) * Hv + hv) * 16384, 16384, &bar_p[buf]);
  };

  // Lane l < 16 owns chunk row i = 16 quad + l for the K-side products (E, D) and lane l + 16 the same
  // row for the Q-side ones (Y, D~, y).
  const int i_row = 16 * quad + (lane & 15);
  const bool kside = lane < 16;
  if (nchunks > 0 && copier) {
    tc::prefetch_tmap(&vmap);
    issue_loads(0);
    if (outputs) issue_p(0);
  }
  uint32_t ph = 0;  // the next phase of bar_mma (three per chunk)
  bool ok = true;
  // the copier's counts of chunks whose loads were issued
  int64_t loads_issued = nchunks > 0 ? 1 : 0, p_issued = nchunks > 0 && outputs ? 1 : 0;
  const uint32_t idA = tc::idesc(tc::kBF16, 128, 64, false, true);
  const uint32_t idT = tc::idesc(tc::kBF16, 128, 64, true, true);
  int64_t ystage_tok = -1;  // first token of the full chunk whose output rows wait in the staging tile
  // The output product P D of a chunk is issued after the chunk's state update and read back during the
  // next chunk, so that neither it nor the output rows sit on the chain of dependent chunks: yq holds
  // that chunk's gamma Q S^T rows (Q-side lanes) until then, prev_tok / prev_L its place.
  float yq[16];
  int64_t prev_tok = -1;
  int prev_L = 0;
  // the output rows of the chunk whose P D is in TMEM at cO
  auto out_rows = [&](float (&y8)[8]) {
    float o2[16], u[16];
    tmem_ld_hl16(tl + cO, half, o2);
#pragma unroll
    for (int j = 0; j < 16; ++j) u[j] = o2[j] + __shfl_xor_sync(0xffffffffu, o2[j], 16);
    // both lanes hold P D's row; the K-side lane forms columns 0-7 (with the Q-side lane's gamma Q S^T),
    // the Q-side lane columns 8-15
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float qy = __shfl_xor_sync(0xffffffffu, yq[j], 16);
      y8[j] = kside ? u[j] + qy : u[8 + j] + yq[8 + j];
    }
  };
  // ... into the staging tile (full chunks, stored by one TMA store after the next barrier) or straight
  // to global memory (the rows of a short chunk before the sequence's end)
  auto put_rows = [&](const float (&y8)[8]) {
    const int hc = kside ? 0 : 1;
    if (prev_L == C) {
      // bf16 rows (64 bytes) in the 64-byte swizzle of the output map: 16-byte chunk c of row r at
      // c ^ ((r >> 1) & 3), which spreads a quarter-warp's eight rows over all banks
      if constexpr (sizeof(Tout) == 2)
        store_row8<Tout>(reinterpret_cast<Tout*>(smem + FW_Y + i_row * 64 + (((2 * half + hc) ^ ((i_row >> 1) & 3)) << 4)),
                         y8);
      else
        store_row8<Tout>(reinterpret_cast<Tout*>(smem + FW_Y) + i_row * DVT + 16 * half + 8 * hc, y8);
    } else if (i_row < prev_L) {  // the rows after a sequence's end belong to the next sequence
      store_row8<Tout>(static_cast<Tout*>(a.y) + ((prev_tok + i_row) * Hv + hv) * (size_t)DV + dv0 + 16 * half + 8 * hc,
                       y8);
    }
  };

  for (int64_t jc = 0; jc < nchunks; ++jc) {
    const int buf = (int)(jc & 1);
    const int64_t cg = c_first + jc;
    const int64_t tok0 = seq0 + jc * C;
    const int L = (int)min((int64_t)C, seq1 - tok0);

    // 1. the chunk-start state as the [hi | lo] operand row dk
    if (epi) tc::st_row_hilo16(smem + FW_S, dk, s, half);
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    const uint32_t kq = tc::smem_u32(smem + FW_KQ + buf * 32768);
    // 2. [K; Q] S^T in one pass (M = 128, N = 64: the state's hi and lo halves); the commit also covers
    //    the last chunk's P D, issued after it
    if (issuer) {
      ok = tc::mbar_wait_or_drain(&bar_tma[buf], (uint32_t)((jc >> 1) & 1), a.err, 10, s_hook);
      tc::fence_after_sync();
      if (ok) {
        mma_run<8, kKmaj128>(tmem + cA, idA, kq, tc::smem_u32(smem + FW_S), false);
        tc::mma_commit(&bar_mma);
      }
    }
    if (copier) {
      if (ystage_tok >= 0) tc::tma_store_3d(&ymap, smem + FW_Y, dv0, hv, (int)ystage_tok);  // an earlier chunk's rows
      tc::bulk_commit();
      // the next chunk's tiles into the buffers of the chunk before this one (whose readers are done);
      // its P image once that chunk's P D, which this round's commit covers, has completed
      if (jc + 1 < nchunks) {
        issue_loads(jc + 1), loads_issued = jc + 2;
        if (outputs) {
          ok = tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 11, s_hook);
          if (ok) issue_p(jc + 1), p_issued = jc + 2;
        }
      }
    }
    float bi = 0.f, be = 0.f, gi = 0.f, bC = 0.f, yp[16];
    if (epi) {
      // meanwhile (training) the chunk-start state, rounded to tf32 (its one reader takes it as a tf32
      // operand), staged for the bulk store of the checkpoint after the next barrier
      if (a.ckpt) {
        float* ck = reinterpret_cast<float*>(smem + FW_CK) + 16 * half * DK + dk;
#pragma unroll
        for (int j = 0; j < 16; ++j) ck[j * DK] = tf32_rna(s[j]);
      }
      ok = ok && tc::mbar_wait_or_drain(&bar_tma[buf], (uint32_t)((jc >> 1) & 1), a.err, 10, s_hook);
      const float* gb = sg[buf];
      bi = gb[i_row], be = gb[64 + i_row], gi = __expf(bi), bC = gb[63];
      float vr[16];  // this row's values (rows past the sequence's end read as zero)
      {
        Row16 raw;
        // the tile in the 64-byte swizzle of its map: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)
        const uint8_t* vrow = smem + FW_V + buf * 4096 + i_row * 64;
        const int sw = (i_row >> 1) & 3;
        raw.w[0] = i_row < L ? *reinterpret_cast<const uint4*>(vrow + (((2 * half) ^ sw) << 4)) : make_uint4(0, 0, 0, 0);
        raw.w[1] = i_row < L ? *reinterpret_cast<const uint4*>(vrow + (((2 * half + 1) ^ sw) << 4)) : make_uint4(0, 0, 0, 0);
        cvt_row16(raw, vr);
      }
      ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 11, s_hook);
      tc::fence_after_sync();
      // 3. K side: E = diag(beta) (V - diag(gamma) K S^T) as the [hi | lo] operand; Q side: gamma Q S^T.
      //    One instruction stream for the lane pair: the K-side lane forms E's columns 0-7 from its
      //    K S^T row, the Q-side lane columns 8-15 from the K-side lane's; the Q-side lane keeps gamma Q S^T
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
    ph ^= 1;
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 4. D = T E  ([T_hi; T_lo] stacked: row i's two products in lanes l and l + 16)
    if (issuer) {
      mma_run<4, kKmaj128>(tmem + cD, idA, tc::smem_u32(smem + FW_T + buf * 16384), tc::smem_u32(smem + FW_E), false);
      tc::mma_commit(&bar_mma);
    }
    if (copier && a.ckpt) {
      tc::bulk_store(a.ckpt + ((cg * Hv + hv) * DV + dv0) * (size_t)DK, smem + FW_CK, DVT * DK * 4);
      tc::bulk_commit();
    }
    if (copier) tc::bulk_wait_read();  // the staging tiles are rewritten below and next chunk
    float y8[8], ds8[8];
    const bool rows = outputs && prev_tok >= 0;
    if (epi) {
      // meanwhile the last chunk's output rows (its P D completed before this chunk's K S^T)
      if (rows) out_rows(y8);
#pragma unroll
      for (int j = 0; j < 16; ++j) yq[j] = yp[j];
      ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 12, s_hook);
      tc::fence_after_sync();
      // both lanes of the pair hold row i of D; one instruction stream for both: the K-side lane writes
      // D as the [hi | lo] operand of P D and keeps columns 0-7 of the tf32 copy, the Q-side lane
      // D~ = diag(lambda) D for the state update and columns 8-15 of the copy
      float d[16];
      tmem_ld_hl16_pair(tl + cD, half, d);
#pragma unroll
      for (int j = 0; j < 8; ++j) ds8[j] = tf32_rna(kside ? d[j] : d[8 + j]);
      const float sc = kside ? 1.f : __expf(bC - bi);
#pragma unroll
      for (int j = 0; j < 16; ++j) d[j] *= sc;
      tc::st_row_hilo16(smem + (kside ? FW_D : FW_DT), i_row, d, half);
    }
    ph ^= 1;
    tc::fence_async_smem();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;
    tc::fence_after_sync();
    if (!ok) break;
    // 5. S update^T = K^T D~ (M = 128 dk rows), committed alone; then O2 = P D ([P_hi; P_lo] stacked),
    //    whose completion the next chunk's first commit (or the one after the walk's last barrier)
    //    covers.  (Not a second commit here: a thread that polled late would find the barrier two
    //    phases on, the parity it waits for current again.)
    if (issuer && outputs) {  // (recompute mode: D was the product)
      mma_run<4, kKT>(tmem + cS, idT, kq, tc::smem_u32(smem + FW_DT), false);
      tc::mma_commit(&bar_mma);
      ok = tc::mbar_wait_or_drain(&bar_p[buf], (uint32_t)((jc >> 1) & 1), a.err, 15, s_hook);
      tc::fence_after_sync();
      if (ok)
        mma_run<4, kKmaj128>(tmem + cO, idA, tc::smem_u32(smem + FW_P + buf * 16384), tc::smem_u32(smem + FW_D), false);
    }
    ystage_tok = -1;
    if (epi) {
      // meanwhile D (tf32-rounded: the gradient kernel's tf32 operand, loaded as is) into its tile
      // [64 rows][32] (16-byte chunks swizzled by the row), and the last chunk's output rows
      if (a.Ds) {
        uint8_t* row = reinterpret_cast<uint8_t*>(a.Ds + ((size_t)(cg * Hv + hv) * (DV / DVT) + blockIdx.x) * 2048) +
                       i_row * 128;
        const int q0 = 4 * half + (kside ? 0 : 2);
#pragma unroll
        for (int q = 0; q < 2; ++q)
          *reinterpret_cast<float4*>(row + (((q0 + q) ^ (i_row & 7)) << 4)) =
              make_float4(ds8[4 * q], ds8[4 * q + 1], ds8[4 * q + 2], ds8[4 * q + 3]);
      }
      if (rows) put_rows(y8);
    }
    if (rows && prev_L == C) ystage_tok = prev_tok;
    prev_tok = tok0, prev_L = L;
    if (outputs && epi) {  // (the phase is not used in recompute mode, whose walk ends here)
      ok = ok && tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 13, s_hook);
      tc::fence_after_sync();
      float u[16];
      tmem_ld_hl16(tl + cS, half, u);
      const float gC = __expf(bC);
#pragma unroll
      for (int j = 0; j < 16; ++j) s[j] = fmaf(gC, s[j], u[j]);
    }
    ph ^= 1;
    tc::fence_async_smem();
    tc::fence_before_sync();
  }
  ok = __syncthreads_and(ok) != 0;  // (the last round's waits were per thread)
  if (!ok) {  // a wait gave up: everything still in flight lands before the TMEM and the CTA go
    if (issuer) {  // every product this thread issued
      tc::mma_commit(&bar_drain);
      tc::mbar_drain(&bar_drain, 0);
    }
    if (copier) {  // each buffer's latest loads (the earlier ones were waited for)
      for (int64_t j = loads_issued > 2 ? loads_issued - 2 : 0; j < loads_issued; ++j)
        tc::mbar_drain(&bar_tma[j & 1], (uint32_t)((j >> 1) & 1));
      for (int64_t j = p_issued > 2 ? p_issued - 2 : 0; j < p_issued; ++j)
        tc::mbar_drain(&bar_p[j & 1], (uint32_t)((j >> 1) & 1));
    }
  }
  if (ok && outputs && prev_tok >= 0) {  // the last chunk's output rows, after the staged ones go out
    if (issuer) tc::mma_commit(&bar_mma);  // every thread saw the round before complete
    if (copier && ystage_tok >= 0) {
      tc::tma_store_3d(&ymap, smem + FW_Y, dv0, hv, (int)ystage_tok);
      tc::bulk_commit();
      tc::bulk_wait_read();
    }
    float y8[8];
    if (epi) {
      ok = tc::mbar_wait_or_drain(&bar_mma, ph, a.err, 14, s_hook);
      tc::fence_after_sync();
      out_rows(y8);
    }
    tc::fence_before_sync();
    ok = __syncthreads_and(ok) != 0;  // (the staging tile is free)
    tc::fence_after_sync();
    if (ok && epi) put_rows(y8);
    tc::fence_async_smem();
    __syncthreads();
    if (ok && prev_L == C && copier) {
      tc::tma_store_3d(&ymap, smem + FW_Y, dv0, hv, (int)prev_tok);
      tc::bulk_commit();
    }
  }
  if (copier) tc::bulk_wait();
  if (ok && outputs && epi && a.hT) {
    float* dst = a.hT + (((size_t)n * Hv + hv) * DV + dv0 + 16 * half) * DK + dk;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[(size_t)j * DK] = s[j];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

cudaError_t launch_chunk_fwd_state(const CUtensorMap& vmap, const CUtensorMap& ymap, const StateArgs& a, int Hv, int N,
                                   bool out_bf16, cudaStream_t st) {
  auto kern = out_bf16 ? gdn_chunk_fwd_state<__nv_bfloat16> : gdn_chunk_fwd_state<float>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FW_SMEM);
  if (e != cudaSuccess) return e;
  // recompute mode: one CTA per (slice, value head, chunk)
  kern<<<dim3(DV / DVT, Hv, a.ckpt_in ? (unsigned)a.geo_chunks : (unsigned)N), 320, FW_SMEM, st>>>(vmap, ymap, a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
