// The per-chunk gradient kernel of the tensor-core path.
#include "gdn_chunk_impl.cuh"

namespace qbgdn {

// 256 threads.  Warp w reads TMEM lanes 32 (w & 3) .. + 31 and handles columns 16 (w >> 2) .. + 15 of a
// 32-wide slice (32 (w >> 2) .. of the 64-wide finalize, 64 (w >> 2) .. of the 128-wide dk).  The
// stacked accumulators hold chunk row i = 16 (w & 3) + l in lane l ("lower": dQ, dO S, dP) and in lane
// l + 16 ("upper": dK, F S, D dS, F D^T).
template <typename Tout>
__global__ void __launch_bounds__(256, 1) gdn_chunk_bwd_grad(const __grid_constant__ CUtensorMap smap_mn,
                                                             const __grid_constant__ CUtensorMap dmap_mn,
                                                             const __grid_constant__ CUtensorMap vmap,
                                                             const __grid_constant__ CUtensorMap dqmap,
                                                             const __grid_constant__ CUtensorMap dkmap, GradArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float sgt[2][128];  // the value heads' gates: b[64], beta[64] (double-buffered)
  __shared__ float srow[6][2][64];           // per-row partial sums from both column halves
  __shared__ float sdb[65], sred[16];
  __shared__ float snorm[2][2][128];
  __shared__ uint64_t bar_kq, bar_h, bar_kk, bar_s[2], bar_mma, bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_hook[2];
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  // a 1-D grid, key heads fastest: the first CTAs take the lowest chunks of every key head, whose state
  // cotangents and [dO; F] rows the reverse walk (chunks high to low) wrote last and L2 may still hold
  const int64_t c = blockIdx.x / a.geo.Hk;
  const int hk = (int)(blockIdx.x % a.geo.Hk), Hv = a.geo.Hv, ratio = Hv / a.geo.Hk;
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
    tc::mbar_init(&bar_drain, 1);
    tc::load_hook(s_hook, a.err);
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
    tc::mbar_arrive_expect_tx(&bar_h, 512);
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
  // failure path bookkeeping: value heads and slices whose loads were issued, and those whose waits
  // this thread ran (the issuing thread's view is the one used)
  int h_issued = 1, h_seen = 0, s_issued = 1, s_seen = 0;
  bool ok = wait_all(&bar_kq, 0, a.err, 30, s_hook);
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
    ok = wait_all(&bar_h, (uint32_t)(r & 1), a.err, 31, s_hook);
    h_seen = r + 1;
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
    if (tid < 64) {  // this row's gate g_t for the gate gradient's recurrence (1 past the sequence's end)
      float lg = 0.f;
      if (tid < L) lg = a.g ? fmaxf(logf(in0), -88.f) : -expf(eA) * softplus_f(in0 + dtb);
      sdb[tid] = __expf(lg);
    }

    for (int sl = 0; sl < NSL && ok; ++sl) {
      const int q = r * NSL + sl, bs = q & 1;
      uint8_t* buf = smem + GR_BUF + bs * GR_BS;
      // each thread waits for the slice's data itself; the barrier at the end of the slice keeps the
      // buffers' reuse ordered and makes a failed wait everyone's
      if (ok) s_seen = q + 1;
      ok = ok && tc::mbar_wait_or_drain(&bar_s[bs], (uint32_t)((q >> 1) & 1), a.err, 37, s_hook);
      // the other buffer's last reader has finished (the finalize uses the second buffer, so the next
      // value head's first slice goes out during this head's last slice)
      if (ok && tid == 32 && q + 1 < ratio * NSL) {
        issue_slice(q + 1);
        s_issued = q + 2;
      }
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
        // (the V rows in the 64-byte swizzle of their map: chunk c of row r at c ^ ((r >> 1) & 3))
        const uint4 w = rvalid ? *reinterpret_cast<const uint4*>(buf + 57344 + i_row * 64 +
                                                                 (((2 * half + hc) ^ ((i_row >> 1) & 3)) << 4))
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
      ok = __syncthreads_and(ok && tc::mbar_wait_or_drain(&bar_mma, ph_mma, a.err, 34, s_hook)) != 0;
      ph_mma ^= 1;
      tc::fence_after_sync();
    }
    if (!ok) break;

    {  // the slices' S (.) dS, per warp (read by the gate gradient after the next barrier)
      float t5w = t5;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t5w += __shfl_xor_sync(0xffffffffu, t5w, o);
      if (lane == 0) sred[warp] = t5w;
    }

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
    ok = wait_all(&bar_kk, 0u, a.err, 35, s_hook);
    if (!ok) break;
    tc::fence_after_sync();
    float* scratch = reinterpret_cast<float*>(smem + GR_SCR);  // [64][65], then 4 x 64 column partials
    float dbl = 0.f;
    {
      // Lane l holds dP[i][32 half + 0..31], lane l + 16 holds F D^T there; one exchange leaves each
      // lane both for 16 columns: j0 = 32 half (lower lane), 32 half + 16 (upper lane).  K K^T row i
      // is in lane l, Q K^T row i in lane l + 16; two exchanges give each lane both for its columns.
      float v[32], kk32[32], dp[16], fd[16], kk[16], qk[16];
      tc::tmem_ld32(tl + cPF + 32 * half, v);
      tc::tmem_ld32(tl + cKK + 32 * half, kk32);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float x = __shfl_xor_sync(0xffffffffu, lower ? v[16 + k] : v[k], 16);
        const float y = __shfl_xor_sync(0xffffffffu, kk32[16 + k], 16);
        const float z = __shfl_xor_sync(0xffffffffu, kk32[k], 16);
        dp[k] = lower ? v[k] : x;
        fd[k] = lower ? x : v[16 + k];
        kk[k] = lower ? kk32[k] : y;
        qk[k] = lower ? z : kk32[16 + k];
      }
      const int j0 = 32 * half + (lower ? 0 : 16);
      // f_ij: the coefficient of the gate product Gamma_ij in the loss (P and L terms, strict lower;
      // the diagonal spans no step), at scratch[i][j + 1] -- column 0 takes the gamma terms below
      float ph[16], kh[16], xs[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int j = j0 + k;
        const float gam = j <= i_row ? __expf(bi - sg[j]) : 0.f;
        const float dl = j < i_row ? -fd[k] : 0.f;
        const float lv = gam * kk[k];  // L_ij / beta_i = Gamma_ij (K K^T)_ij
        dbl = fmaf(dl, lv, dbl);
        xs[k] = j < i_row ? fmaf(dp[k], qk[k], dl * be * kk[k]) : 0.f;
        ph[k] = dp[k] * gam;        // dP^
        kh[k] = dl * be * gam;      // dKK
      }
      if (i_row == 63) {  // row 63 is the chunk's end: the end state's products lambda_j
#pragma unroll
        for (int k = 0; k < 16; ++k) xs[k] += srow[3][0][j0 + k] + srow[3][1][j0 + k];
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) scratch[i_row * 65 + 1 + j0 + k] = xs[k];
      if (lower && half == 0) {  // column 0: the gamma terms (and the end state's gamma_C <S, dS>)
        float c0v = (srow[0][0][i_row] + srow[0][1][i_row]) - be * (srow[2][0][i_row] + srow[2][1][i_row]);
        if (i_row == 63)
          for (int w = 0; w < 8; ++w) c0v += sred[w];
        scratch[i_row * 65] = c0v;
      }
      const int rr = img_row(i_row), c0 = j0 >> 3;
      st_hilo16_chunks(smem + GR_FHI, smem + GR_FLO, rr, ph, c0);
      st_hilo16_chunks(smem + GR_FHI, smem + GR_FLO, rr + 16, kh, c0);
    }
    {  // the L terms of d beta, both lanes of the pair, per column half
      const float db2 = dbl + __shfl_xor_sync(0xffffffffu, dbl, 16);
      if (lower) srow[5][half][i_row] = db2;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // the next value head's gates (into the other gate buffer)
    if (r + 1 < ratio) {
      if (tid == 32) issue_head(r + 1);
      h_issued = r + 2;
    }
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
    // The gate gradient, formed directly (a gate near zero keeps full relative precision; no division):
    //   dg_t = sum_{i >= t} Gamma_{i,t} A_{i,t},  A_{i,t} = sum_{e <= t} f[i][e] Gamma_{t-1, e-1}
    // (e = 0 is the chunk start, Gamma_{t-1,-1} = gamma_{t-1}).  A is a linear recurrence in t,
    // A_{i,t+1} = g_t A_{i,t} + f[i][t+1], run as four 16-step segments per row (the four lanes of a
    // quad) joined by their carries.  The coefficients f (column 0: the gamma terms, row 63: the end
    // state's) and the gates g_t are in shared memory since the last barrier.
    // 1. thread (row i, segment part): its 16 values of A, then the contributions Gamma_{i,t} A_{i,t}
    //    in place over the consumed coefficients
    {
      const int i = tid >> 2, part = tid & 3, s0 = 16 * part;
      const float* fr = scratch + i * 65;
      float B[16], R[16];
      float b = 0.f, rr = 1.f;  // local sum over this segment's e, and Gamma_{t-1, s0-1}
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int t = s0 + u;
        b = u == 0 ? fr[t] : fmaf(sdb[t - 1], b, fr[t]);
        rr = u == 0 ? 1.f : rr * sdb[t - 1];
        B[u] = b, R[u] = rr;
      }
      const float gl = sdb[s0 + 15];
      const float bout = gl * b, rout = gl * rr;  // this segment's share of A and decay at t = s0 + 16
      float cin = 0.f;
      const int q0 = (lane & ~3);
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const float bq = __shfl_sync(0xffffffffu, bout, q0 + q);
        const float rq = __shfl_sync(0xffffffffu, rout, q0 + q);
        if (q < part) cin = fmaf(rq, cin, bq);
      }
      const float bi_ = sg[i];
      float* fw = scratch + i * 65;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int t = s0 + u;
        const float A = fmaf(R[u], cin, B[u]);
        fw[t] = i >= t ? __expf(bi_ - sg[t]) * A : 0.f;
      }
    }
    __syncthreads();
    // 2. dg_t = the column sums (fixed order: four 16-row partials, then their sum)
    {
      const int col = tid & 63, part = tid >> 6;
      float cs = 0.f;
#pragma unroll 4
      for (int i = 16 * part; i < 16 * part + 16; ++i) cs += scratch[i * 65 + col];
      scratch[64 * 65 + part * 64 + col] = cs;
    }
    __syncthreads();
    float pa = 0.f, pd = 0.f;  // layer mode: this row's share of the head's dA_log, ddt_bias
    if (tid < 64 && tid < L) {
      const int i = tid;
      const float* cp = scratch + 64 * 65;
      const float dgi = (cp[i] + cp[64 + i]) + (cp[128 + i] + cp[192 + i]);  // dg_i
      const float dl = sdb[i] * dgi;                                      // d log g_i = g_i dg_i
      const int64_t gi_idx = (tok0 + i) * Hv + hv;
      // d beta = F . (V - gamma R) + the L terms;  F . R = K . (F S) = t2
      const float gi_ = __expf(sg[i]);
      const float t1_ = (srow[1][0][i] + srow[1][1][i]) - gi_ * (srow[2][0][i] + srow[2][1][i]);
      const float dbe = t1_ + srow[5][0][i] + srow[5][1][i];
      if (a.g) {
        a.dg[gi_idx] = dgi;
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
    ok = wait_all(&bar_mma, ph_mma, a.err, 36, s_hook);
    ph_mma ^= 1;
    tc::fence_after_sync();
  }
  if (!ok) {  // a wait gave up: everything still in flight lands before the TMEM and the CTA go
    if (tid == 0) {  // every product this thread issued
      tc::mma_commit(&bar_drain);
      tc::mbar_drain(&bar_drain, 0);
    }
    if (tid == 32) {
      for (int m = h_seen; m < h_issued; ++m) tc::mbar_drain(&bar_h, (uint32_t)(m & 1));
      for (int q = s_seen; q < s_issued; ++q) tc::mbar_drain(&bar_s[q & 1], (uint32_t)((q >> 1) & 1));
    }
  }
  // f. dq (lower lanes) and dk (upper lanes) rows of this key head, 64 columns per thread (layer mode:
  //    through the norms to the raw q, k)
  if (!a.g) cp_async_wait_all();
  // A full chunk of a bf16 result leaves by four TMA stores of 64 x 64 tiles, staged where the raw rows
  // were (read before the norm's barrier below): plain stores of a thread's 64-column row put 16 bytes
  // into each of 32 rows 4 KB apart per instruction, and cost this phase thousands of cycles.  Other
  // chunks' rows (a sequence's last, whose rows past its end belong to the next) go out by plain stores.
  const bool tile_out = sizeof(Tout) == 2 && L == C;
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
    if (tile_out) {  // row i_row of the dq (lower) or dk (upper) tile, columns 64 half .. + 63
      uint8_t* row = smem + GR_RAW + (lower ? 0 : 16384) + half * 8192 + i_row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float* x = c < 4 ? v0 + 8 * c : v1 + 8 * (c - 4);
        *reinterpret_cast<uint4*>(row + ((c ^ (i_row & 7)) << 4)) =
            make_uint4(tc::pack_bf16(x[0], x[1]), tc::pack_bf16(x[2], x[3]), tc::pack_bf16(x[4], x[5]),
                       tc::pack_bf16(x[6], x[7]));
      }
    } else if (rvalid) {
      store_row32<Tout>(out, v0);
      store_row32<Tout>(out + 32, v1);
    }
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  if (ok && tile_out && tid == 32) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tc::tma_store_3d(&dqmap, smem + GR_RAW + h * 8192, 64 * h, hk, (int)tok0);
      tc::tma_store_3d(&dkmap, smem + GR_RAW + 16384 + h * 8192, 64 * h, hk, (int)tok0);
    }
    tc::bulk_commit();
    tc::bulk_wait();  // the staging stays in place until the stores have read it
  }
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
  if (!a.g) {
    // layer mode: the CTA that finishes last sums every chunk's head terms, in chunk order (the same
    // result whichever CTA it is):  dA_log[h], ddt_bias[h] = sum over chunks of head_part[c][h][0 | 1]
    if (tid == 0) {
      __threadfence();
      s_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int64_t nc = gridDim.x / a.geo.Hk;
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

cudaError_t launch_chunk_bwd_grad(const CUtensorMap& smap_mn, const CUtensorMap& dmap_mn, const CUtensorMap& vmap,
                                  const CUtensorMap& dqmap, const CUtensorMap& dkmap, const GradArgs& a,
                                  int64_t n_chunks, int Hk, bool out_bf16, cudaStream_t st) {
  auto kern = out_bf16 ? gdn_chunk_bwd_grad<__nv_bfloat16> : gdn_chunk_bwd_grad<float>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GR_SMEM);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)(n_chunks * Hk), 256, GR_SMEM, st>>>(smap_mn, dmap_mn, vmap, dqmap, dkmap, a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace qbgdn
