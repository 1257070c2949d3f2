// The generic backward of the recurrence on CUDA cores, in float32: any Dk in {32, 64, 128, 256},
// any Dv, float32 or bf16 activations.  It serves every call the tensor-core path does not (float32
// activations -- the reference's own dtype, src/deltanet.cpp:54-59, src/delta_grad.cpp:169-170 --
// and shapes other than Dk = Dv = 128).
//
// It is the chunked (WY) form of the backward, the same decomposition as the tensor-core kernels but
// with every product an fp32 FMA: per chunk of C = 64 steps with start state S (from the forward's
// chunk-start states) the chunk's outputs are O = diag(gamma) Q S^T + P D and its end state
// S' = gamma_C S + D^T diag(lambda) K, with D = T E, E = diag(beta) (V - diag(gamma) K S^T),
// T = (I + L)^-1, L = strict-lower(beta_i Gamma_ij (K K^T)_ij), P = lower(Gamma_ij (Q K^T)_ij),
// Gamma_ij = g_{j+1} ... g_i, gamma_i = Gamma_{i,-1}, lambda_j = Gamma_{C-1,j}.  Going back, with dS
// the cotangent of S' and dO that of O:
//   dD = P^T dO + diag(lambda) K dS^T,  F = T^T dD,  dV = diag(beta) F,
//   dS_start = gamma_C dS + (diag(gamma) dO)^T Q - (diag(beta gamma) F)^T K,
//   dQ = diag(gamma) dO S + dP^ K,  dK = dP^^T Q + diag(lambda) D dS - diag(beta gamma) F S + dKK K + dKK^T K,
//   dP^ = Gamma (.) (dO D^T) (lower),  dKK = -beta_i Gamma_ij (F D^T)_ij (strict lower),
//   dbeta_i = F_i . V_i - gamma_i F_i . (S k_i) + sum_j (-F D^T)_ij Gamma_ij (K K^T)_ij.
// The gate gradient is formed directly, not as d log g / g: every gate product Gamma_ij that spans
// step t (j < t <= i) contributes f_ij Gamma_it Gamma_{t-1,j} to dg_t, where f_ij is the product's
// coefficient in the loss (the extended index j = -1 stands for the chunk start: the gamma terms).
// Every factor is a product of gates, so a gate near zero (g ~ 1e-30) still gets dg to full relative
// precision, with no division and no cancellation.
//
// Kernels (256 threads each):
//   cc_prep     (chunks, Hk)          K K^T, Q K^T; per value head the gate products Gamma (running
//                                     products down each column), L, P and T by forward substitution
//   cc_delta    (chunks, Hv, Dv/32)   K S^T, Q S^T from the chunk-start state, E, D = T E
//   cc_walk     (sequences, Hv, Dv/R) the chunks in reverse with R rows of dS in shared memory: dD, F,
//                                     dV, the chunk's dS kept for the gradient kernels, dS carried
//   cc_grad_rows (chunks, Hv)         dO D^T, F D^T and the row terms over Dv; dg, dbeta, dP^, dKK
//   cc_grad_qk  (chunks, Hk, Dk/32)   dQ, dK for a 32-column tile, the value heads of the key head
//                                     summed in head order (deterministic, no atomics)
// The workspace holds every intermediate in fp32 (about (7 Dv + 2 Dv Dk / 64 + 200) floats per
// token and value head).
#include "gdn_cc.cuh"
#include "gdn_common.cuh"
#include "launch_count.cuh"

namespace qbgdn {

namespace {

constexpr int C = kChunk;
constexpr int NT = 256;

__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Fixed-order sum over the block's 256 threads (thread 0 gets the total).
__device__ __forceinline__ float block_sum(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < NT / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

// The four lanes of a quad (lanes 4m .. 4m + 3) summed, the same order in every quad.
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Per (chunk, key head): K K^T and Q K^T, then for each value head of the group the gate products,
// L, P and T.  Gamma_e[i][e] = Gamma_{i, e-1}: column 0 holds gamma_i, column j + 1 Gamma_ij (j <= i).
template <typename Tin>
__global__ void __launch_bounds__(NT) cc_prep(CcArgs a) {
  extern __shared__ float smem[];
  float(*sk)[33] = reinterpret_cast<float(*)[33]>(smem);                       // [C][33]
  float(*sq)[33] = reinterpret_cast<float(*)[33]>(smem + C * 33);              // [C][33]
  float(*sG)[C + 1] = reinterpret_cast<float(*)[C + 1]>(smem + 2 * C * 33);   // [C][C + 1]
  float(*sL)[C + 1] = sG + C;                                                  // [C][C + 1]
  float(*sT)[C + 1] = sL + C;                                                  // [C][C + 1]
  float* sg = smem + 2 * C * 33 + 3 * C * (C + 1);                             // [C]
  float* sb = sg + C;                                                          // [C]
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const int hk = blockIdx.y, Hk = a.geo.Hk, Hv = a.geo.Hv, ratio = Hv / Hk, Dk = a.Dk;
  int n, L;
  int64_t tok0;
  chunk_info(a.geo, c, n, tok0, L);
  const Tin* q = static_cast<const Tin*>(a.q);
  const Tin* k = static_cast<const Tin*>(a.k);

  // thread t: row i = t / 4, columns j0 .. j0 + 15 of both products
  const int i = tid >> 2, j0 = (tid & 3) * 16;
  float kk[16], qk[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) kk[u] = qk[u] = 0.f;
  for (int d0 = 0; d0 < Dk; d0 += 32) {
    for (int e = tid; e < C * 32; e += NT) {
      const int r = e >> 5, col = e & 31;
      const size_t off = ((size_t)(tok0 + r) * Hk + hk) * Dk + d0 + col;
      sk[r][col] = r < L ? to_f(k[off]) : 0.f;
      sq[r][col] = r < L ? to_f(q[off]) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int d = 0; d < 32; ++d) {
      const float ki = sk[i][d], qi = sq[i][d];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        kk[u] = fmaf(ki, sk[j0 + u][d], kk[u]);
        qk[u] = fmaf(qi, sk[j0 + u][d], qk[u]);
      }
    }
    __syncthreads();
  }
  {
    float* gk = a.kk + ((size_t)(c * Hk + hk) * C + i) * C + j0;
    float* gq = a.qk + ((size_t)(c * Hk + hk) * C + i) * C + j0;
#pragma unroll
    for (int u = 0; u < 16; ++u) gk[u] = kk[u], gq[u] = qk[u];
  }

  for (int r = 0; r < ratio; ++r) {
    const int hv = hk * ratio + r;
    const size_t ch = (size_t)c * Hv + hv;
    if (tid < C) {  // steps past the end: g = 1, beta = 0 (they change nothing)
      const bool v = tid < L;
      sg[tid] = v ? a.g[(tok0 + tid) * Hv + hv] : 1.f;
      sb[tid] = v ? a.beta[(tok0 + tid) * Hv + hv] : 0.f;
    }
    __syncthreads();
    // gate products: column e of Gamma_e runs down the rows as one running product
    if (tid <= C) {
      const int j = tid - 1;
      float p = 1.f;
      for (int ii = 0; ii < C; ++ii) {
        if (ii > j) p *= sg[ii];
        sG[ii][tid] = ii >= j ? p : 0.f;
      }
    }
    __syncthreads();
    {
      float* gp = a.pm + (ch * C + i) * C + j0;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int j = j0 + u;
        const float gam = sG[i][j + 1];
        sL[i][j] = j < i ? sb[i] * gam * kk[u] : 0.f;
        gp[u] = j <= i ? gam * qk[u] : 0.f;
      }
    }
    __syncthreads();
    // T = (I + L)^-1 by forward substitution down the rows: column j = t / 4, the quad splits the sum
    {
      const int j = tid >> 2, part = tid & 3;
      for (int ii = 0; ii < C; ++ii) {
        float s = 0.f;
        for (int m = part; m < ii; m += 4) s = fmaf(sL[ii][m], sT[m][j], s);
        s = quad_sum(s);
        if (part == 0) sT[ii][j] = (ii == j ? 1.f : 0.f) - s;
        __syncwarp();
      }
    }
    __syncthreads();
    {
      float* gt = a.tm + ch * C * C;
      for (int e = tid; e < C * C; e += NT) gt[e] = sT[e >> 6][e & 63];
      float* gg = a.gam + ch * C * (C + 1);
      for (int e = tid; e < C * (C + 1); e += NT) gg[e] = sG[e / (C + 1)][e % (C + 1)];
      if (tid < C) {
        float* gs = a.gates + ch * 4 * C;
        gs[tid] = sb[tid];                  // beta
        gs[C + tid] = sG[tid][0];           // gamma
        gs[2 * C + tid] = sG[C - 1][tid + 1];  // lambda
        gs[3 * C + tid] = sg[tid];          // g
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// Per (chunk, value head, 32 value rows): K S^T, Q S^T from the chunk-start state, E, D = T E.
template <typename Tin>
__global__ void __launch_bounds__(NT) cc_delta(CcArgs a) {
  __shared__ float sk[C][33], sq[C][33], ss[32][33], sE[C][33], sT[C][C + 1];
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const int hv = blockIdx.y, Hk = a.geo.Hk, Hv = a.geo.Hv, hk = hv / (Hv / Hk), Dk = a.Dk, Dv = a.Dv;
  const int v0 = blockIdx.z * 32, nv = min(32, Dv - v0);
  int n, L;
  int64_t tok0;
  chunk_info(a.geo, c, n, tok0, L);
  const size_t ch = (size_t)c * Hv + hv;
  const Tin* q = static_cast<const Tin*>(a.q);
  const Tin* k = static_cast<const Tin*>(a.k);
  const Tin* v = static_cast<const Tin*>(a.v);

  const int i = tid >> 2, w0 = (tid & 3) * 8;  // row i, value columns w0 .. w0 + 7 of the tile
  float ks[8], qs[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) ks[u] = qs[u] = 0.f;
  const float* S = a.ckpt + (ch * Dv + v0) * Dk;
  for (int d0 = 0; d0 < Dk; d0 += 32) {
    for (int e = tid; e < C * 32; e += NT) {
      const int r = e >> 5, col = e & 31;
      const size_t off = ((size_t)(tok0 + r) * Hk + hk) * Dk + d0 + col;
      sk[r][col] = r < L ? to_f(k[off]) : 0.f;
      sq[r][col] = r < L ? to_f(q[off]) : 0.f;
    }
    for (int e = tid; e < 32 * 32; e += NT) {
      const int r = e >> 5, col = e & 31;
      ss[r][col] = r < nv ? S[(size_t)r * Dk + d0 + col] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int d = 0; d < 32; ++d) {
      const float ki = sk[i][d], qi = sq[i][d];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        ks[u] = fmaf(ki, ss[w0 + u][d], ks[u]);
        qs[u] = fmaf(qi, ss[w0 + u][d], qs[u]);
      }
    }
    __syncthreads();
  }
  const float* gs = a.gates + ch * 4 * C;
  const float be = gs[i], ga = gs[C + i];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int w = w0 + u;
    const float vv = (i < L && w < nv) ? to_f(v[((size_t)(tok0 + i) * Hv + hv) * Dv + v0 + w]) : 0.f;
    sE[i][w] = be * (vv - ga * ks[u]);
    if (w < nv) {
      const size_t o = (ch * C + i) * Dv + v0 + w;
      a.ks[o] = ks[u];
      a.qs[o] = qs[u];
    }
  }
  for (int e = tid; e < C * C; e += NT) sT[e >> 6][e & 63] = a.tm[ch * C * C + e];
  __syncthreads();
  float dl[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) dl[u] = 0.f;
  for (int m = 0; m <= i; ++m) {
    const float t = sT[i][m];
#pragma unroll
    for (int u = 0; u < 8; ++u) dl[u] = fmaf(t, sE[m][w0 + u], dl[u]);
  }
#pragma unroll
  for (int u = 0; u < 8; ++u)
    if (w0 + u < nv) a.dl[(ch * C + i) * Dv + v0 + w0 + u] = dl[u];
}

// ------------------------------------------------------------------------------------------------
// The reverse walk: one CTA per (sequence, value head, RB rows of dS), the chunks backwards.
template <int RB, typename Tin, typename Tout>
__global__ void __launch_bounds__(NT) cc_walk(CcArgs a) {
  extern __shared__ float smem[];
  const int Dk = a.Dk, Dv = a.Dv, Hk = a.geo.Hk, Hv = a.geo.Hv;
  const int KP = Dk + 1;  // padded row
  float* sK = smem;                   // [C][KP]
  float* sQ = sK + C * KP;            // [C][KP]
  float* sdS = sQ + C * KP;           // [RB][KP]
  float* sT = sdS + RB * KP;          // [C][C + 1]
  float* sP = sT + C * (C + 1);       // [C][C + 1]
  float* sdO = sP + C * (C + 1);      // [C][RB + 1]
  float* sX = sdO + C * (RB + 1);     // [C][RB + 1]  X = K dS^T, then gamma dO
  float* sDD = sX + C * (RB + 1);     // [C][RB + 1]  dD, then beta gamma F
  float* sF = sDD + C * (RB + 1);     // [C][RB + 1]
  float* sgt = sF + C * (RB + 1);     // beta, gamma, lambda [3][C]
  float* sred = sgt + 3 * C;          // [8]
  const int RP = RB + 1;

  const int tid = threadIdx.x;
  const int n = blockIdx.x, hv = blockIdx.y, hk = hv / (Hv / Hk);
  const int r0 = blockIdx.z * RB, nr = min(RB, Dv - r0);
  int64_t c_first, nchunks, seq0, seq1;
  seq_chunks(a.geo, n, c_first, nchunks, seq0, seq1);
  const Tin* q = static_cast<const Tin*>(a.q);
  const Tin* k = static_cast<const Tin*>(a.k);
  const Tin* dy = static_cast<const Tin*>(a.dy);
  Tout* dv = static_cast<Tout*>(a.dv);
  const size_t srow = ((size_t)n * Hv + hv) * Dv + r0;  // first state row of this block

  for (int e = tid; e < RB * Dk; e += NT) {
    const int r = e / Dk, d = e - r * Dk;
    sdS[r * KP + d] = (r < nr && a.dhT) ? a.dhT[(srow + r) * Dk + d] : 0.f;
  }
  const int i = tid >> 2, rg = (tid & 3) * (RB / 4);  // row i, dS rows rg .. rg + RB/4 - 1
  constexpr int RU = RB / 4;
  for (int64_t it = 0; it < nchunks; ++it) {
    const int64_t jc = nchunks - 1 - it, cg = c_first + jc, tok0 = seq0 + jc * C;
    const int L = (int)min((int64_t)C, seq1 - tok0);
    const size_t ch = (size_t)cg * Hv + hv;
    __syncthreads();  // the previous chunk's readers are done
    for (int e = tid; e < C * Dk; e += NT) {
      const int r = e / Dk, d = e - r * Dk;
      const size_t off = ((size_t)(tok0 + r) * Hk + hk) * Dk + d;
      sK[r * KP + d] = r < L ? to_f(k[off]) : 0.f;
      sQ[r * KP + d] = r < L ? to_f(q[off]) : 0.f;
    }
    for (int e = tid; e < C * C; e += NT) {
      sT[(e >> 6) * (C + 1) + (e & 63)] = a.tm[ch * C * C + e];
      sP[(e >> 6) * (C + 1) + (e & 63)] = a.pm[ch * C * C + e];
    }
    for (int e = tid; e < C * RB; e += NT) {
      const int r = e / RB, w = e - r * RB;
      sdO[r * RP + w] = (r < L && w < nr) ? to_f(dy[((size_t)(tok0 + r) * Hv + hv) * Dv + r0 + w]) : 0.f;
    }
    if (tid < 3 * C) sgt[tid] = a.gates[ch * 4 * C + tid];
    // this chunk's end-state cotangent, kept for the gradient kernels, and its share of <S, dS>
    float st = 0.f;
    for (int e = tid; e < nr * Dk; e += NT) {
      const int r = e / Dk, d = e - r * Dk;
      const size_t o = (ch * Dv + r0 + r) * Dk + d;
      const float x = sdS[r * KP + d];
      a.dsb[o] = x;
      st = fmaf(x, a.ckpt[o], st);
    }
    st = block_sum(st, sred);
    if (tid == 0) a.st5p[ch * gridDim.z + blockIdx.z] = st;
    // X = K dS^T
    {
      float x[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) x[u] = 0.f;
      for (int d = 0; d < Dk; ++d) {
        const float kv = sK[i * KP + d];
#pragma unroll
        for (int u = 0; u < RU; ++u) x[u] = fmaf(kv, sdS[(rg + u) * KP + d], x[u]);
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) sX[i * RP + rg + u] = x[u];
    }
    __syncthreads();
    // dD = P^T dO + diag(lambda) X
    {
      const float lam = sgt[2 * C + i];
      float x[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) x[u] = lam * sX[i * RP + rg + u];
      for (int j = i; j < C; ++j) {
        const float p = sP[j * (C + 1) + i];
#pragma unroll
        for (int u = 0; u < RU; ++u) x[u] = fmaf(p, sdO[j * RP + rg + u], x[u]);
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) sDD[i * RP + rg + u] = x[u];
      // X is kept for the gate gradient: t4_i = D_i . X_i
#pragma unroll
      for (int u = 0; u < RU; ++u)
        if (rg + u < nr) a.xs[(ch * C + i) * Dv + r0 + rg + u] = sX[i * RP + rg + u];
    }
    __syncthreads();
    // F = T^T dD; dV = diag(beta) F
    {
      const float be = sgt[i], ga = sgt[C + i];
      float f[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) f[u] = 0.f;
      for (int j = i; j < C; ++j) {
        const float t = sT[j * (C + 1) + i];
#pragma unroll
        for (int u = 0; u < RU; ++u) f[u] = fmaf(t, sDD[j * RP + rg + u], f[u]);
      }
      __syncthreads();  // every read of sDD and sX above is done before they are reused
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int w = rg + u;
        sF[i * RP + w] = f[u];
        sX[i * RP + w] = ga * sdO[i * RP + w];  // gamma dO
        sDD[i * RP + w] = be * ga * f[u];       // beta gamma F
        if (w < nr) {
          a.fb[(ch * C + i) * Dv + r0 + w] = f[u];
          if (i < L) dv[((size_t)(tok0 + i) * Hv + hv) * Dv + r0 + w] = from_f<Tout>(be * f[u]);
        }
      }
    }
    __syncthreads();
    // dS <- gamma_C dS + (gamma dO)^T Q - (beta gamma F)^T K
    {
      const float gC = sgt[C + C - 1];
      for (int e = tid; e < RB * Dk; e += NT) {
        const int r = e / Dk, d = e - r * Dk;
        float x = gC * sdS[r * KP + d];
        for (int m = 0; m < C; ++m)
          x = fmaf(sX[m * RP + r], sQ[m * KP + d], fmaf(-sDD[m * RP + r], sK[m * KP + d], x));
        sdS[r * KP + d] = x;  // each element is read and written by its own thread only
      }
    }
  }
  __syncthreads();
  if (a.dh0)
    for (int e = tid; e < nr * Dk; e += NT) {
      const int r = e / Dk, d = e - r * Dk;
      a.dh0[(srow + r) * Dk + d] = sdS[r * KP + d];
    }
}

// ------------------------------------------------------------------------------------------------
// Per (chunk, value head): dO D^T and F D^T over Dv, the row terms, then dg, dbeta, dP^ and dKK.
template <typename Tin>
__global__ void __launch_bounds__(NT) cc_grad_rows(CcArgs a, int nrb) {
  extern __shared__ float smem[];
  float(*sO)[33] = reinterpret_cast<float(*)[33]>(smem);                       // [C][33] dO slice
  float(*sF)[33] = sO + C;                                                     // [C][33] F slice
  float(*sD)[33] = sF + C;                                                     // [C][33] D slice
  float(*sG)[C + 1] = reinterpret_cast<float(*)[C + 1]>(smem + 3 * C * 33);   // [C][C + 1]
  float(*sf)[C + 1] = sG + C;                                                  // [C][C + 1]
  float(*srow)[C] = reinterpret_cast<float(*)[C]>(smem + 3 * C * 33 + 2 * C * (C + 1));  // [4][C]
  float* sgt = smem + 3 * C * 33 + 2 * C * (C + 1) + 4 * C;                   // [4 C]
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const int hv = blockIdx.y, Hk = a.geo.Hk, Hv = a.geo.Hv, hk = hv / (Hv / Hk), Dv = a.Dv;
  int n, L;
  int64_t tok0;
  chunk_info(a.geo, c, n, tok0, L);
  const size_t ch = (size_t)c * Hv + hv;
  const Tin* dy = static_cast<const Tin*>(a.dy);
  const Tin* v = static_cast<const Tin*>(a.v);

  const int i = tid >> 2, part = tid & 3, j0 = part * 16;
  // row terms over Dv: F.V, F.KS (t2), dO.QS (t3), D.X (t4); the quad splits the columns
  {
    float fv = 0.f, t2 = 0.f, t3 = 0.f, t4 = 0.f;
    if (i < L) {
      const size_t rw = (ch * C + i) * Dv;
      const size_t tw = ((size_t)(tok0 + i) * Hv + hv) * Dv;
      for (int w = part; w < Dv; w += 4) {
        const float f = a.fb[rw + w];
        fv = fmaf(f, to_f(v[tw + w]), fv);
        t2 = fmaf(f, a.ks[rw + w], t2);
        t3 = fmaf(to_f(dy[tw + w]), a.qs[rw + w], t3);
        t4 = fmaf(a.dl[rw + w], a.xs[rw + w], t4);
      }
    }
    fv = quad_sum(fv), t2 = quad_sum(t2), t3 = quad_sum(t3), t4 = quad_sum(t4);
    if (part == 0) srow[0][i] = fv, srow[1][i] = t2, srow[2][i] = t3, srow[3][i] = t4;
  }
  // dO D^T and F D^T, Dv in slices of 32
  float dp[16], fd[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) dp[u] = fd[u] = 0.f;
  for (int w0 = 0; w0 < Dv; w0 += 32) {
    const int nw = min(32, Dv - w0);
    for (int e = tid; e < C * 32; e += NT) {
      const int r = e >> 5, w = e & 31;
      const bool ok = r < L && w < nw;
      const size_t rw = (ch * C + r) * Dv + w0 + w;
      sO[r][w] = ok ? to_f(dy[((size_t)(tok0 + r) * Hv + hv) * Dv + w0 + w]) : 0.f;
      sF[r][w] = ok ? a.fb[rw] : 0.f;
      sD[r][w] = ok ? a.dl[rw] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int w = 0; w < 32; ++w) {
      const float o = sO[i][w], f = sF[i][w];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        dp[u] = fmaf(o, sD[j0 + u][w], dp[u]);
        fd[u] = fmaf(f, sD[j0 + u][w], fd[u]);
      }
    }
    __syncthreads();
  }
  for (int e = tid; e < C * (C + 1); e += NT) sG[e / (C + 1)][e % (C + 1)] = a.gam[ch * C * (C + 1) + e];
  if (tid < 4 * C) sgt[tid] = a.gates[ch * 4 * C + tid];
  float st5 = 0.f;
  for (int b = 0; b < nrb; ++b) st5 += a.st5p[ch * nrb + b];
  __syncthreads();
  const float be = sgt[i], ga = sgt[C + i];
  // coefficients of the gate products (column 0: the gamma terms), dbeta, dP^ and dKK
  {
    const float* kk = a.kk + ((size_t)(c * Hk + hk) * C + i) * C + j0;
    const float* qk = a.qk + ((size_t)(c * Hk + hk) * C + i) * C + j0;
    float* gdp = a.dph + (ch * C + i) * C + j0;
    float* gdk = a.dkk + (ch * C + i) * C + j0;
    float dbl = 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int j = j0 + u;
      const float gam = sG[i][j + 1], kv = kk[u], qv = qk[u];
      float f = j < i ? dp[u] * qv - fd[u] * be * kv : 0.f;
      if (i == C - 1) f += srow[3][j];  // lambda_j (the end state's products)
      sf[i][j + 1] = f;
      if (j < i) dbl = fmaf(-fd[u] * gam, kv, dbl);
      gdp[u] = j <= i ? gam * dp[u] : 0.f;
      gdk[u] = j < i ? -be * gam * fd[u] : 0.f;
    }
    dbl = quad_sum(dbl);
    if (part == 0) {
      sf[i][0] = srow[2][i] - be * srow[1][i] + (i == C - 1 ? st5 : 0.f);
      if (i < L) a.dbeta[(tok0 + i) * Hv + hv] = srow[0][i] - ga * srow[1][i] + dbl;
    }
  }
  __syncthreads();
  // dg_t = sum_{i >= t} Gamma_{i,t} A_{i,t},  A_{i,t} = sum_{e <= t} f[i][e] Gamma_{t-1, e-1}
  // (Gamma_{-1,-1} = 1): thread (i, part) forms A for t in its 16 and its contribution to dg_t
  float* scon = smem;  // [C][C + 1] contributions, over the slices (3 C x 33 floats, free now)
  for (int tt = 0; tt < 16; ++tt) {
    const int t = part * 16 + tt;
    float A = 0.f;
    if (t == 0) {
      A = sf[i][0];
    } else {
      for (int e = 0; e <= t; ++e) A = fmaf(sf[i][e], sG[t - 1][e], A);
    }
    scon[t * (C + 1) + i] = i >= t ? sG[i][t + 1] * A : 0.f;
  }
  __syncthreads();
  if (tid < L) {
    float s = 0.f;
    for (int ii = tid; ii < C; ++ii) s += scon[tid * (C + 1) + ii];
    a.dg[(tok0 + tid) * Hv + hv] = s;
  }
}

// ------------------------------------------------------------------------------------------------
// Per (chunk, key head, 32 columns of Dk): dQ and dK, the value heads of the group in order.
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(NT) cc_grad_qk(CcArgs a) {
  extern __shared__ float smem[];
  float* sK = smem;               // [C][33]
  float* sQ = sK + C * 33;        // [C][33]
  float* sM = sQ + C * 33;        // [C][C + 1]  dP^
  float* sN = sM + C * (C + 1);   // [C][C + 1]  dKK
  float* sO = sN + C * (C + 1);   // [C][33]  dO slice
  float* sF = sO + C * 33;        // [C][33]  F slice
  float* sD = sF + C * 33;        // [C][33]  D slice
  float* sS = sD + C * 33;        // [32][33] S slice
  float* sE = sS + 32 * 33;       // [32][33] dS slice
  float* sgt = sE + 32 * 33;      // [4][C]
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x;
  const int hk = blockIdx.y, Hk = a.geo.Hk, Hv = a.geo.Hv, ratio = Hv / Hk, Dk = a.Dk, Dv = a.Dv;
  const int d0 = blockIdx.z * 32;
  int n, L;
  int64_t tok0;
  chunk_info(a.geo, c, n, tok0, L);
  const Tin* q = static_cast<const Tin*>(a.q);
  const Tin* k = static_cast<const Tin*>(a.k);
  const Tin* dy = static_cast<const Tin*>(a.dy);

  for (int e = tid; e < C * 32; e += NT) {
    const int r = e >> 5, d = e & 31;
    const size_t off = ((size_t)(tok0 + r) * Hk + hk) * Dk + d0 + d;
    sK[r * 33 + d] = r < L ? to_f(k[off]) : 0.f;
    sQ[r * 33 + d] = r < L ? to_f(q[off]) : 0.f;
  }
  const int i = tid >> 2, u0 = (tid & 3) * 8;  // row i, columns u0 .. u0 + 7 of the tile
  float dq[8], dk[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) dq[u] = dk[u] = 0.f;
  for (int r = 0; r < ratio; ++r) {
    const int hv = hk * ratio + r;
    const size_t ch = (size_t)c * Hv + hv;
    __syncthreads();
    for (int e = tid; e < C * C; e += NT) {
      sM[(e >> 6) * (C + 1) + (e & 63)] = a.dph[ch * C * C + e];
      sN[(e >> 6) * (C + 1) + (e & 63)] = a.dkk[ch * C * C + e];
    }
    if (tid < 4 * C) sgt[tid] = a.gates[ch * 4 * C + tid];
    __syncthreads();
    for (int j = 0; j < C; ++j) {
      const float mp = sM[i * (C + 1) + j], mt = sM[j * (C + 1) + i];
      const float nk = sN[i * (C + 1) + j] + sN[j * (C + 1) + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float kv = sK[j * 33 + u0 + u];
        dq[u] = fmaf(mp, kv, dq[u]);
        dk[u] = fmaf(mt, sQ[j * 33 + u0 + u], fmaf(nk, kv, dk[u]));
      }
    }
    float yq[8], yf[8], yd[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) yq[u] = yf[u] = yd[u] = 0.f;
    for (int w0 = 0; w0 < Dv; w0 += 32) {
      const int nw = min(32, Dv - w0);
      __syncthreads();
      for (int e = tid; e < C * 32; e += NT) {
        const int rr = e >> 5, w = e & 31;
        const bool ok = rr < L && w < nw;
        const size_t rw = (ch * C + rr) * Dv + w0 + w;
        sO[rr * 33 + w] = ok ? to_f(dy[((size_t)(tok0 + rr) * Hv + hv) * Dv + w0 + w]) : 0.f;
        sF[rr * 33 + w] = ok ? a.fb[rw] : 0.f;
        sD[rr * 33 + w] = ok ? a.dl[rw] : 0.f;
      }
      for (int e = tid; e < 32 * 32; e += NT) {
        const int w = e >> 5, d = e & 31;
        const size_t so = (ch * Dv + w0 + w) * Dk + d0 + d;
        sS[w * 33 + d] = w < nw ? a.ckpt[so] : 0.f;
        sE[w * 33 + d] = w < nw ? a.dsb[so] : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int w = 0; w < 32; ++w) {
        const float o = sO[i * 33 + w], f = sF[i * 33 + w], dd = sD[i * 33 + w];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float s0 = sS[w * 33 + u0 + u], s1 = sE[w * 33 + u0 + u];
          yq[u] = fmaf(o, s0, yq[u]);
          yf[u] = fmaf(f, s0, yf[u]);
          yd[u] = fmaf(dd, s1, yd[u]);
        }
      }
    }
    const float be = sgt[i], ga = sgt[C + i], lam = sgt[2 * C + i];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      dq[u] = fmaf(ga, yq[u], dq[u]);
      dk[u] = fmaf(lam, yd[u], fmaf(-be * ga, yf[u], dk[u]));
    }
  }
  if (i < L) {
    const size_t off = ((size_t)(tok0 + i) * Hk + hk) * Dk + d0 + u0;
    Tout* oq = static_cast<Tout*>(a.dq) + off;
    Tout* ok = static_cast<Tout*>(a.dk) + off;
#pragma unroll
    for (int u = 0; u < 8; ++u) oq[u] = from_f<Tout>(dq[u]), ok[u] = from_f<Tout>(dk[u]);
  }
}

// ------------------------------------------------------------------------------------------------
// Host side.
namespace {

int64_t a256(int64_t x) { return (x + 255) & ~int64_t(255); }

int walk_rows(int Dk) { return Dk >= 256 ? 16 : 32; }

size_t walk_smem(int Dk, int RB) {
  const int KP = Dk + 1;
  return sizeof(float) * ((size_t)2 * C * KP + (size_t)RB * KP + 2 * C * (C + 1) + 4 * C * (RB + 1) + 3 * C + 8);
}

size_t qk_smem() { return sizeof(float) * (5 * C * 33 + 2 * C * (C + 1) + 2 * 32 * 33 + 4 * C); }
size_t prep_smem() { return sizeof(float) * (2 * C * 33 + 3 * C * (C + 1) + 2 * C); }
size_t rows_smem() { return sizeof(float) * (3 * C * 33 + 2 * C * (C + 1) + 8 * C); }

}  // namespace

int64_t cc_ws_layout(int Hk, int Hv, int Dk, int Dv, int64_t n_chunks, char* base, CcArgs* out) {
  int64_t off = 0;
  auto take = [&](int64_t floats) {
    char* at = base ? base + off : nullptr;
    off += a256(floats * 4);
    return reinterpret_cast<float*>(at);
  };
  const int64_t nch = n_chunks * Hv, nck = n_chunks * Hk;
  const int nrb = ceil_div(Dv, walk_rows(Dk));
  CcArgs a{};
  a.kk = take(nck * C * C);
  a.qk = take(nck * C * C);
  a.tm = take(nch * C * C);
  a.pm = take(nch * C * C);
  a.gam = take(nch * C * (C + 1));
  a.gates = take(nch * 4 * C);
  a.ks = take(nch * C * Dv);
  a.qs = take(nch * C * Dv);
  a.dl = take(nch * C * Dv);
  a.xs = take(nch * C * Dv);
  a.fb = take(nch * C * Dv);
  a.dsb = take(nch * (int64_t)Dv * Dk);
  a.st5p = take(nch * nrb);
  a.dph = take(nch * C * C);
  a.dkk = take(nch * C * C);
  if (out) {
    CcArgs& o = *out;
    o.kk = a.kk, o.qk = a.qk, o.tm = a.tm, o.pm = a.pm, o.gam = a.gam, o.gates = a.gates;
    o.ks = a.ks, o.qs = a.qs, o.dl = a.dl, o.xs = a.xs, o.fb = a.fb, o.dsb = a.dsb, o.st5p = a.st5p;
    o.dph = a.dph, o.dkk = a.dkk;
  }
  return off;
}

template <typename Tin, typename Tout>
static cudaError_t cc_launch(const CcArgs& a, int N, cudaStream_t st) {
  const int Hk = a.geo.Hk, Hv = a.geo.Hv;
  const unsigned nc = (unsigned)a.n_chunks;
  cudaError_t e;
  if (nc > 0) {
    if ((e = cudaFuncSetAttribute(cc_prep<Tin>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem())) !=
        cudaSuccess)
      return e;
    cc_prep<Tin><<<dim3(nc, Hk), NT, prep_smem(), st>>>(a);
    note_launch();
    cc_delta<Tin><<<dim3(nc, Hv, ceil_div(a.Dv, 32)), NT, 0, st>>>(a);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const int RB = walk_rows(a.Dk);
  const size_t ws = walk_smem(a.Dk, RB);
  const dim3 wg(N, Hv, ceil_div(a.Dv, RB));
  if (RB == 32) {
    auto kern = cc_walk<32, Tin, Tout>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ws)) != cudaSuccess) return e;
    kern<<<wg, NT, ws, st>>>(a);
  } else {
    auto kern = cc_walk<16, Tin, Tout>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ws)) != cudaSuccess) return e;
    kern<<<wg, NT, ws, st>>>(a);
  }
  note_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (nc == 0) return cudaSuccess;
  if ((e = cudaFuncSetAttribute(cc_grad_rows<Tin>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rows_smem())) !=
      cudaSuccess)
    return e;
  cc_grad_rows<Tin><<<dim3(nc, Hv), NT, rows_smem(), st>>>(a, (int)wg.z);
  note_launch();
  const size_t qs = qk_smem();
  auto kq = cc_grad_qk<Tin, Tout>;
  if ((e = cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qs)) != cudaSuccess) return e;
  kq<<<dim3(nc, Hk, a.Dk / 32), NT, qs, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

cudaError_t cc_bwd(const CcArgs& a, int N, int in_bf16, int out_bf16, cudaStream_t st) {
  if (a.Dk % 32 || a.Dk > 256 || a.Dv < 1) return cudaErrorInvalidValue;
  if (in_bf16 && out_bf16) return cc_launch<__nv_bfloat16, __nv_bfloat16>(a, N, st);
  if (in_bf16) return cc_launch<__nv_bfloat16, float>(a, N, st);
  if (out_bf16) return cc_launch<float, __nv_bfloat16>(a, N, st);
  return cc_launch<float, float>(a, N, st);
}

}  // namespace qbgdn
