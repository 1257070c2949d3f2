// Host-visible interface of the CUDA-core chunked backward (gdn_cc.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_common.cuh"

namespace qbgdn {

struct CcArgs {
  Geo geo;
  int64_t n_chunks;
  int Dk, Dv;
  const void *q, *k, *v, *dy;  // activation dtype
  const float *g, *beta;       // [tokens, Hv]
  const float* ckpt;           // [chunks, Hv, Dv, Dk] the forward's chunk-start states
  const float* dhT;            // [N, Hv, Dv, Dk] or null
  void *dq, *dk, *dv;          // output dtype
  float *dg, *dbeta, *dh0;
  // workspace (cc_ws_layout)
  float *kk, *qk;              // [chunks, Hk, 64, 64]
  float *tm, *pm;              // [chunks, Hv, 64, 64]  T and P
  float* gam;                  // [chunks, Hv, 64, 65]  gate products (column 0: gamma)
  float* gates;                // [chunks, Hv, 4, 64]   beta, gamma, lambda, g
  float *ks, *qs, *dl, *xs, *fb;  // [chunks, Hv, 64, Dv]  K S^T, Q S^T, D, K dS^T, F
  float* dsb;                  // [chunks, Hv, Dv, Dk]  each chunk's end-state cotangent
  float* st5p;                 // [chunks, Hv, row blocks]  <S, dS> partials of the walk
  float *dph, *dkk;            // [chunks, Hv, 64, 64]  dP^ and dKK
};

// Carves the backward's intermediates from base (null: just the size in bytes).
int64_t cc_ws_layout(int Hk, int Hv, int Dk, int Dv, int64_t n_chunks, char* base, CcArgs* out);
// The backward from the forward's chunk-start states; N sequences.
cudaError_t cc_bwd(const CcArgs& a, int N, int in_bf16, int out_bf16, cudaStream_t st);

}  // namespace qbgdn
