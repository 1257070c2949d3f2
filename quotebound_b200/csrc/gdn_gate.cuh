// Host-visible interface of the gate / beta / q-k norm kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace qbgdn {

struct GateArgs {
  int64_t P;  // tokens
  int Hk, Hv, Dk;
  const void *q, *k;              // [P, Hk, Dk] input dtype
  const float *a, *b;             // [P, Hv]
  const float *A_log, *dt_bias;   // [Hv]
  void *qn, *kn;                  // forward outputs, output dtype
  float *g, *beta;                // forward outputs [P, Hv]
  const void *dqn, *dkn;          // backward inputs, input dtype
  const float *dg, *dbeta;        // backward inputs [P, Hv]
  void *dq, *dk;                  // backward outputs, output dtype
  float *da, *db;                 // [P, Hv]
  float *dA_log, *ddt_bias;       // [Hv]
};

int gate_head_blocks(int64_t P);
cudaError_t gate_fwd(const GateArgs& a, int in_bf16, int out_bf16, cudaStream_t st);
cudaError_t gate_bwd(const GateArgs& a, int in_bf16, int out_bf16, float* partial, cudaStream_t st);

}  // namespace qbgdn
