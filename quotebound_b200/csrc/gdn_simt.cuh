// Host-visible interface of the row-parallel (SIMT) kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace qbgdn {

enum class SimtKind { Fwd, Step, Verify, Bwd };

// One struct for every row-parallel kernel; unused fields are null / zero.
struct SimtArgs {
  int T, Hk, Hv, Dk, Dv;
  int rows_per_block;          // warps per block; divides Dv for the backward
  const int32_t* cu;           // device offsets [N + 1] or null
  const int64_t* chunk_off;    // device, [N + 1] chunk offsets (varlen) or null
  const void *q, *k, *v, *dy;  // activation dtype
  const float *g, *beta;
  const float *h0, *dhT;       // [N, Hv, Dv, Dk] or null (step/verify: h0 = state_in)
  void *y, *dv;                // output dtype
  float *hT, *dh0;             // step: hT = state_out
  float* ckpt;                 // fwd: chunk starts out (or null); bwd: chunk starts in; verify: states out
  float *dq_part, *dk_part;    // [tokens, Hv, NB, Dk]
  float *dg_part, *dbeta_part; // [tokens, Hv, NB]
};

struct ReduceArgs {
  int64_t tokens;
  int Hk, Hv, Dk, NB;
  const float *dq_part, *dk_part, *dg_part, *dbeta_part;
  void *dq, *dk;
  float *dg, *dbeta;
};

int simt_rows_per_block(int Dv);
cudaError_t simt_launch(SimtKind kind, const SimtArgs& a, int n_seqs, int in_bf16, int out_bf16, cudaStream_t st);
cudaError_t simt_reduce_parts(const ReduceArgs& a, int out_bf16, cudaStream_t st);
cudaError_t launch_keep_rows(int N, int V, int64_t per_seq, const float* states, const int32_t* keep, float* out,
                             int32_t* status, cudaStream_t st);
cudaError_t launch_chunk_offsets(const int32_t* cu, int N, int64_t* chunk_off, cudaStream_t st);

}  // namespace qbgdn
