// Host-visible interface of the row-parallel (SIMT) kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace qbgdn {

enum class SimtKind { Fwd, Step, Verify };

// One struct for every row-parallel kernel; unused fields are null / zero.
struct SimtArgs {
  int T, Hk, Hv, Dk, Dv;
  int rows_per_block;          // warps per block
  const int32_t* cu;           // device offsets [N + 1] or null
  const int64_t* chunk_off;    // device, [N + 1] chunk offsets (varlen) or null
  const void *q, *k, *v;       // activation dtype
  const float *g, *beta;
  const float* h0;             // [N, Hv, Dv, Dk] or null (step/verify: h0 = state_in)
  void* y;                     // output dtype
  float* hT;                   // step: hT = state_out
  float* ckpt;                 // fwd: chunk starts out (or null); verify: states out
};

int simt_rows_per_block(int Dv);
cudaError_t simt_launch(SimtKind kind, const SimtArgs& a, int n_seqs, int in_bf16, int out_bf16, cudaStream_t st);
cudaError_t launch_keep_rows(int N, int V, int64_t per_seq, const float* states, const int32_t* keep, float* out,
                             int32_t* status, cudaStream_t st);
cudaError_t launch_chunk_offsets(const int32_t* cu, int N, int64_t* chunk_off, cudaStream_t st);

}  // namespace qbgdn
