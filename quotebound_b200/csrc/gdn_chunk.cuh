// Host-visible interface of the tensor-core chunked path (Dk = Dv = 128).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace qbgdn {

struct ChunkFwdArgs {
  int B, T, Hk, Hv, Dk, Dv, N;
  int64_t n_chunks;
  const int32_t* cu;
  const void *q, *k, *v;
  const float *g, *beta, *h0;
  void* y;
  float* hT;
  void* saved;
  int in_bf16, out_bf16;
};

struct ChunkBwdArgs {
  int B, T, Hk, Hv, Dk, Dv, N;
  int64_t n_chunks;
  const int32_t* cu;
  const void *q, *k, *v, *dy;
  const float *g, *beta, *h0, *dhT;
  const void* saved;
  void *dq, *dk, *dv;
  float *dg, *dbeta, *dh0;
  int in_bf16, out_bf16;
};

bool chunked_supported(int Dk, int Dv);
// Whether the backward has its own chunked kernels; until then a chunked forward's saved buffer starts
// with the row-parallel backward's chunk-start states and that backward runs.
bool chunked_bwd_ready();
int64_t chunked_saved_bytes(int Hv, int Dk, int Dv, int64_t n_chunks, int64_t tokens);
int64_t chunked_ws_bytes(int Hv, int Hk, int Dk, int Dv, int N, int64_t n_chunks, int64_t tokens, bool varlen, int op,
                         bool with_saved);
cudaError_t chunked_fwd(const ChunkFwdArgs& a, void* ws, cudaStream_t st);
cudaError_t chunked_bwd(const ChunkBwdArgs& a, void* ws, cudaStream_t st);

}  // namespace qbgdn
