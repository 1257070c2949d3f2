// Host-visible interface of the tensor-core chunked path (Dk = Dv = 128).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace qbgdn {

// g == nullptr selects layer mode: q, k are the raw (pre-norm) rows and the gates come from
// a, b, A_log, dt_bias (the norm and gate graph of src/deltanet.cpp:94-100 fused into the kernels).
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
  const float *a_raw, *b_raw, *A_log, *dt_bias;
  // non-null: recompute mode -- given these chunk-start states [chunks, Hv, Dv, Dk], fill saved (without
  // its checkpoint part) chunk by chunk in parallel; y is not written (hT must be null)
  const float* ckpt_in;
};

// Layer mode as above: dg, dbeta then receive da, db, and dA_log, ddt_bias the head sums.
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
  const float *a_raw, *b_raw, *A_log, *dt_bias;
  float *dA_log, *ddt_bias;
  // with saved null: the caller's chunk-start states [chunks, Hv, Dv, Dk] (the rest is recomputed from
  // them chunk by chunk), or null to recompute everything with the forward walk
  const float* ckpt_in;
};

bool chunked_supported(int Dk, int Dv);
// Whether the backward has its own chunked kernels; until then a chunked forward's saved buffer starts
// with the row-parallel backward's chunk-start states and that backward runs.
bool chunked_bwd_ready();
// layer: the saved buffer / workspace of the layer-mode path (adds the normalised q, k rows)
int64_t chunked_saved_bytes(int Hv, int Hk, int64_t n_chunks, int64_t tokens, bool layer);
int64_t chunked_ws_bytes(int Hv, int Hk, int N, int64_t n_chunks, int64_t tokens, bool varlen, int op, bool with_saved,
                         bool layer, bool ckpt_external = false);
// Both report into a status block the caller has initialised (init_status): chunked_fwd into
// `status` (the one opening ws, or a recomputing backward's own), chunked_bwd into the one opening ws.
cudaError_t chunked_fwd(const ChunkFwdArgs& a, void* ws, cudaStream_t st, int* status);
cudaError_t chunked_bwd(const ChunkBwdArgs& a, void* ws, cudaStream_t st);

}  // namespace qbgdn
