// Tensor-core chunked path: not built yet, so no shape selects it.
#include "gdn_chunk.cuh"

namespace qbgdn {
bool chunked_supported(int, int) { return false; }
int64_t chunked_saved_bytes(int, int, int, int64_t, int64_t) { return 0; }
int64_t chunked_ws_bytes(int, int, int, int, int, int64_t, int64_t, bool, int, bool) { return 0; }
cudaError_t chunked_fwd(const ChunkFwdArgs&, void*, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t chunked_bwd(const ChunkBwdArgs&, void*, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace qbgdn
