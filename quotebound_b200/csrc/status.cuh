// The status block: the first kStatusBytes of every workspace that qb_gdn_fwd, qb_gdn_bwd,
// qb_gdn_layer_fwd and qb_gdn_layer_bwd take.  Each call initialises it on its stream before its first
// kernel; the kernels' bounded waits report into it (tc::mbar_wait); qb_gdn_status reads word 0.
//   word 0  status code: 0, or the code of the first bounded wait that gave up (the table in
//           include/qb_gdn.h); the outputs of that call are then not valid
//   word 2  the gradient kernel's count of finished CTAs (layer mode)
//   word 4  test hook: the code of the one wait that gives up early (0 = none)
//   word 5  test hook: after how many polls it gives up
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace qbgdn {

constexpr int kStatusBytes = 256;  // 256 keeps every buffer carved after it 256-byte aligned

// Clears the block on `st` and writes the process-wide test hook (set_test_wait_limit) into it.
cudaError_t init_status(int* status, cudaStream_t st);
// Test hook for the failure path: the wait with this code gives up after `polls` polls in every call
// that follows (code 0 turns it off).
void set_test_wait_limit(int code, uint32_t polls);

}  // namespace qbgdn
