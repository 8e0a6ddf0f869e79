// spmm24_host.h -- host-side helpers shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>

namespace spmm24 {
// Records `why` as the calling thread's spmm24_last_error() and returns
// cudaErrorInvalidValue.
cudaError_t record_invalid(const char* why);
// Clears the calling thread's spmm24_last_error().
void clear_last_error();
}  // namespace spmm24
