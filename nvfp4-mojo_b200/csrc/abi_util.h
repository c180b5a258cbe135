// abi_util.h -- error reporting helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace nvfp4 {

// Records a printf-style message as the thread's last error; returns `code`.
int fail(int code, const char *fmt, ...);
// NVFP4_OK, or NVFP4_ERR_CUDA with the CUDA error text recorded.
int check_launch(cudaError_t e, const char *what);
bool aligned(const void *p, size_t a);

}  // namespace nvfp4
