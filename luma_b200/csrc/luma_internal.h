// luma_internal.h — declarations shared by the library's translation units
// (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>

#define LUMA_HIDDEN __attribute__((visibility("hidden")))

// Message of the last failed C-ABI call on this thread (luma_last_error).
LUMA_HIDDEN extern thread_local char luma_g_err[512];

// Record a formatted message and return `code`.
LUMA_HIDDEN int luma_fail(int code, const char* fmt, ...);

// Record "<what>: <CUDA error string>" and return LUMA_ERR_CUDA.
LUMA_HIDDEN int luma_cuda_fail(cudaError_t e, const char* what);
