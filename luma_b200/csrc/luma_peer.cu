// luma_peer.cu — peer-memory plumbing of the copy-engine all-gather.
//
// The ZeRO-1 step ends with every rank holding the full updated params.  With
// NCCL's all-gather the transfer runs in NCCL kernels that occupy SMs the
// (instruction-bound) step kernels need.  The copy-engine path instead maps
// every peer's flat param buffer into this process (CUDA IPC) and pushes this
// rank's updated pieces into each peer with one cudaMemcpyAsync per (bucket,
// peer): the copy engines move the bytes over NVLink and the SMs stay with the
// step.  Ordering across ranks is the caller's (luma_b200/zero.py: a
// stream-ordered barrier before the first push and after the last).
//
// No counterpart in the reference, whose optimizer never exchanges data (its
// FSDP integration leaves the gather to FSDP, optimizer.py:399-407).

#include "luma_b200.h"
#include "luma_internal.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

static_assert(sizeof(LumaIpcHandle) == sizeof(cudaIpcMemHandle_t), "LumaIpcHandle layout");

namespace {

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange from the driver, found through the runtime (the
// library does not link libcuda).
GetAddressRangeFn address_range_fn() {
  static std::once_flag once;
  static GetAddressRangeFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  });
  return fn;
}

// Grid-stride copy of 16-byte units into a multicast mapping (multimem.st of
// four 32-bit words: the NVSwitch writes them to every bound GPU).
__global__ void __launch_bounds__(512) luma_mc_copy_kernel(uint4* __restrict__ dst,
                                                           const uint4* __restrict__ src,
                                                           uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * 512 + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * 512) {
    const uint4 v = __ldcs(src + i);
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + i),
                 "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
                 "f"(__uint_as_float(v.w))
                 : "memory");
  }
  __threadfence_system();
}

}  // namespace

extern "C" {

int luma_ipc_export(const void* ptr, LumaIpcHandle* handle, uint64_t* offset) {
  luma_g_err[0] = '\0';
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return luma_fail(LUMA_ERR_INVALID, "luma_ipc_export: NULL pointer");
  GetAddressRangeFn range = address_range_fn();
  if (range == nullptr)
    return luma_fail(LUMA_ERR_CUDA, "luma_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS)
    return luma_fail(LUMA_ERR_CUDA, "luma_ipc_export: cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return luma_cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle->bytes, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return LUMA_OK;
}

int luma_ipc_open(const LumaIpcHandle* handle, void** base) {
  luma_g_err[0] = '\0';
  if (handle == nullptr || base == nullptr)
    return luma_fail(LUMA_ERR_INVALID, "luma_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return luma_cuda_fail(e, "cudaIpcOpenMemHandle");
  return LUMA_OK;
}

int luma_ipc_close(void* base) {
  luma_g_err[0] = '\0';
  if (base == nullptr) return luma_fail(LUMA_ERR_INVALID, "luma_ipc_close: NULL pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return luma_cuda_fail(e, "cudaIpcCloseMemHandle");
  return LUMA_OK;
}

int luma_copy_async(void* dst, const void* src, uint64_t bytes, void* stream) {
  luma_g_err[0] = '\0';
  if (bytes == 0) return LUMA_OK;
  if (dst == nullptr || src == nullptr)
    return luma_fail(LUMA_ERR_INVALID, "luma_copy_async: NULL pointer");
  const cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return luma_cuda_fail(e, "cudaMemcpyAsync");
  return LUMA_OK;
}

int luma_mc_copy(void* mc_dst, const void* src, uint64_t bytes, void* stream) {
  luma_g_err[0] = '\0';
  if (bytes == 0) return LUMA_OK;
  if (mc_dst == nullptr || src == nullptr)
    return luma_fail(LUMA_ERR_INVALID, "luma_mc_copy: NULL pointer");
  if (((uintptr_t)mc_dst | (uintptr_t)src | bytes) % 16 != 0)
    return luma_fail(LUMA_ERR_INVALID, "luma_mc_copy: addresses and size must be multiples of 16");
  const uint64_t n = bytes / 16;
  const uint64_t want = (n + 511) / 512;
  // a few CTAs suffice: the copy is bound by the NVLink links, not the SMs
  const int blocks = (int)(want < 64 ? want : 64);
  luma_mc_copy_kernel<<<blocks, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(mc_dst), static_cast<const uint4*>(src), n);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return luma_cuda_fail(e, "launch luma_mc_copy");
  return LUMA_OK;
}

}  // extern "C"
