// Host-side helpers shared by the C-ABI translation units (not part of the ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "sejong.h"

namespace sj {

// Record a thread-local error message and return the code.
int fail(int code, const char* fmt, ...);
// Map a CUDA runtime status to SJ_OK / SJ_ERR_CUDA with a message naming `what`.
int cuda_check(cudaError_t e, const char* what);
// Number of SMs of the current device (cached per device).
int sm_count();
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// 2-D bf16 TMA map with 128-byte swizzle: `inner` contiguous elements per row, `outer` rows, row
// stride `ld` elements, box box_inner x box_outer (gemm.cu).
int bf16_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
             uint32_t box_outer);
// TMA map of any rank (gemm.cu): dims[0] contiguous elements, strides_bytes[i] the byte stride of
// dimension i + 1, box[i] elements per copy along dimension i.
int tensor_map(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Per-device record of a kernel whose dynamic shared-memory limit has been raised.  Each call site
// owns one (a function-local static); the flags are atomics, so host threads that drive different
// devices do not race, and two threads that set the same device both just set the attribute
// (cudaFuncSetAttribute is idempotent).
struct KernelAttrOnce {
  static constexpr int kMaxDevices = 64;
  std::atomic<unsigned char> done[kMaxDevices] = {};
};
// Raise `kernel`'s dynamic shared-memory limit to `bytes` on the current device, once per device.
inline int ensure_max_smem(KernelAttrOnce& once, const void* kernel, int bytes, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_check(e, what);
  const bool tracked = dev >= 0 && dev < KernelAttrOnce::kMaxDevices;
  if (tracked && once.done[dev].load(std::memory_order_acquire)) return SJ_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_check(e, what);
  if (tracked) once.done[dev].store(1, std::memory_order_release);
  return SJ_OK;
}

// Zero `bytes` bytes at `ptr` on `stream` with a kernel (elementwise.cu).
int zero_async(void* ptr, size_t bytes, cudaStream_t stream);

// Whether kernels are launched with programmatic stream serialization (default on; SJ_PDL=0 in the
// environment turns it off, read once per process).
bool pdl_enabled();

// kernel<<<grid, block, smem, stream>>>(args...) with programmatic stream serialization: the kernel
// may begin while the previous kernel of the stream finishes, and waits for it (pdl_wait) before
// touching global memory.  Errors are left for SJ_LAUNCH_CHECK (cudaGetLastError).
template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // arguments converted to the parameter types, as <<<...>>> would (const parameters included)
  [&](KArgs... coerced) {
    void* pargs[] = {const_cast<void*>(static_cast<const void*>(&coerced))...};
    cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), pargs);
  }(std::forward<Args>(args)...);
}

}  // namespace sj

#define SJ_LAUNCH_CHECK(what)                                     \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return ::sj::cuda_check(_e, what);     \
  } while (0)
