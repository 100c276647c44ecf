// Host-side helpers shared by the C-ABI translation units (not part of the ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <string>

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

}  // namespace sj

#define SJ_LAUNCH_CHECK(what)                                     \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return ::sj::cuda_check(_e, what);     \
  } while (0)
