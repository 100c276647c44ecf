// RMSNorm forward and backward (warp per row, 16-byte vectors, two-level dw reduction without
// atomics).  Restates python/sejong_kernels/ops/kernels.py:54-87 and the host autotuned pair
// rmsnorm_backward_partial/_reduce (crates/sejong-gpu/src/norm_ops.rs:14-134); the backward is
// fused with the residual-gradient accumulation the tape performs with separate `add` launches
// (crates/sejong-gpu/src/graph.rs:503-513).
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace sj {

constexpr int kNormMaxVec = 4;  // 4 x 8 elements per lane: d <= 1024
constexpr int kNormWarps = 8;
constexpr int kNormRowsPerCta = 32;

template <typename T>
SJ_DEVICE void load8(const T* p, float (&v)[8]);
template <>
SJ_DEVICE void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 w = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
template <>
SJ_DEVICE void load8<float>(const float* p, float (&v)[8]) {
  float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename Y>
SJ_DEVICE void store8(Y* p, const float (&v)[8]);
template <>
SJ_DEVICE void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
SJ_DEVICE void store8_bf16(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 w;
  w.x = pack_bf16x2(v[0], v[1]);
  w.y = pack_bf16x2(v[2], v[3]);
  w.z = pack_bf16x2(v[4], v[5]);
  w.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = w;
}

template <>
SJ_DEVICE void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) { store8_bf16(p, v); }

// Warp per R consecutive rows (R = 4 / VEC, at least 1): the loads of all R rows are issued before
// any reduction, so a warp keeps R rows of x in flight (the narrow local-stage rows of 256 would
// otherwise leave each warp one 1 KB load at a time).
template <typename T, int VEC, typename Y = __nv_bfloat16>
__global__ void rmsnorm_fwd_kernel(const T* x, const float* w, Y* y,
                                   float* inv_rms, int rows, int d, float eps) {
  pdl_wait();
  constexpr int R = VEC >= 4 ? 1 : 4 / VEC;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = warp * R;
  if (row0 >= rows) return;
  float v[R][VEC][8];
#pragma unroll
  for (int q = 0; q < R; ++q) {
    const size_t base = static_cast<size_t>(row0 + q) * d;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int col = (lane + 32 * i) * 8;
      if (row0 + q < rows && col < d) load8<T>(x + base + col, v[q][i]);
    }
  }
  float inv[R];
#pragma unroll
  for (int q = 0; q < R; ++q) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int col = (lane + 32 * i) * 8;
      if (row0 + q < rows && col < d) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += v[q][i][j] * v[q][i][j];
      }
    }
    ss = warp_sum(ss);
    inv[q] = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int col = (lane + 32 * i) * 8;
    if (col < d) {
      float wv[8];
      load8<float>(w + col, wv);
#pragma unroll
      for (int q = 0; q < R; ++q) {
        if (row0 + q < rows) {
          float o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = v[q][i][j] * inv[q] * wv[j];
          store8<Y>(y + static_cast<size_t>(row0 + q) * d + col, o);
        }
      }
    }
  }
  if (inv_rms && lane < R && row0 + lane < rows) {
#pragma unroll
    for (int q = 0; q < R; ++q)
      if (lane == q) inv_rms[row0 + q] = inv[q];
  }
}

// One CTA = kNormWarps warps over kNormRowsPerCta rows; per-CTA dw partial row in `partials`.
template <typename T, int VEC>
__global__ void __launch_bounds__(kNormWarps * 32)
    rmsnorm_bwd_kernel(const T* x, const float* w,
                       const float* inv_rms, const float* dz, float* dres,
                       __nv_bfloat16* dres_bf16, float* partials, int rows, int d, int accumulate) {
  pdl_wait();
  __shared__ float red[kNormWarps][VEC * 256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float dw_acc[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dw_acc[i][j] = 0.f;
  const float inv_d = 1.0f / static_cast<float>(d);
  // R of the warp's rows (r, r + 8, ...) at a time, all their loads issued before any reduction
  constexpr int R = VEC == 1 ? 2 : 1;
  const int end = min(rows, (blockIdx.x + 1) * kNormRowsPerCta);
  float wv[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int col = (lane + 32 * i) * 8;
    if (col < d) load8<float>(w + col, wv[i]);
  }
  for (int r0 = blockIdx.x * kNormRowsPerCta + warp; r0 < end; r0 += kNormWarps * R) {
    float xv[R][VEC][8], gv[R][VEC][8], o[R][VEC][8], inv[R];
#pragma unroll
    for (int q = 0; q < R; ++q) {
      const int r = r0 + q * kNormWarps;
      if (r < end) {
        const size_t base = static_cast<size_t>(r) * d;
        inv[q] = inv_rms[r];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const int col = (lane + 32 * i) * 8;
          if (col < d) {
            load8<T>(x + base + col, xv[q][i]);
            load8<float>(dz + base + col, gv[q][i]);
            if (accumulate) {
              load8<float>(dres + base + col, o[q][i]);
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) o[q][i][j] = 0.f;
            }
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < R; ++q) {
      const int r = r0 + q * kNormWarps;
      if (r >= end) continue;  // warp-uniform
      const size_t base = static_cast<size_t>(r) * d;
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int col = (lane + 32 * i) * 8;
        if (col < d) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float dzv = gv[q][i][j];
            gv[q][i][j] = dzv * wv[i][j];
            dot += gv[q][i][j] * xv[q][i][j];
            dw_acc[i][j] += dzv * xv[q][i][j] * inv[q];
          }
        }
      }
      dot = warp_sum(dot);
      const float coef = dot * inv_d * inv[q] * inv[q];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int col = (lane + 32 * i) * 8;
        if (col < d) {
          float (&oi)[8] = o[q][i];
#pragma unroll
          for (int j = 0; j < 8; ++j) oi[j] += inv[q] * (gv[q][i][j] - xv[q][i][j] * coef);
          float4* dst = reinterpret_cast<float4*>(dres + base + col);
          dst[0] = make_float4(oi[0], oi[1], oi[2], oi[3]);
          dst[1] = make_float4(oi[4], oi[5], oi[6], oi[7]);
          if (dres_bf16) store8_bf16(dres_bf16 + base + col, oi);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int col = (lane + 32 * i) * 8;
    if (col < d)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp][col + j] = dw_acc[i][j];
  }
  __syncthreads();
  for (int col = threadIdx.x; col < d; col += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kNormWarps; ++k) s += red[k][col];
    partials[static_cast<size_t>(blockIdx.x) * d + col] = s;
  }
}

// out[col] += sum over groups of partials[g][col]: 32 columns per CTA, the 32 warps split the
// groups (warp w takes w, w + 32, ...), each with four independent running sums so that four
// coalesced 128-byte row reads are in flight per warp, then one shared-memory reduction.  The
// order of the additions is fixed: the result does not depend on timing.
__global__ void __launch_bounds__(1024) column_reduce_add_kernel(const float* partials, int groups, int d,
                                                                float* out) {
  pdl_wait();
  __shared__ float red[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (col < d) {
    const float* src = partials + col;
    int g = warp;
    for (; g + 96 < groups; g += 128) {
      s0 += src[static_cast<size_t>(g) * d];
      s1 += src[static_cast<size_t>(g + 32) * d];
      s2 += src[static_cast<size_t>(g + 64) * d];
      s3 += src[static_cast<size_t>(g + 96) * d];
    }
    for (; g < groups; g += 32) s0 += src[static_cast<size_t>(g) * d];
  }
  red[warp][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (warp == 0 && col < d) {
    float t = 0.f;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) t += red[k][lane];
    out[col] += t;
  }
}

}  // namespace sj

namespace sj {

template <typename T, int VEC, typename Y = __nv_bfloat16>
static void launch_norm_fwd(const void* x, const float* w, void* y, float* inv, int rows, int d, float eps,
                            cudaStream_t s) {
  constexpr int R = VEC >= 4 ? 1 : 4 / VEC;  // rows per warp, as in the kernel
  const int threads = 256, rows_per_cta = threads / 32 * R;
  launch(rmsnorm_fwd_kernel<T, VEC, Y>, (rows + rows_per_cta - 1) / rows_per_cta, threads, 0, s,
      static_cast<const T*>(x), w, static_cast<Y*>(y), inv, rows, d, eps);
}

template <typename T, int VEC>
static void launch_norm_bwd(const void* x, const float* w, const float* inv, const float* dz, float* dres,
                            void* dres_b, float* partials, int rows, int d, int accumulate, cudaStream_t s) {
  const int groups = (rows + kNormRowsPerCta - 1) / kNormRowsPerCta;
  launch(rmsnorm_bwd_kernel<T, VEC>, groups, kNormWarps * 32, 0, s, static_cast<const T*>(x), w, inv, dz, dres,
         static_cast<__nv_bfloat16*>(dres_b), partials, rows, d, accumulate);
}

template <typename T>
static void dispatch_norm_fwd(const void* x, const float* w, void* y, float* inv, int rows, int d, float eps,
                              cudaStream_t s) {
  switch ((d + 255) / 256) {
    case 1: launch_norm_fwd<T, 1>(x, w, y, inv, rows, d, eps, s); break;
    case 2: launch_norm_fwd<T, 2>(x, w, y, inv, rows, d, eps, s); break;
    case 3: launch_norm_fwd<T, 3>(x, w, y, inv, rows, d, eps, s); break;
    default: launch_norm_fwd<T, 4>(x, w, y, inv, rows, d, eps, s); break;
  }
}

template <typename T>
static void dispatch_norm_bwd(const void* x, const float* w, const float* inv, const float* dz, float* dres,
                              void* dres_b, float* partials, int rows, int d, int accumulate, cudaStream_t s) {
  switch ((d + 255) / 256) {
    case 1: launch_norm_bwd<T, 1>(x, w, inv, dz, dres, dres_b, partials, rows, d, accumulate, s); break;
    case 2: launch_norm_bwd<T, 2>(x, w, inv, dz, dres, dres_b, partials, rows, d, accumulate, s); break;
    case 3: launch_norm_bwd<T, 3>(x, w, inv, dz, dres, dres_b, partials, rows, d, accumulate, s); break;
    default: launch_norm_bwd<T, 4>(x, w, inv, dz, dres, dres_b, partials, rows, d, accumulate, s); break;
  }
}

}  // namespace sj

extern "C" int sj_rmsnorm_fwd(const void* x, int x_dtype, const float* w, void* y, float* inv_rms, int rows, int d,
                              float eps, void* stream) {
  using namespace sj;
  if (rows <= 0 || d <= 0 || d % 8 || d > 32 * 8 * kNormMaxVec)
    return fail(SJ_ERR_SHAPE, "sj_rmsnorm_fwd: d=%d must be a multiple of 8 up to 1024", d);
  if (!aligned16(x) || !aligned16(y) || !aligned16(w))
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_fwd: x/y/w must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == SJ_BF16)
    dispatch_norm_fwd<__nv_bfloat16>(x, w, y, inv_rms, rows, d, eps, s);
  else if (x_dtype == SJ_F32)
    dispatch_norm_fwd<float>(x, w, y, inv_rms, rows, d, eps, s);
  else
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_fwd: x must be bf16 or f32");
  SJ_LAUNCH_CHECK("rmsnorm_fwd");
  return SJ_OK;
}

extern "C" int sj_rmsnorm_fwd_f32(const float* x, const float* w, float* y, float* inv_rms, int rows, int d, float eps,
                                  void* stream) {
  using namespace sj;
  if (rows <= 0 || d <= 0 || d % 8 || d > 32 * 8 * kNormMaxVec)
    return fail(SJ_ERR_SHAPE, "sj_rmsnorm_fwd_f32: d=%d must be a multiple of 8 up to 1024", d);
  if (!aligned16(x) || !aligned16(y) || !aligned16(w))
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_fwd_f32: x/y/w must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  switch ((d + 255) / 256) {
    case 1: launch_norm_fwd<float, 1, float>(x, w, y, inv_rms, rows, d, eps, s); break;
    case 2: launch_norm_fwd<float, 2, float>(x, w, y, inv_rms, rows, d, eps, s); break;
    case 3: launch_norm_fwd<float, 3, float>(x, w, y, inv_rms, rows, d, eps, s); break;
    default: launch_norm_fwd<float, 4, float>(x, w, y, inv_rms, rows, d, eps, s); break;
  }
  SJ_LAUNCH_CHECK("rmsnorm_fwd_f32");
  return SJ_OK;
}

extern "C" size_t sj_rmsnorm_workspace(int rows, int d) {
  if (rows <= 0 || d <= 0) return 0;
  return static_cast<size_t>((rows + sj::kNormRowsPerCta - 1) / sj::kNormRowsPerCta) * static_cast<size_t>(d);
}

extern "C" int sj_rmsnorm_bwd_ex(const void* x, int x_dtype, const float* w, const float* inv_rms, const float* dz,
                                 float* dres, void* dres_bf16, float* dw, float* partials, int rows, int d,
                                 int accumulate, void* stream) {
  using namespace sj;
  if (rows <= 0 || d <= 0 || d % 8 || d > 32 * 8 * kNormMaxVec)
    return fail(SJ_ERR_SHAPE, "sj_rmsnorm_bwd: bad d=%d", d);
  if (!x || !w || !inv_rms || !dz || !dres || !dw || !partials)
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_bwd: null pointer");
  if (!aligned16(x) || !aligned16(dz) || !aligned16(dres) || !aligned16(w) || (dres_bf16 && !aligned16(dres_bf16)))
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_bwd: rows must be 16-byte aligned");
  const int groups = (rows + kNormRowsPerCta - 1) / kNormRowsPerCta;
  cudaStream_t s = as_stream(stream);
  if (x_dtype == SJ_BF16)
    dispatch_norm_bwd<__nv_bfloat16>(x, w, inv_rms, dz, dres, dres_bf16, partials, rows, d, accumulate, s);
  else if (x_dtype == SJ_F32)
    dispatch_norm_bwd<float>(x, w, inv_rms, dz, dres, dres_bf16, partials, rows, d, accumulate, s);
  else
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_bwd: x must be bf16 or f32");
  SJ_LAUNCH_CHECK("rmsnorm_bwd");
  launch(column_reduce_add_kernel, (d + 31) / 32, 1024, 0, s, partials, groups, d, dw);
  SJ_LAUNCH_CHECK("rmsnorm_bwd reduce");
  return SJ_OK;
}

extern "C" int sj_rmsnorm_bwd(const void* x, int x_dtype, const float* w, const float* inv_rms, const float* dz,
                              float* dres, void* dres_bf16, float* dw, float* partials, int rows, int d,
                              void* stream) {
  return sj_rmsnorm_bwd_ex(x, x_dtype, w, inv_rms, dz, dres, dres_bf16, dw, partials, rows, d, 1, stream);
}

// ------------------------------------------------------------------ RMSNorm backward without a workspace
// Some callers cannot hand over device memory for the dw partials: a plugin whose interface
// passes only the tensors of the op, or a process whose device memory is all reserved by
// another allocator so that a cudaMalloc here would fail (and a cudaFree would stall the whole
// device).  sj_rmsnorm_bwd_noalloc keeps the partials in a fixed array that lives in the
// library's own device image instead, so the call itself allocates nothing.
//
// Limit: ceil(rows / 32) * d <= kNoAllocPartials floats (4 MiB per GPU, held by every GPU that
// loads the library until the process exits), e.g. 32768 rows at d = 1024 or 131072 at d = 256.
// Larger shapes are rejected with SJ_ERR_CAPACITY.  The array is shared by all calls on a device,
// so two calls that overlap in time on the same device (two streams, two host threads) race
// on it; serialise them.  Nothing in it has to start at zero: every CTA of the backward kernel
// writes its full partial row before the column reduction reads it.
namespace sj {

constexpr size_t kNoAllocPartials = size_t(1) << 20;
static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartials];

// Device address of g_noalloc_partials in the current context.  In host code the array's name is
// only a host-side stand-in, so the address is asked of the runtime; it is asked on every call
// rather than cached, because it belongs to one CUDA context (a cudaDeviceReset or another context
// made current on the device would leave a cached value pointing at nothing).  The first call in
// a context loads the library's device image there if it is not loaded yet, so that first call
// should come before any stream capture on the device.
static int noalloc_partials(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
  if (e != cudaSuccess) return cuda_check(e, "sj_rmsnorm_bwd_noalloc: cudaGetSymbolAddress");
  if (!p) return fail(SJ_ERR_CUDA, "sj_rmsnorm_bwd_noalloc: null scratch address");
  *out = static_cast<float*>(p);
  return SJ_OK;
}

}  // namespace sj

extern "C" size_t sj_rmsnorm_noalloc_limit(void) { return sj::kNoAllocPartials; }

extern "C" int sj_rmsnorm_bwd_noalloc(const void* x, int x_dtype, const float* w, const float* inv_rms,
                                      const float* dz, float* dres, void* dres_bf16, float* dw, int rows, int d,
                                      void* stream) {
  using namespace sj;
  if (rows <= 0 || d <= 0 || d % 8 || d > 32 * 8 * kNormMaxVec)
    return fail(SJ_ERR_SHAPE, "sj_rmsnorm_bwd_noalloc: bad d=%d", d);
  const size_t need = sj_rmsnorm_workspace(rows, d);
  if (need > kNoAllocPartials)
    return fail(SJ_ERR_CAPACITY,
                "sj_rmsnorm_bwd_noalloc: rows=%d d=%d needs %zu partial floats, above the static limit of %zu",
                rows, d, need, kNoAllocPartials);
  if (!x || !w || !inv_rms || !dz || !dres || !dw)
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_bwd_noalloc: null pointer");
  if (!aligned16(x) || !aligned16(dz) || !aligned16(dres) || !aligned16(w) || (dres_bf16 && !aligned16(dres_bf16)))
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_bwd_noalloc: rows must be 16-byte aligned");
  if (x_dtype != SJ_BF16 && x_dtype != SJ_F32)
    return fail(SJ_ERR_ARGUMENT, "sj_rmsnorm_bwd_noalloc: x must be bf16 or f32");
  float* partials = nullptr;
  const int status = noalloc_partials(&partials);
  if (status != SJ_OK) return status;
  const int groups = (rows + kNormRowsPerCta - 1) / kNormRowsPerCta;
  cudaStream_t s = as_stream(stream);
  if (x_dtype == SJ_BF16)
    dispatch_norm_bwd<__nv_bfloat16>(x, w, inv_rms, dz, dres, dres_bf16, partials, rows, d, 1, s);
  else
    dispatch_norm_bwd<float>(x, w, inv_rms, dz, dres, dres_bf16, partials, rows, d, 1, s);
  SJ_LAUNCH_CHECK("rmsnorm_bwd_noalloc");
  launch(column_reduce_add_kernel, (d + 31) / 32, 1024, 0, s, partials, groups, d, dw);
  SJ_LAUNCH_CHECK("rmsnorm_bwd_noalloc reduce");
  return SJ_OK;
}
