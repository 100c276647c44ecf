// Bandwidth-bound kernels of the step: embedding gather / scatter, RoPE, SwiGLU backward,
// hierarchy patch pooling and broadcast, casts and adds.  All use 16-byte vector accesses along
// the contiguous feature dimension.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {

// ---------------------------------------------------------------- zero fill
// Bytes [0, head) and the `tail` bytes after the 16-byte-aligned middle are written one by one, the
// n16 vectors of the middle with 16-byte stores.  Used instead of a memset node so that every
// operation of the library on a stream is a kernel that orders itself with pdl_wait.
__global__ void zero_kernel(uint8_t* p, size_t head, size_t n16, size_t tail) {
  pdl_wait();
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  if (tid < head) p[tid] = 0;
  uint4* v = reinterpret_cast<uint4*>(p + head);
  for (size_t i = tid; i < n16; i += stride) v[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid < tail) p[head + 16 * n16 + tid] = 0;
}

int zero_async(void* ptr, size_t bytes, cudaStream_t stream) {
  if (bytes == 0) return SJ_OK;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(ptr);
  const size_t head = std::min(bytes, static_cast<size_t>((16 - (addr & 15u)) & 15u));
  const size_t n16 = (bytes - head) / 16;
  const size_t tail = bytes - head - 16 * n16;
  const size_t blocks = std::min<size_t>((n16 + 255) / 256 + 1, static_cast<size_t>(sm_count()) * 8);
  launch(zero_kernel, static_cast<unsigned>(blocks), 256, 0, stream, static_cast<uint8_t*>(ptr), head, n16, tail);
  SJ_LAUNCH_CHECK("zero");
  return SJ_OK;
}

// ---------------------------------------------------------------- embedding (kernels.py:41-52)
// One thread per 8 columns (one 16-byte bf16 vector of the weight row).
template <bool F32_OUT>
__global__ void embedding_fwd_kernel(const uint4* w, const int32_t* ids, void* y,
                                     int n, int vec_per_row, int vocab) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(n) * vec_per_row) return;
  const int row = static_cast<int>(i / vec_per_row), c = static_cast<int>(i % vec_per_row);
  const int id = ids[row];
  uint4 v = make_uint4(0, 0, 0, 0);
  if (id >= 0 && id < vocab)
    v = w[static_cast<size_t>(id) * vec_per_row + c];
  else if (c == 0)
    record_error(SJ_DEV_BAD_INDEX);
  if (!F32_OUT) {
    reinterpret_cast<uint4*>(y)[i] = v;
  } else {
    const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), cc = unpack_bf16x2(v.z), d = unpack_bf16x2(v.w);
    float4* o = reinterpret_cast<float4*>(y) + 2 * i;
    o[0] = make_float4(a.x, a.y, b.x, b.y);
    o[1] = make_float4(cc.x, cc.y, d.x, d.y);
  }
}

// Row-chunk x 32-column slices accumulated in shared memory, flushed with one atomic per
// (vocab row, column) per CTA; avoids per-element global atomics on frequent bytes.
constexpr int kEmbRows = 1024;
constexpr int kEmbBatch = 8;  // rows whose loads a warp issues before its shared-memory adds
__global__ void __launch_bounds__(256)
    embedding_bwd_kernel(const float* dy, const int32_t* ids, float* dw, int n,
                         int d, int vocab) {
  pdl_wait();
  extern __shared__ float acc[];  // [vocab][32]
  const int col = blockIdx.y * 32 + (threadIdx.x & 31);
  for (int i = threadIdx.x; i < vocab * 32; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();
  const int r0 = blockIdx.x * kEmbRows, r1 = min(n, r0 + kEmbRows);
  const int warps = blockDim.x >> 5;
  if (col < d) {
    for (int rb = r0 + (threadIdx.x >> 5); rb < r1; rb += warps * kEmbBatch) {
      int id[kEmbBatch];
      float g[kEmbBatch];
#pragma unroll
      for (int q = 0; q < kEmbBatch; ++q) {
        const int r = rb + q * warps;
        id[q] = r < r1 ? ids[r] : -1;
        g[q] = r < r1 ? dy[static_cast<size_t>(r) * d + col] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < kEmbBatch; ++q)
        if (id[q] >= 0 && id[q] < vocab) atomicAdd(&acc[id[q] * 32 + (threadIdx.x & 31)], g[q]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < vocab * 32; i += blockDim.x) {
    const int v = i >> 5, c = blockIdx.y * 32 + (i & 31);
    if (c < d && acc[i] != 0.f) atomicAdd(&dw[static_cast<size_t>(v) * d + c], acc[i]);
  }
}

// ---------------------------------------------------------------- RoPE (kernels.py:103-113)
__global__ void rope_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int rows, int heads,
                            int hd, int t, int offset, float log_theta, float sign) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t pairs_per_row = static_cast<size_t>(heads) * (hd / 2);
  if (i >= static_cast<size_t>(rows) * pairs_per_row) return;
  const int row = static_cast<int>(i / pairs_per_row);
  const int pair = static_cast<int>(i % (hd / 2));
  const float pos = static_cast<float>(row % t + offset);
  const float angle = pos * expf((-2.0f * static_cast<float>(pair) / static_cast<float>(hd)) * log_theta);
  float s, c;
  sincosf(angle, &s, &c);
  s *= sign;
  const size_t base = 2 * i;
  const float a = bf2f(x[base]), b = bf2f(x[base + 1]);
  y[base] = f2bf(a * c - b * s);
  y[base + 1] = f2bf(a * s + b * c);
}

__global__ void rope_table_kernel(float2* table, int t, int half, int offset, float log_theta,
                                  float hd) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= t * half) return;
  const int pos = i / half, pair = i % half;
  const float angle = static_cast<float>(pos + offset) * expf((-2.0f * static_cast<float>(pair) / hd) * log_theta);
  float s, c;
  sincosf(angle, &s, &c);
  table[i] = make_float2(c, s);
}

// ---------------------------------------------------------------- SwiGLU backward (kernels.py:95-101)
// gu: per row, blocks of 32 columns = 16 gate features then the same 16 up features.
// `live` (optional, device): the number of leading rows that hold data (a packed MoE buffer
// whose used extent is known only on the device); the grid strides over them.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* gu, const __nv_bfloat16* dh,
                                  __nv_bfloat16* dgu, int rows, int f, const int32_t* live) {
  pdl_wait();
  const int groups = f / 8;
  if (live != nullptr) rows = min(rows, *live);
  const size_t n = static_cast<size_t>(rows) * groups;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;  // one per 8 features
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
  const int row = static_cast<int>(i / groups);
  const int f0 = static_cast<int>(i % groups) * 8;
  const int gcol = (f0 / 16) * 32 + (f0 % 16);
  const size_t rb = static_cast<size_t>(row) * 2 * f;
  const uint4 gw = *reinterpret_cast<const uint4*>(gu + rb + gcol);
  const uint4 uw = *reinterpret_cast<const uint4*>(gu + rb + gcol + 16);
  const uint4 hw = *reinterpret_cast<const uint4*>(dh + static_cast<size_t>(row) * f + f0);
  const uint32_t ga[4] = {gw.x, gw.y, gw.z, gw.w}, ua[4] = {uw.x, uw.y, uw.z, uw.w}, ha[4] = {hw.x, hw.y, hw.z, hw.w};
  uint32_t dg[4], du[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 g = unpack_bf16x2(ga[j]), u = unpack_bf16x2(ua[j]), dy = unpack_bf16x2(ha[j]);
    const float s0 = 1.0f / (1.0f + __expf(-g.x)), s1 = 1.0f / (1.0f + __expf(-g.y));
    dg[j] = pack_bf16x2(dy.x * u.x * s0 * (1.0f + g.x * (1.0f - s0)), dy.y * u.y * s1 * (1.0f + g.y * (1.0f - s1)));
    du[j] = pack_bf16x2(dy.x * g.x * s0, dy.y * g.y * s1);
  }
  *reinterpret_cast<uint4*>(dgu + rb + gcol) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
  *reinterpret_cast<uint4*>(dgu + rb + gcol + 16) = make_uint4(du[0], du[1], du[2], du[3]);
  }
}

// ---------------------------------------------------------------- hierarchy (hierarchy.py:107-172)
__global__ void patch_pool_fwd_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int batch,
                                      int t, int d, int patch) {
  pdl_wait();
  const int patches = (t + patch - 1) / patch;
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // one per 8 columns
  const int vec = d / 8;
  if (i >= static_cast<size_t>(batch) * patches * vec) return;
  const int prow = static_cast<int>(i / vec), c = static_cast<int>(i % vec) * 8;
  const int b = prow / patches, p = prow % patches;
  const int start = p * patch, count = min(patch, t - start);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int k = 0; k < count; ++k) {
    const uint4 w = *reinterpret_cast<const uint4*>(x + (static_cast<size_t>(b) * t + start + k) * d + c);
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f2 = unpack_bf16x2(a[j]);
      acc[2 * j] += f2.x;
      acc[2 * j + 1] += f2.y;
    }
  }
  const float inv = 1.0f / static_cast<float>(count);
  uint4 o;
  o.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  o.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
  o.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
  *reinterpret_cast<uint4*>(y + static_cast<size_t>(prow) * d + c) = o;
}

__global__ void patch_pool_bwd_kernel(const float* dy, float* dx, int batch, int t, int d,
                                      int patch) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // one per 4 columns
  const int vec = d / 4;
  if (i >= static_cast<size_t>(batch) * t * vec) return;
  const int row = static_cast<int>(i / vec), c = static_cast<int>(i % vec) * 4;
  const int b = row / t, pos = row % t, p = pos / patch;
  const int patches = (t + patch - 1) / patch;
  const float inv = 1.0f / static_cast<float>(min(patch, t - p * patch));
  const float4 g = *reinterpret_cast<const float4*>(dy + (static_cast<size_t>(b) * patches + p) * d + c);
  float4* o = reinterpret_cast<float4*>(dx + static_cast<size_t>(row) * d + c);
  float4 v = *o;
  v.x += g.x * inv;
  v.y += g.y * inv;
  v.z += g.z * inv;
  v.w += g.w * inv;
  *o = v;
}

template <bool F32_OUT>
__global__ void patch_broadcast_fwd_kernel(const __nv_bfloat16* z, const __nv_bfloat16* bos,
                                           void* yv, int add, int batch, int t, int d, int patch) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // one per 8 columns
  const int vec = d / 8;
  if (i >= static_cast<size_t>(batch) * t * vec) return;
  const int row = static_cast<int>(i / vec), c = static_cast<int>(i % vec) * 8;
  const int b = row / t, pos = row % t, p = pos / patch - 1;
  const int patches = (t + patch - 1) / patch;
  const __nv_bfloat16* src = p >= 0 ? z + (static_cast<size_t>(b) * patches + p) * d + c : bos + c;
  const uint4 sw = *reinterpret_cast<const uint4*>(src);
  if (F32_OUT) {
    const float2 a = unpack_bf16x2(sw.x), bb = unpack_bf16x2(sw.y), cc = unpack_bf16x2(sw.z), dd = unpack_bf16x2(sw.w);
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(yv) + static_cast<size_t>(row) * d + c);
    float4 o0 = make_float4(a.x, a.y, bb.x, bb.y), o1 = make_float4(cc.x, cc.y, dd.x, dd.y);
    if (add) {
      const float4 y0 = o[0], y1 = o[1];
      o0.x += y0.x; o0.y += y0.y; o0.z += y0.z; o0.w += y0.w;
      o1.x += y1.x; o1.y += y1.y; o1.z += y1.z; o1.w += y1.w;
    }
    o[0] = o0;
    o[1] = o1;
    return;
  }
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(yv);
  uint4* dst = reinterpret_cast<uint4*>(y + static_cast<size_t>(row) * d + c);
  if (!add) {
    *dst = sw;
    return;
  }
  const uint4 yw = *dst;
  const uint32_t sa[4] = {sw.x, sw.y, sw.z, sw.w}, ya[4] = {yw.x, yw.y, yw.z, yw.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 a = unpack_bf16x2(ya[j]), s = unpack_bf16x2(sa[j]);
    o[j] = pack_bf16x2(a.x + s.x, a.y + s.y);
  }
  *dst = make_uint4(o[0], o[1], o[2], o[3]);
}

// dz[b,p,:] = sum_{k<P} dy[b, (p+1)P + k, :]  (bf16 out); blocks past the body reduce dbos.
__global__ void patch_broadcast_bwd_kernel(const float* dy, __nv_bfloat16* dz,
                                           __nv_bfloat16* dbos, int batch, int t, int d, int patch,
                                           int body_threads) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int patches = (t + patch - 1) / patch;
  if (i < body_threads) {
    const int prow = i / d, c = i % d;
    const int b = prow / patches, p = prow % patches;
    float s = 0.f;
    for (int k = 0; k < patch; ++k) {
      const int pos = (p + 1) * patch + k;
      if (pos < t) s += dy[(static_cast<size_t>(b) * t + pos) * d + c];
    }
    dz[static_cast<size_t>(prow) * d + c] = f2bf(s);
    return;
  }
  const int c = i - body_threads;
  if (c >= d) return;
  float s = 0.f;
  for (int b = 0; b < batch; ++b)
    for (int k = 0; k < min(patch, t); ++k) s += dy[(static_cast<size_t>(b) * t + k) * d + c];
  dbos[c] = f2bf(s);
}

// ---------------------------------------------------------------- cast / add
template <typename S, typename D>
__global__ void cast_kernel(const S* x, D* y, size_t n);
template <>
__global__ void cast_kernel<float, __nv_bfloat16>(const float* x, __nv_bfloat16* y, size_t n) {
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = f2bf(x[i]);
}
template <>
__global__ void cast_kernel<__nv_bfloat16, float>(const __nv_bfloat16* x, float* y, size_t n) {
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = bf2f(x[i]);
}
template <>
__global__ void cast_kernel<float, double>(const float* x, double* y, size_t n) {
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = static_cast<double>(x[i]);
}
template <>
__global__ void cast_kernel<double, float>(const double* x, float* y, size_t n) {
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = static_cast<float>(x[i]);
}

template <typename T>
__global__ void add_kernel(const T* x, const T* z, T* y, size_t n, float alpha) {
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if constexpr (sizeof(T) == 2)
      y[i] = f2bf(bf2f(x[i]) + alpha * bf2f(z[i]));
    else
      y[i] = x[i] + alpha * z[i];
  }
}

static int grid_for(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  const size_t cap = static_cast<size_t>(sm_count()) * 32;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace sj

using namespace sj;

extern "C" int sj_embedding_fwd(const void* w, const int32_t* ids, void* y, int y_dtype, int n, int d, int vocab,
                                void* stream) {
  if (n <= 0 || d <= 0 || d % 8 || vocab <= 0)
    return fail(SJ_ERR_SHAPE, "sj_embedding_fwd: d=%d must be a multiple of 8", d);
  if (!aligned16(w) || !aligned16(y)) return fail(SJ_ERR_ARGUMENT, "sj_embedding_fwd: 16-byte alignment required");
  const int vpr = d / 8;
  const size_t total = static_cast<size_t>(n) * vpr;
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  if (y_dtype == SJ_BF16)
    launch(embedding_fwd_kernel<false>, grid, 256, 0, as_stream(stream), static_cast<const uint4*>(w), ids, y, n, vpr, vocab);
  else if (y_dtype == SJ_F32)
    launch(embedding_fwd_kernel<true>, grid, 256, 0, as_stream(stream), static_cast<const uint4*>(w), ids, y, n, vpr, vocab);
  else
    return fail(SJ_ERR_ARGUMENT, "sj_embedding_fwd: y must be bf16 or f32");
  SJ_LAUNCH_CHECK("embedding_fwd");
  return SJ_OK;
}

// f32 table and output: the same 16-byte row gather, four floats per vector.
extern "C" int sj_embedding_fwd_f32(const float* w, const int32_t* ids, float* y, int n, int d, int vocab,
                                    void* stream) {
  if (n <= 0 || d <= 0 || d % 4 || vocab <= 0)
    return fail(SJ_ERR_SHAPE, "sj_embedding_fwd_f32: d=%d must be a multiple of 4", d);
  if (!aligned16(w) || !aligned16(y) || !ids)
    return fail(SJ_ERR_ARGUMENT, "sj_embedding_fwd_f32: 16-byte alignment required");
  const int vpr = d / 4;
  const size_t total = static_cast<size_t>(n) * vpr;
  launch(embedding_fwd_kernel<false>, static_cast<unsigned>((total + 255) / 256), 256, 0, as_stream(stream),
         reinterpret_cast<const uint4*>(w), ids, static_cast<void*>(y), n, vpr, vocab);
  SJ_LAUNCH_CHECK("embedding_fwd_f32");
  return SJ_OK;
}

extern "C" int sj_embedding_bwd(const float* dy, const int32_t* ids, float* dw, int n, int d, int vocab, void* stream) {
  if (n <= 0 || d <= 0 || vocab <= 0 || vocab > 1024) return fail(SJ_ERR_SHAPE, "sj_embedding_bwd: bad shape");
  dim3 grid((n + kEmbRows - 1) / kEmbRows, (d + 31) / 32);
  const size_t smem = static_cast<size_t>(vocab) * 32 * sizeof(float);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(embedding_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  }
  launch(embedding_bwd_kernel, grid, 256, smem, as_stream(stream), dy, ids, dw, n, d, vocab);
  SJ_LAUNCH_CHECK("embedding_bwd");
  return SJ_OK;
}

extern "C" int sj_rope(const void* x, void* y, int rows, int heads, int head_dim, int t, int offset, float theta,
                       int inverse, void* stream) {
  if (rows <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 2 || t <= 0)
    return fail(SJ_ERR_SHAPE, "sj_rope: bad shape");
  const size_t pairs = static_cast<size_t>(rows) * heads * (head_dim / 2);
  launch(rope_kernel, static_cast<unsigned>((pairs + 255) / 256), 256, 0, as_stream(stream), 
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), rows, heads, head_dim, t, offset,
      logf(theta), inverse ? -1.0f : 1.0f);
  SJ_LAUNCH_CHECK("rope");
  return SJ_OK;
}

extern "C" int sj_rope_table(float* table, int t, int head_dim, int offset, float theta, void* stream) {
  if (!table || t <= 0 || head_dim <= 0 || head_dim % 2 || theta <= 0.f)
    return fail(SJ_ERR_ARGUMENT, "sj_rope_table: bad arguments");
  if (reinterpret_cast<uintptr_t>(table) & 7) return fail(SJ_ERR_ARGUMENT, "sj_rope_table: table must be 8-byte aligned");
  const int n = t * (head_dim / 2);
  launch(rope_table_kernel, (n + 255) / 256, 256, 0, as_stream(stream), reinterpret_cast<float2*>(table), t,
                                                                   head_dim / 2, offset, logf(theta),
                                                                   static_cast<float>(head_dim));
  SJ_LAUNCH_CHECK("rope_table");
  return SJ_OK;
}

static int swiglu_bwd(const void* gu, const void* dh, void* dgu, int rows, int f, const int32_t* live,
                      void* stream) {
  if (rows <= 0 || f <= 0 || f % 16) return fail(SJ_ERR_SHAPE, "sj_swiglu_bwd: f=%d must be a multiple of 16", f);
  if (!aligned16(gu) || !aligned16(dh) || !aligned16(dgu))
    return fail(SJ_ERR_ARGUMENT, "sj_swiglu_bwd: 16-byte alignment required");
  const size_t threads = static_cast<size_t>(rows) * (f / 8);
  size_t blocks = (threads + 255) / 256;
  if (live != nullptr) blocks = std::min<size_t>(blocks, static_cast<size_t>(sm_count()) * 8);
  launch(swiglu_bwd_kernel, static_cast<unsigned>(blocks), 256, 0, as_stream(stream),
      static_cast<const __nv_bfloat16*>(gu), static_cast<const __nv_bfloat16*>(dh), static_cast<__nv_bfloat16*>(dgu),
      rows, f, live);
  SJ_LAUNCH_CHECK("swiglu_bwd");
  return SJ_OK;
}

extern "C" int sj_swiglu_bwd(const void* gu, const void* dh, void* dgu, int rows, int f, void* stream) {
  return swiglu_bwd(gu, dh, dgu, rows, f, nullptr, stream);
}

extern "C" int sj_swiglu_bwd_live(const void* gu, const void* dh, void* dgu, int rows, int f, const int32_t* live_rows,
                                  void* stream) {
  if (!live_rows) return fail(SJ_ERR_ARGUMENT, "sj_swiglu_bwd_live: null row count");
  return swiglu_bwd(gu, dh, dgu, rows, f, live_rows, stream);
}

extern "C" int sj_patch_pool_fwd(const void* x, void* y, int batch, int t, int d, int patch, void* stream) {
  if (batch <= 0 || t <= 0 || d % 8 || patch <= 0) return fail(SJ_ERR_SHAPE, "sj_patch_pool_fwd: bad shape");
  const int patches = (t + patch - 1) / patch;
  const size_t threads = static_cast<size_t>(batch) * patches * (d / 8);
  launch(patch_pool_fwd_kernel, static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream), 
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), batch, t, d, patch);
  SJ_LAUNCH_CHECK("patch_pool_fwd");
  return SJ_OK;
}

extern "C" int sj_patch_pool_bwd(const float* dy, float* dx, int batch, int t, int d, int patch, void* stream) {
  if (batch <= 0 || t <= 0 || d % 4 || patch <= 0) return fail(SJ_ERR_SHAPE, "sj_patch_pool_bwd: bad shape");
  const size_t threads = static_cast<size_t>(batch) * t * (d / 4);
  launch(patch_pool_bwd_kernel, static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream), dy, dx, batch, t,
                                                                                                    d, patch);
  SJ_LAUNCH_CHECK("patch_pool_bwd");
  return SJ_OK;
}

extern "C" int sj_patch_broadcast_fwd(const void* z, const void* bos, void* y, int y_dtype, int add, int batch, int t,
                                      int d, int patch, void* stream) {
  if (batch <= 0 || t <= 0 || d % 8 || patch <= 0) return fail(SJ_ERR_SHAPE, "sj_patch_broadcast_fwd: bad shape");
  const size_t threads = static_cast<size_t>(batch) * t * (d / 8);
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  const auto* zz = static_cast<const __nv_bfloat16*>(z);
  const auto* bb = static_cast<const __nv_bfloat16*>(bos);
  if (y_dtype == SJ_BF16)
    launch(patch_broadcast_fwd_kernel<false>, grid, 256, 0, as_stream(stream), zz, bb, y, add, batch, t, d, patch);
  else if (y_dtype == SJ_F32)
    launch(patch_broadcast_fwd_kernel<true>, grid, 256, 0, as_stream(stream), zz, bb, y, add, batch, t, d, patch);
  else
    return fail(SJ_ERR_ARGUMENT, "sj_patch_broadcast_fwd: y must be bf16 or f32");
  SJ_LAUNCH_CHECK("patch_broadcast_fwd");
  return SJ_OK;
}

extern "C" int sj_patch_broadcast_bwd(const float* dy, void* dz, void* dbos, int batch, int t, int d, int patch,
                                      void* stream) {
  if (batch <= 0 || t <= 0 || d <= 0 || patch <= 0) return fail(SJ_ERR_SHAPE, "sj_patch_broadcast_bwd: bad shape");
  const int patches = (t + patch - 1) / patch;
  const int body = batch * patches * d;
  const int total = body + d;
  launch(patch_broadcast_bwd_kernel, (total + 255) / 256, 256, 0, as_stream(stream), 
      dy, static_cast<__nv_bfloat16*>(dz), static_cast<__nv_bfloat16*>(dbos), batch, t, d, patch, body);
  SJ_LAUNCH_CHECK("patch_broadcast_bwd");
  return SJ_OK;
}

extern "C" int sj_cast(const void* x, int x_dtype, void* y, int y_dtype, size_t n, void* stream) {
  if (n == 0) return SJ_OK;
  cudaStream_t s = as_stream(stream);
  const int g = grid_for(n, 256);
  if (x_dtype == SJ_F32 && y_dtype == SJ_BF16)
    launch(cast_kernel<float, __nv_bfloat16>, g, 256, 0, s, static_cast<const float*>(x), static_cast<__nv_bfloat16*>(y), n);
  else if (x_dtype == SJ_BF16 && y_dtype == SJ_F32)
    launch(cast_kernel<__nv_bfloat16, float>, g, 256, 0, s, static_cast<const __nv_bfloat16*>(x), static_cast<float*>(y), n);
  else if (x_dtype == SJ_F32 && y_dtype == SJ_F64)
    launch(cast_kernel<float, double>, g, 256, 0, s, static_cast<const float*>(x), static_cast<double*>(y), n);
  else if (x_dtype == SJ_F64 && y_dtype == SJ_F32)
    launch(cast_kernel<double, float>, g, 256, 0, s, static_cast<const double*>(x), static_cast<float*>(y), n);
  else
    return fail(SJ_ERR_UNSUPPORTED, "sj_cast: %d -> %d not supported", x_dtype, y_dtype);
  SJ_LAUNCH_CHECK("cast");
  return SJ_OK;
}

extern "C" int sj_add(const void* x, const void* z, void* y, size_t n, float alpha, int dtype, void* stream) {
  if (n == 0) return SJ_OK;
  cudaStream_t s = as_stream(stream);
  const int g = grid_for(n, 256);
  if (dtype == SJ_F32)
    launch(add_kernel<float>, g, 256, 0, s, static_cast<const float*>(x), static_cast<const float*>(z),
                                         static_cast<float*>(y), n, alpha);
  else if (dtype == SJ_BF16)
    launch(add_kernel<__nv_bfloat16>, g, 256, 0, s, static_cast<const __nv_bfloat16*>(x),
                                                 static_cast<const __nv_bfloat16*>(z), static_cast<__nv_bfloat16*>(y),
                                                 n, alpha);
  else
    return fail(SJ_ERR_UNSUPPORTED, "sj_add: dtype %d", dtype);
  SJ_LAUNCH_CHECK("add");
  return SJ_OK;
}
