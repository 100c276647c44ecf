// KV-cached inference (crates/sejong-model/src/architecture.rs:395-533, `cached_blocks`): the rows
// of a new chunk attend to every cached position before them.
//
//   attn_cached_kernel   Engine::attention_grouped with OFFSET (hierarchy.py:7-39 with offset): row
//                        i of the chunk sits at position offset + i and sees the cached keys
//                        max(0, offset + i + 1 - window) .. offset + i.  One CTA per (row, query
//                        head), four warps: scores q.k (a warp per key, lanes over the 64 dims) into
//                        shared memory, the softmax, then P V with the warps over keys and the
//                        lanes over dim pairs.  Reads each visible K and V row of the head once:
//                        a decode step is bound by the cache bytes it reads.
//   copy_rows_kernel     the K/V append (Engine::copy_into of the chunk's rows into the cache).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {
constexpr int kCachedThreads = 128, kCachedWarps = kCachedThreads / 32, kHeadDim = 64;
constexpr int kMaxCachedKeys = 16384;
}  // namespace

__global__ void __launch_bounds__(kCachedThreads) attn_cached_kernel(const __nv_bfloat16* q, int ldq,
                                                                     const __nv_bfloat16* kc, int ldk,
                                                                     const __nv_bfloat16* vc, int ldv,
                                                                     __nv_bfloat16* o, int ldo, int offset, int hq,
                                                                     int hk, int window) {
  pdl_wait();
  extern __shared__ float sc[];  // scores / probabilities of the visible keys
  __shared__ float qs[kHeadDim];
  __shared__ float red[kCachedWarps];
  __shared__ float part[kCachedWarps][kHeadDim];
  const int i = blockIdx.x, h = blockIdx.y, kvh = h / (hq / hk);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int pos = offset + i;
  const int lo = window > 0 ? max(0, pos + 1 - window) : 0;
  const int nkeys = pos - lo + 1;
  const float scale = rsqrtf(static_cast<float>(kHeadDim));
  if (t < kHeadDim) qs[t] = bf2f(q[static_cast<size_t>(i) * ldq + h * kHeadDim + t]) * scale;
  __syncthreads();
  float mx = -INFINITY;
  for (int j = warp; j < nkeys; j += kCachedWarps) {
    const float2 kv = unpack_bf16x2(
        *reinterpret_cast<const uint32_t*>(kc + static_cast<size_t>(lo + j) * ldk + kvh * kHeadDim + 2 * lane));
    float s = qs[2 * lane] * kv.x + qs[2 * lane + 1] * kv.y;
    s = warp_sum(s);
    if (lane == 0) sc[j] = s;
    mx = fmaxf(mx, s);
  }
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < kCachedWarps; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int j = t; j < nkeys; j += kCachedThreads) {
    const float p = expf(sc[j] - mx);
    sc[j] = p;
    sum += p;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < kCachedWarps; ++w) total += red[w];
  float a0 = 0.f, a1 = 0.f;
  for (int j = warp; j < nkeys; j += kCachedWarps) {
    const float2 vv = unpack_bf16x2(
        *reinterpret_cast<const uint32_t*>(vc + static_cast<size_t>(lo + j) * ldv + kvh * kHeadDim + 2 * lane));
    const float p = sc[j];
    a0 = fmaf(p, vv.x, a0);
    a1 = fmaf(p, vv.y, a1);
  }
  part[warp][2 * lane] = a0;
  part[warp][2 * lane + 1] = a1;
  __syncthreads();
  if (t < kHeadDim) {
    float acc = 0.f;
    for (int w = 0; w < kCachedWarps; ++w) acc += part[w][t];
    o[static_cast<size_t>(i) * ldo + h * kHeadDim + t] = f2bf(acc / total);
  }
}

// rows x (row_bytes / 16) 16-byte vectors
__global__ void copy_rows_kernel(const uint8_t* src, size_t ld_src, uint8_t* dst, size_t ld_dst, int rows,
                                 int vec_per_row) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * vec_per_row) return;
  const int r = static_cast<int>(i / vec_per_row), c = static_cast<int>(i % vec_per_row);
  *reinterpret_cast<uint4*>(dst + r * ld_dst + c * 16) = *reinterpret_cast<const uint4*>(src + r * ld_src + c * 16);
}

// acc[c] = (reset ? 0 : acc[c]) + sum_r x[r, c]  (f32; thread per column) -- the running sum of the
// encoded bytes of the current patch (architecture.rs:749-756, row_mean x count)
__global__ void rows_sum_kernel(const __nv_bfloat16* x, int ldx, int rows, int d, float* acc, int reset) {
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float s = reset ? 0.f : acc[c];
  for (int r = 0; r < rows; ++r) s += bf2f(x[static_cast<size_t>(r) * ldx + c]);
  acc[c] = s;
}

// y = bf16(x * alpha): the pooled patch (architecture.rs:760-762)
__global__ void scale_to_bf16_kernel(const float* x, int n, float alpha, __nv_bfloat16* y) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = f2bf(x[i] * alpha);
}

}  // namespace sj

using namespace sj;

extern "C" int sj_rows_sum_f32(const void* x, int ldx, int rows, int d, float* acc, int reset, void* stream) {
  if (rows < 0 || d <= 0 || ldx < d) return fail(SJ_ERR_SHAPE, "sj_rows_sum_f32: bad shape");
  if (!acc || (rows > 0 && !x)) return fail(SJ_ERR_ARGUMENT, "sj_rows_sum_f32: null");
  launch(rows_sum_kernel, (d + 127) / 128, 128, 0, as_stream(stream), static_cast<const __nv_bfloat16*>(x), ldx, rows,
         d, acc, reset);
  SJ_LAUNCH_CHECK("rows_sum");
  return SJ_OK;
}

extern "C" int sj_scale_to_bf16(const float* x, int n, float alpha, void* y, void* stream) {
  if (n <= 0 || !x || !y) return fail(SJ_ERR_ARGUMENT, "sj_scale_to_bf16: bad argument");
  launch(scale_to_bf16_kernel, (n + 255) / 256, 256, 0, as_stream(stream), x, n, alpha, static_cast<__nv_bfloat16*>(y));
  SJ_LAUNCH_CHECK("scale_to_bf16");
  return SJ_OK;
}

extern "C" int sj_attn_cached(const void* q, int ldq, const void* k_cache, int ldk, const void* v_cache, int ldv,
                              void* o, int ldo, int rows, int offset, int hq, int hk, int head_dim, int window,
                              void* stream) {
  if (head_dim != kHeadDim) return fail(SJ_ERR_UNSUPPORTED, "sj_attn_cached: head_dim %d (this build: 64)", head_dim);
  if (rows <= 0 || offset < 0 || hq <= 0 || hk <= 0 || hq % hk || window < 0)
    return fail(SJ_ERR_SHAPE, "sj_attn_cached: rows=%d offset=%d hq=%d hk=%d window=%d", rows, offset, hq, hk, window);
  const int keys = offset + rows;
  const int visible = window > 0 ? std::min(keys, window) : keys;
  if (visible > kMaxCachedKeys)
    return fail(SJ_ERR_SHAPE, "sj_attn_cached: %d visible keys (this build: up to %d)", visible, kMaxCachedKeys);
  if (!q || !k_cache || !v_cache || !o || (ldq | ldk | ldv | ldo) % 2)
    return fail(SJ_ERR_ARGUMENT, "sj_attn_cached: null operand or odd row stride");
  const size_t smem = static_cast<size_t>(visible) * sizeof(float);
  static KernelAttrOnce attr_once;
  const int attr_rc = ensure_max_smem(attr_once, reinterpret_cast<const void*>(attn_cached_kernel),
                                      static_cast<int>(kMaxCachedKeys * sizeof(float)), "sj_attn_cached: shared memory");
  if (attr_rc != SJ_OK) return attr_rc;
  launch(attn_cached_kernel, dim3(rows, hq), kCachedThreads, smem, as_stream(stream),
         static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(k_cache), ldk,
         static_cast<const __nv_bfloat16*>(v_cache), ldv, static_cast<__nv_bfloat16*>(o), ldo, offset, hq, hk, window);
  SJ_LAUNCH_CHECK("attn_cached");
  return SJ_OK;
}

extern "C" int sj_copy_rows(const void* src, size_t ld_src_bytes, void* dst, size_t ld_dst_bytes, int rows,
                            size_t row_bytes, void* stream) {
  if (rows <= 0 || row_bytes == 0 || row_bytes % 16 || ld_src_bytes % 16 || ld_dst_bytes % 16)
    return fail(SJ_ERR_SHAPE, "sj_copy_rows: rows and strides must be 16-byte multiples");
  if (!aligned16(src) || !aligned16(dst)) return fail(SJ_ERR_ARGUMENT, "sj_copy_rows: 16-byte aligned operands");
  const int vpr = static_cast<int>(row_bytes / 16);
  const size_t n = static_cast<size_t>(rows) * vpr;
  launch(copy_rows_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream),
         static_cast<const uint8_t*>(src), ld_src_bytes, static_cast<uint8_t*>(dst), ld_dst_bytes, rows, vpr);
  SJ_LAUNCH_CHECK("copy_rows");
  return SJ_OK;
}
