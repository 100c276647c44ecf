// MiniLM-shaped BERT encoder forward (the frozen text encoder of the reference's native models):
// embedding gather + LayerNorm, LayerNorm, and single-tile non-causal attention on tcgen05.
//
// Restates BertEncoder::hidden (crates/sejong-model/src/native/bert.rs:360-411), which runs one
// unpadded sequence at a time.  Here a batch of sequences is packed row after row (cu_seqlens
// gives each sequence's first row), so no padding enters any product and every sequence sees
// exactly its own keys, as in the reference.  The linear layers run on the tcgen05 GEMM with the
// bias / GELU / residual epilogues (gemm.cu, sj_gemm_bias).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {

constexpr int kBertMaxLen = 128;   // one 128-row tile per sequence
constexpr int kBertHead = 32;      // head dim (MiniLM: 384 / 12)

// Sequence of packed row `row`: the s with cu[s] <= row < cu[s + 1] (cu non-decreasing).
SJ_DEVICE int sequence_of(const int32_t* cu, int batch, int row) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Warp-per-row LayerNorm of NV float4 per lane (d = 128 NV): common.py:6-14 — mean, centred
// variance over d, y = (x - mean) / sqrt(var + eps) * w + b.  Writes f32 and (optionally) bf16.
template <int NV>
SJ_DEVICE void layernorm_row(float (&x)[NV][4], const float* w, const float* b, float eps, int d, int lane, float* y,
                             __nv_bfloat16* yb) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) s += x[i][e];
  const float mean = warp_sum(s) / static_cast<float>(d);
  float v = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      x[i][e] -= mean;
      v += x[i][e] * x[i][e];
    }
  const float inv = 1.0f / sqrtf(warp_sum(v) / static_cast<float>(d) + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = 4 * (lane + 32 * i);
    const float4 w4 = *reinterpret_cast<const float4*>(w + col);
    const float4 b4 = *reinterpret_cast<const float4*>(b + col);
    const float o0 = x[i][0] * inv * w4.x + b4.x, o1 = x[i][1] * inv * w4.y + b4.y;
    const float o2 = x[i][2] * inv * w4.z + b4.z, o3 = x[i][3] * inv * w4.w + b4.w;
    *reinterpret_cast<float4*>(y + col) = make_float4(o0, o1, o2, o3);
    if (yb) *reinterpret_cast<uint2*>(yb + col) = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
  }
}

}  // namespace

// x = LayerNorm(word[id] + position[pos] + type[0]) per packed row (bert.rs:364-385).
template <int NV>
__global__ void bert_embed_kernel(const int32_t* ids, const int32_t* cu, int batch, const float* word, int vocab,
                                  const float* position, int max_pos, const float* type0, const float* w,
                                  const float* b, float eps, float* y, __nv_bfloat16* yb, int rows, int d) {
  pdl_wait();
  const int row = static_cast<int>((static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int s = sequence_of(cu, batch, row);
  const int pos = row - cu[s];
  int id = ids[row];
  const bool ok = id >= 0 && id < vocab && pos >= 0 && pos < max_pos;
  if (!ok) {
    if (lane == 0) record_error(SJ_DEV_BAD_INDEX);
    id = 0;
  }
  const int p = ok ? pos : 0;
  float x[NV][4];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = 4 * (lane + 32 * i);
    const float4 a = *reinterpret_cast<const float4*>(word + static_cast<size_t>(id) * d + col);
    const float4 c = *reinterpret_cast<const float4*>(position + static_cast<size_t>(p) * d + col);
    const float4 t = *reinterpret_cast<const float4*>(type0 + col);
    x[i][0] = (a.x + c.x) + t.x;
    x[i][1] = (a.y + c.y) + t.y;
    x[i][2] = (a.z + c.z) + t.z;
    x[i][3] = (a.w + c.w) + t.w;
  }
  layernorm_row<NV>(x, w, b, eps, d, lane, y + static_cast<size_t>(row) * d,
                    yb ? yb + static_cast<size_t>(row) * d : nullptr);
}

template <int NV>
__global__ void layernorm_kernel(const float* x, const float* w, const float* b, float eps, float* y,
                                 __nv_bfloat16* yb, int rows, int d) {
  pdl_wait();
  const int row = static_cast<int>((static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[NV][4];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 a = *reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * d + 4 * (lane + 32 * i));
    v[i][0] = a.x;
    v[i][1] = a.y;
    v[i][2] = a.z;
    v[i][3] = a.w;
  }
  layernorm_row<NV>(v, w, b, eps, d, lane, y + static_cast<size_t>(row) * d,
                    yb ? yb + static_cast<size_t>(row) * d : nullptr);
}

// ------------------------------------------------------------------ single-tile attention
// One CTA per (sequence, head), 4 warps, thread t <-> query row t (TMEM lane t).  Q, K and V rows of
// the head (32 bf16) are written into 128-byte-swizzled shared memory rows, zero-padded to 64
// columns; S = Q K^T (M128 N128, two K16 steps over the 32 real columns) goes to TMEM columns
// 0-127; each thread turns its row into P = exp(scale (s - max)) over the sequence's keys (bf16, K-
// major in shared memory) and its sum; O = P V (M128 N64 K128, V read as an MN-major operand) goes
// to TMEM columns 128-191, and row t is written as O / sum (kernels.py:115-136 with CAUSAL false).
namespace {
constexpr int kTileRows = 128;
constexpr int kRowBytes = 128;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileRows * kRowBytes;      // 16 KB each
constexpr int kOffV = kOffK + kTileRows * kRowBytes;
constexpr int kOffP = kOffV + kTileRows * kRowBytes;      // two 64-key halves, 16 KB each
constexpr int kOffBar = kOffP + 2 * kTileRows * kRowBytes;
constexpr int kSmemAttn = kOffBar + 64 + 1024;
constexpr uint32_t kTmemAttn = 256;

SJ_DEVICE void store_row_swizzled(uint8_t* tile, int r, const uint4 (&chunks)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(tile + r * kRowBytes + ((j ^ (r & 7)) << 4)) = chunks[j];
}
}  // namespace

__global__ void __launch_bounds__(128) bert_attention_kernel(const __nv_bfloat16* qkv, int ldqkv,
                                                             const int32_t* cu, int heads, float scale_log2,
                                                             __nv_bfloat16* out, int ldo) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int t = threadIdx.x, warp = t >> 5;
  const int seq = blockIdx.x / heads, h = blockIdx.x % heads;
  pdl_wait();
  const int row0 = cu[seq];
  const int len = min(cu[seq + 1] - row0, kTileRows);
  // rows of Q, K, V for this head (zero beyond the sequence and in columns 32-63)
  {
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    uint4 cq[8], ck[8], cv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) cq[j] = ck[j] = cv[j] = zero;
    if (t < len) {
      const __nv_bfloat16* base = qkv + static_cast<size_t>(row0 + t) * ldqkv + h * kBertHead;
      const int stride = heads * kBertHead;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cq[j] = reinterpret_cast<const uint4*>(base)[j];
        ck[j] = reinterpret_cast<const uint4*>(base + stride)[j];
        cv[j] = reinterpret_cast<const uint4*>(base + 2 * stride)[j];
      }
    }
    store_row_swizzled(smem + kOffQ, t, cq);
    store_row_swizzled(smem + kOffK, t, ck);
    store_row_swizzled(smem + kOffV, t, cv);
  }
  if (t == 0) {
    mbar_init(bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemAttn);
    tmem_relinquish();
  }
  fence_proxy_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t kIdS = umma_idesc_bf16(kTileRows, kTileRows, 0, 0);  // K-major A and B
  constexpr uint32_t kIdO = umma_idesc_bf16(kTileRows, 64, 0, 1);         // K-major A, MN-major B
  if (t == 0) {
    const uint64_t dq = umma_desc(smem_u32(smem + kOffQ), 16, 1024), dk = umma_desc(smem_u32(smem + kOffK), 16, 1024);
#pragma unroll
    for (int kk = 0; kk < kBertHead / 16; ++kk) umma_f16(tmem, dq + kk * 2, dk + kk * 2, kIdS, kk > 0 ? 1u : 0u);
    umma_commit(bar);
  }
  bool ok = mbar_wait(bar, 0, nullptr, SJ_DEV_ATTN_WAIT);
  tc_fence_after();
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  // row max over the sequence's keys, then P and its sum
  float mx = -INFINITY;
#pragma unroll
  for (int c = 0; c < kTileRows / 32; ++c) {
    uint32_t sv[32];
    tmem_ld_32x32b_x32(tmem + lane_off + c * 32, sv);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c * 32 + j < len) mx = fmaxf(mx, __uint_as_float(sv[j]));
  }
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < kTileRows / 32; ++c) {
    uint32_t sv[32];
    tmem_ld_32x32b_x32(tmem + lane_off + c * 32, sv);
    tmem_wait_ld();
    uint32_t pw[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      float pr[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = c * 32 + j + e;
        float pe = 0.f;
        if (key < len && t < len) {
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(pe) : "f"((__uint_as_float(sv[j + e]) - mx) * scale_log2));
        }
        pr[e] = pe;
        sum += pe;
      }
      pw[j >> 1] = pack_bf16x2(pr[0], pr[1]);
    }
    // keys 32c .. 32c + 31: half c / 2 of P, 16-byte chunks 4 (c & 1) .. 4 (c & 1) + 3 of row t
    uint8_t* half = smem + kOffP + (c >> 1) * kTileRows * kRowBytes;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int j = (c & 1) * 4 + q;
      *reinterpret_cast<uint4*>(half + t * kRowBytes + ((j ^ (t & 7)) << 4)) =
          make_uint4(pw[4 * q], pw[4 * q + 1], pw[4 * q + 2], pw[4 * q + 3]);
    }
  }
  fence_proxy_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (t == 0) {
    const uint64_t dp = umma_desc(smem_u32(smem + kOffP), 16, 1024);
    const uint64_t dv = umma_desc(smem_u32(smem + kOffV), 8192, 1024);
#pragma unroll
    for (int kk = 0; kk < kTileRows / 16; ++kk) {
      const uint64_t kmaj = ((kk >> 2) * kTileRows * kRowBytes + (kk & 3) * 32) >> 4;
      umma_f16(tmem + 128, dp + kmaj, dv + ((kk * 2048) >> 4), kIdO, kk > 0 ? 1u : 0u);
    }
    umma_commit(bar);
  }
  ok = mbar_wait(bar, 1, nullptr, SJ_DEV_ATTN_WAIT) && ok;
  tc_fence_after();
  {
    uint32_t ov[32];
    tmem_ld_32x32b_x32(tmem + lane_off + 128, ov);
    tmem_wait_ld();
    if (ok && t < len) {
      const float inv = 1.0f / sum;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) w[j >> 1] = pack_bf16x2(__uint_as_float(ov[j]) * inv, __uint_as_float(ov[j + 1]) * inv);
      uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row0 + t) * ldo + h * kBertHead);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemAttn);
  }
}

}  // namespace sj

using namespace sj;

extern "C" int sj_bert_embed(const int32_t* ids, const int32_t* cu_seqlens, int batch, const float* word, int vocab,
                             const float* position, int max_position, const float* type0, const float* ln_w,
                             const float* ln_b, float eps, float* x, void* x_bf16, int rows, int d, void* stream) {
  if (rows <= 0 || batch <= 0 || d <= 0 || d % 128 || d > 1024)
    return fail(SJ_ERR_SHAPE, "sj_bert_embed: d=%d must be a multiple of 128 up to 1024", d);
  if (!ids || !cu_seqlens || !word || !position || !type0 || !ln_w || !ln_b || !x)
    return fail(SJ_ERR_ARGUMENT, "sj_bert_embed: null pointer");
  if (!aligned16(word) || !aligned16(position) || !aligned16(type0) || !aligned16(ln_w) || !aligned16(ln_b) ||
      !aligned16(x) || (x_bf16 && (reinterpret_cast<uintptr_t>(x_bf16) & 7)))
    return fail(SJ_ERR_ARGUMENT, "sj_bert_embed: tables and outputs must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>((static_cast<size_t>(rows) * 32 + 255) / 256);
  auto* xb = static_cast<__nv_bfloat16*>(x_bf16);
  switch (d / 128) {
    case 1: launch(bert_embed_kernel<1>, grid, 256, 0, s, ids, cu_seqlens, batch, word, vocab, position, max_position, type0, ln_w, ln_b, eps, x, xb, rows, d); break;
    case 2: launch(bert_embed_kernel<2>, grid, 256, 0, s, ids, cu_seqlens, batch, word, vocab, position, max_position, type0, ln_w, ln_b, eps, x, xb, rows, d); break;
    case 3: launch(bert_embed_kernel<3>, grid, 256, 0, s, ids, cu_seqlens, batch, word, vocab, position, max_position, type0, ln_w, ln_b, eps, x, xb, rows, d); break;
    case 4: launch(bert_embed_kernel<4>, grid, 256, 0, s, ids, cu_seqlens, batch, word, vocab, position, max_position, type0, ln_w, ln_b, eps, x, xb, rows, d); break;
    case 6: launch(bert_embed_kernel<6>, grid, 256, 0, s, ids, cu_seqlens, batch, word, vocab, position, max_position, type0, ln_w, ln_b, eps, x, xb, rows, d); break;
    case 8: launch(bert_embed_kernel<8>, grid, 256, 0, s, ids, cu_seqlens, batch, word, vocab, position, max_position, type0, ln_w, ln_b, eps, x, xb, rows, d); break;
    default: return fail(SJ_ERR_SHAPE, "sj_bert_embed: d=%d not supported (128, 256, 384, 512, 768, 1024)", d);
  }
  SJ_LAUNCH_CHECK("bert_embed");
  return SJ_OK;
}

extern "C" int sj_layernorm(const float* x, const float* w, const float* b, float eps, float* y, void* y_bf16,
                            int rows, int d, void* stream) {
  if (rows <= 0 || d <= 0 || d % 128 || d > 1024)
    return fail(SJ_ERR_SHAPE, "sj_layernorm: d=%d must be a multiple of 128 up to 1024", d);
  if (!x || !w || !b || !y) return fail(SJ_ERR_ARGUMENT, "sj_layernorm: null pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(y) ||
      (y_bf16 && (reinterpret_cast<uintptr_t>(y_bf16) & 7)))
    return fail(SJ_ERR_ARGUMENT, "sj_layernorm: operands must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>((static_cast<size_t>(rows) * 32 + 255) / 256);
  auto* yb = static_cast<__nv_bfloat16*>(y_bf16);
  switch (d / 128) {
    case 1: launch(layernorm_kernel<1>, grid, 256, 0, s, x, w, b, eps, y, yb, rows, d); break;
    case 2: launch(layernorm_kernel<2>, grid, 256, 0, s, x, w, b, eps, y, yb, rows, d); break;
    case 3: launch(layernorm_kernel<3>, grid, 256, 0, s, x, w, b, eps, y, yb, rows, d); break;
    case 4: launch(layernorm_kernel<4>, grid, 256, 0, s, x, w, b, eps, y, yb, rows, d); break;
    case 6: launch(layernorm_kernel<6>, grid, 256, 0, s, x, w, b, eps, y, yb, rows, d); break;
    case 8: launch(layernorm_kernel<8>, grid, 256, 0, s, x, w, b, eps, y, yb, rows, d); break;
    default: return fail(SJ_ERR_SHAPE, "sj_layernorm: d=%d not supported (128, 256, 384, 512, 768, 1024)", d);
  }
  SJ_LAUNCH_CHECK("layernorm");
  return SJ_OK;
}

extern "C" int sj_bert_attention(const void* qkv, int ldqkv, const int32_t* cu_seqlens, int batch, int max_len,
                                 int heads, int head_dim, void* out, int ldo, void* stream) {
  if (head_dim != kBertHead) return fail(SJ_ERR_UNSUPPORTED, "sj_bert_attention: head_dim %d (this build: 32)", head_dim);
  if (batch <= 0 || heads <= 0 || max_len <= 0 || max_len > kBertMaxLen)
    return fail(SJ_ERR_SHAPE, "sj_bert_attention: batch=%d heads=%d max_len=%d (<= %d)", batch, heads, max_len,
                kBertMaxLen);
  if (!qkv || !cu_seqlens || !out) return fail(SJ_ERR_ARGUMENT, "sj_bert_attention: null pointer");
  if (!aligned16(qkv) || !aligned16(out) || (ldqkv % 8) || (ldo % 8) || ldqkv < 3 * heads * head_dim ||
      ldo < heads * head_dim)
    return fail(SJ_ERR_ARGUMENT, "sj_bert_attention: 16-byte aligned rows of [q | k | v] and of the output required");
  static KernelAttrOnce attr_once;
  const int attr_rc = ensure_max_smem(attr_once, reinterpret_cast<const void*>(bert_attention_kernel), kSmemAttn,
                                      "bert attention shared-memory attribute");
  if (attr_rc != SJ_OK) return attr_rc;
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
  launch(bert_attention_kernel, static_cast<unsigned>(batch * heads), 128, kSmemAttn, as_stream(stream),
         static_cast<const __nv_bfloat16*>(qkv), ldqkv, cu_seqlens, heads, scale_log2,
         static_cast<__nv_bfloat16*>(out), ldo);
  SJ_LAUNCH_CHECK("bert_attention");
  return SJ_OK;
}
