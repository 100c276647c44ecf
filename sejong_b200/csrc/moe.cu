// Mixture-of-experts routing and data movement for the byte model's MoE blocks.
//
// Restates the reference's route / pack / combine kernels (python/sejong_kernels/ops/hierarchy.py:
// 174-250; Engine::route_topk, expert_routes, expert_combine and their backwards, crates/sejong-gpu/
// src/hierarchy_ops.rs:280-454; the block, crates/sejong-model/src/architecture.rs:229-241): softmax
// over the experts, top-k by logit with the lowest index on ties, gate = the full-softmax
// probability of the chosen expert, every routed row kept.  Two opt-in additions that the reference
// lacks (the MoE benchmark configuration asks for them): an expert capacity (sj_route_capacity) and the load-balancing
// loss (sj_moe_aux); with capacity unlimited and weight 0 the path is the reference's.
//
// Where the reference reads the expert counts back to the host and runs one small GEMM per expert,
// everything here stays on the device: the pack writes, per expert, a segment of packed rows padded
// to a multiple of 128 (group_rows[e] .. group_rows[e+1]), so that one grouped tcgen05 GEMM covers
// all experts (sj_gemm_grouped) and the step can be captured in a CUDA graph.  The packed order
// inside a segment is the reference's: routed slots (row * k + j) in increasing order.  Combine and
// its backward are gathers (one writer per output element), so they are deterministic.
#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {
constexpr int kMaxExperts = 32;
constexpr int kSegment = 128;
constexpr int kPackThreads = 1024;

SJ_DEVICE void load8_bf16(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
}  // namespace

// hierarchy.py:174-190, thread per row.
__global__ void route_topk_kernel(const float* logits, int ld, int rows, int experts, int k, int32_t* ids,
                                  float* gates) {
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float s[kMaxExperts];
  float mx = -INFINITY;
  for (int e = 0; e < experts; ++e) {
    s[e] = logits[static_cast<size_t>(r) * ld + e];
    mx = fmaxf(mx, s[e]);
  }
  float den = 0.f;
  for (int e = 0; e < experts; ++e) den += expf(s[e] - mx);
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int idx = experts;
    for (int e = 0; e < experts; ++e)
      if (s[e] > best || (s[e] == best && e < idx)) {
        best = s[e];
        idx = e;
      }
    ids[static_cast<size_t>(r) * k + j] = idx;
    gates[static_cast<size_t>(r) * k + j] = expf(best - mx) / den;
    s[idx] = -INFINITY;
  }
}

// One CTA: histogram of the routed slots, padded segment offsets, then the stable placement of every
// slot (chunks of 1024 slots; warp ballots rank the slots of each expert inside a chunk).
__global__ void __launch_bounds__(kPackThreads) route_pack_kernel(const int32_t* ids, int slots, int experts,
                                                                  int32_t* group_rows, int32_t* pos,
                                                                  int32_t* row_slot, int cap) {
  pdl_wait();
  __shared__ int count[kMaxExperts], base[kMaxExperts], seg[kMaxExperts + 1];
  __shared__ int warp_count[kPackThreads / 32][kMaxExperts];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (t < kMaxExperts) count[t] = 0;
  __syncthreads();
  for (int i = t; i < slots; i += kPackThreads) {
    const int e = ids[i];
    if (e >= 0 && e < experts) atomicAdd(&count[e], 1);
  }
  __syncthreads();
  if (t == 0) {
    int off = 0;
    for (int e = 0; e < experts; ++e) {
      seg[e] = off;
      base[e] = off;
      off += (count[e] + kSegment - 1) / kSegment * kSegment;
    }
    seg[experts] = off;
  }
  __syncthreads();
  for (int e = t; e <= experts; e += kPackThreads) group_rows[e] = seg[e];
  // padding rows (and everything past the last segment) route nowhere
  for (int r = t; r < cap; r += kPackThreads) {
    int e = 0;
    while (e < experts && r >= seg[e + 1]) ++e;
    if (e >= experts || r >= seg[e] + count[e]) row_slot[r] = -1;
  }
  for (int c0 = 0; c0 < slots; c0 += kPackThreads) {
    const int i = c0 + t;
    const int e = i < slots ? ids[i] : -1;
    const unsigned lt = (1u << lane) - 1u;
    int rank = 0;
    for (int x = 0; x < experts; ++x) {
      const unsigned m = __ballot_sync(0xffffffffu, e == x);
      if (lane == 0) warp_count[warp][x] = __popc(m);
      if (e == x) rank = __popc(m & lt);
    }
    __syncthreads();
    if (e >= 0 && e < experts) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += warp_count[w][e];
      const int p = base[e] + before + rank;
      pos[i] = p;
      row_slot[p] = i;
    } else if (i < slots) {
      pos[i] = -1;
    }
    __syncthreads();
    if (t < experts) {
      int total = 0;
      for (int w = 0; w < kPackThreads / 32; ++w) total += warp_count[w][t];
      base[t] += total;
    }
    __syncthreads();
  }
}

// A[r] = z[slot / k] for routed rows, 0 for padding; thread per 8 columns.
__global__ void moe_dispatch_kernel(const __nv_bfloat16* z, int ldz, const int32_t* row_slot, int cap, int k, int d,
                                    __nv_bfloat16* a) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int vpr = d / 8;
  if (i >= static_cast<size_t>(cap) * vpr) return;
  const int r = static_cast<int>(i / vpr), c = static_cast<int>(i % vpr) * 8;
  const int slot = row_slot[r];
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (slot >= 0) v = *reinterpret_cast<const uint4*>(z + static_cast<size_t>(slot / k) * ldz + c);
  *reinterpret_cast<uint4*>(a + static_cast<size_t>(r) * d + c) = v;
}

// y[t] = x[t] + sum_j gate[t, j] out[pos[t, j]] (hierarchy.py:229-234 and the block's residual add),
// thread per 8 columns of a token.
__global__ void moe_combine_kernel(const __nv_bfloat16* out, const int32_t* pos, const float* gates, const float* x,
                                   float* y, int rows, int k, int d) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int vpr = d / 8;
  if (i >= static_cast<size_t>(rows) * vpr) return;
  const int t = static_cast<int>(i / vpr), c = static_cast<int>(i % vpr) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const int p = pos[static_cast<size_t>(t) * k + j];
    if (p < 0) continue;
    const float g = gates[static_cast<size_t>(t) * k + j];
    float v[8];
    load8_bf16(out + static_cast<size_t>(p) * d + c, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(g, v[e], acc[e]);
  }
  const float4* xs = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * d + c);
  const float4 a = xs[0], b = xs[1];
  float4* ys = reinterpret_cast<float4*>(y + static_cast<size_t>(t) * d + c);
  ys[0] = make_float4(a.x + acc[0], a.y + acc[1], a.z + acc[2], a.w + acc[3]);
  ys[1] = make_float4(b.x + acc[4], b.y + acc[5], b.z + acc[6], b.w + acc[7]);
}

// hierarchy.py:237-250: d_out[r] = gate * dy[t], d_gate[slot] = <out[r], dy[t]>; warp per packed row.
__global__ void moe_combine_bwd_kernel(const __nv_bfloat16* out, const int32_t* row_slot, const float* gates,
                                       const float* dy, __nv_bfloat16* d_out, float* d_gates, int cap, int k, int d) {
  pdl_wait();
  const int r = static_cast<int>((static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= cap) return;
  const int slot = row_slot[r];
  __nv_bfloat16* dst = d_out + static_cast<size_t>(r) * d;
  if (slot < 0) {
    for (int c = lane * 8; c < d; c += 256) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const int t = slot / k;
  const float g = gates[slot];
  float dot = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    float v[8];
    load8_bf16(out + static_cast<size_t>(r) * d + c, v);
    const float4* ds = reinterpret_cast<const float4*>(dy + static_cast<size_t>(t) * d + c);
    const float4 a = ds[0], b = ds[1];
    const float q[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint4 w;
    w.x = pack_bf16x2(g * q[0], g * q[1]);
    w.y = pack_bf16x2(g * q[2], g * q[3]);
    w.z = pack_bf16x2(g * q[4], g * q[5]);
    w.w = pack_bf16x2(g * q[6], g * q[7]);
    *reinterpret_cast<uint4*>(dst + c) = w;
#pragma unroll
    for (int e = 0; e < 8; ++e) dot = fmaf(v[e], q[e], dot);
  }
  dot = warp_sum(dot);
  if (lane == 0) d_gates[slot] = dot;
}

// hierarchy.py:193-208: dlogits = p * (dy on the chosen experts - sum_j gate_j dy_j), thread per row.
__global__ void route_topk_bwd_kernel(const float* logits, int ld, const int32_t* ids, const float* gates,
                                      const float* d_gates, __nv_bfloat16* dlogits, int ldd, int rows, int experts,
                                      int k) {
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float s[kMaxExperts], sel[kMaxExperts];
  float mx = -INFINITY;
  for (int e = 0; e < experts; ++e) {
    s[e] = logits[static_cast<size_t>(r) * ld + e];
    mx = fmaxf(mx, s[e]);
    sel[e] = 0.f;
  }
  float den = 0.f;
  for (int e = 0; e < experts; ++e) {
    s[e] = expf(s[e] - mx);
    den += s[e];
  }
  float total = 0.f;
  for (int j = 0; j < k; ++j) {
    const int e = ids[static_cast<size_t>(r) * k + j];
    if (e < 0 || e >= experts) continue;  // a slot dropped by the capacity: no output, no gradient
    const float dyj = d_gates[static_cast<size_t>(r) * k + j];
    sel[e] += dyj;
    total += gates[static_cast<size_t>(r) * k + j] * dyj;
  }
  for (int e = 0; e < ldd; ++e)
    dlogits[static_cast<size_t>(r) * ldd + e] = f2bf(e < experts ? s[e] / den * (sel[e] - total) : 0.f);
}

// dz[t] = sum_j dA[pos[t, j]] (gather backward of the dispatch), thread per 8 columns.
__global__ void moe_dispatch_bwd_kernel(const float* da, const int32_t* pos, float* dz, int ldz, int rows, int k,
                                        int d) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int vpr = d / 8;
  if (i >= static_cast<size_t>(rows) * vpr) return;
  const int t = static_cast<int>(i / vpr), c = static_cast<int>(i % vpr) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const int p = pos[static_cast<size_t>(t) * k + j];
    if (p < 0) continue;
    const float4* s = reinterpret_cast<const float4*>(da + static_cast<size_t>(p) * d + c);
    const float4 a = s[0], b = s[1];
    acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
    acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
  }
  float4* o = reinterpret_cast<float4*>(dz + static_cast<size_t>(t) * ldz + c);
  o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// Expert capacity (an addition to the reference, whose experts take every routed row): each expert
// keeps at most `capacity` slots; every row's first choice comes before any second choice, and within
// one choice rows go in order; a dropped slot's expert id becomes -1, so the pack, the combine and the
// backwards leave it out (its row keeps the residual and its other experts).  One CTA: per choice j,
// chunks of 1024 rows ranked per expert with warp ballots on top of the running fill.
__global__ void __launch_bounds__(kPackThreads) route_capacity_kernel(int32_t* ids, int rows, int k, int experts,
                                                                      int capacity) {
  pdl_wait();
  __shared__ int fill[kMaxExperts];
  __shared__ int warp_count[kPackThreads / 32][kMaxExperts];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (t < kMaxExperts) fill[t] = 0;
  __syncthreads();
  for (int j = 0; j < k; ++j) {
    for (int r0 = 0; r0 < rows; r0 += kPackThreads) {
      const int r = r0 + t;
      int32_t* slot = ids + static_cast<size_t>(r) * k + j;
      const int e = r < rows ? *slot : -1;
      const unsigned lt = (1u << lane) - 1u;
      int rank = 0;
      for (int x = 0; x < experts; ++x) {
        const unsigned m = __ballot_sync(0xffffffffu, e == x);
        if (lane == 0) warp_count[warp][x] = __popc(m);
        if (e == x) rank = __popc(m & lt);
      }
      __syncthreads();
      if (e >= 0 && e < experts) {
        int before = fill[e];
        for (int w = 0; w < warp; ++w) before += warp_count[w][e];
        if (before + rank >= capacity) *slot = -1;
      }
      __syncthreads();
      if (t < experts) {
        int total = 0;
        for (int w = 0; w < kPackThreads / 32; ++w) total += warp_count[w][t];
        fill[t] += total;
      }
      __syncthreads();
    }
  }
}

// Load-balancing loss (an addition; the Switch Transformer form): aux = weight * E * sum_e f_e P_e with
// f_e the fraction of the rows' top-k choices (before any capacity drop) that picked expert e and
// P_e the mean router probability of e.  f is piecewise constant, so d aux / d logit[r, e'] =
// weight * E / rows * p[r, e'] * (f_e' - sum_e f_e p[r, e]).  One CTA: the routing and probabilities
// are recomputed from the logits (the rule of route_topk_kernel), reduced, then the loss is added to
// the FP64 loss sum (times loss_seed) and the gradient (times grad_scale) to the bf16 router gradient.
constexpr int kAuxThreads = 256;  // rows per CTA (thread per row) of the two load-balancing kernels

// Pass 1: per CTA (256 rows), the rows' top-k choice counts and summed router probabilities, written
// to partials[cta][0 .. E) (counts) and [E .. 2E) (probability sums); no atomics on global memory, so
// pass 2 reduces them in a fixed order.
__global__ void __launch_bounds__(kAuxThreads) moe_aux_stats_kernel(const float* logits, int ld, int rows, int experts,
                                                                    int k, float* partials) {
  pdl_wait();
  __shared__ float part[kAuxThreads / 32][2 * kMaxExperts];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int r = blockIdx.x * kAuxThreads + t;
  // per-expert arrays indexed by compile-time constants only (guarded by `experts`): registers
  float s[kMaxExperts], x[kMaxExperts], cnt[kMaxExperts];
  float mx = -INFINITY, den = 0.f;
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) {
    s[e] = (r < rows && e < experts) ? logits[static_cast<size_t>(r) * ld + e] : -INFINITY;
    mx = fmaxf(mx, s[e]);
    cnt[e] = 0.f;
  }
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) {
    x[e] = (r < rows && e < experts) ? expf(s[e] - mx) : 0.f;
    den += x[e];
  }
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) x[e] = r < rows ? x[e] / den : 0.f;
  if (r < rows) {
    for (int j = 0; j < k; ++j) {
      float best = -INFINITY;
      int idx = experts;
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e)
        if (e < experts && s[e] > best) {  // strict: the lowest index wins a tie
          best = s[e];
          idx = e;
        }
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e)
        if (e == idx) {
          cnt[e] += 1.f;
          s[e] = -INFINITY;
        }
    }
  }
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) {
    if (e >= experts) break;
    const float c = warp_sum(cnt[e]), q = warp_sum(x[e]);
    if (lane == 0) {
      part[warp][e] = c;
      part[warp][experts + e] = q;
    }
  }
  __syncthreads();
  if (t < 2 * experts) {
    float tot = 0.f;
    for (int w = 0; w < kAuxThreads / 32; ++w) tot += part[w][t];
    partials[static_cast<size_t>(blockIdx.x) * 2 * experts + t] = tot;
  }
}

// Pass 2: every CTA reduces the partials (same order in every CTA), then adds the loss (CTA 0) and the
// gradient of its 256 rows to the bf16 router gradient.
__global__ void __launch_bounds__(kAuxThreads) moe_aux_grad_kernel(const float* logits, int ld, int rows, int experts,
                                                                   int k, int ctas, const float* partials,
                                                                   float weight, double loss_seed, double* loss_sum,
                                                                   __nv_bfloat16* dlogits, int ldd, float grad_scale) {
  pdl_wait();
  __shared__ float fP[2 * kMaxExperts];
  const int t = threadIdx.x;
  if (t < 2 * experts) {
    float tot = 0.f;
    for (int c = 0; c < ctas; ++c) tot += partials[static_cast<size_t>(c) * 2 * experts + t];
    fP[t] = t < experts ? tot / static_cast<float>(rows * k) : tot / static_cast<float>(rows);
  }
  __syncthreads();
  if (blockIdx.x == 0 && t == 0) {
    double aux = 0.0;
    for (int e = 0; e < experts; ++e) aux += static_cast<double>(fP[e]) * fP[experts + e];
    loss_sum[0] += loss_seed * static_cast<double>(weight) * experts * aux;
  }
  const int r = blockIdx.x * kAuxThreads + t;
  if (r >= rows) return;
  float p[kMaxExperts], fr[kMaxExperts];
  float mx = -INFINITY, den = 0.f, fp = 0.f;
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) {
    p[e] = e < experts ? logits[static_cast<size_t>(r) * ld + e] : -INFINITY;
    fr[e] = e < experts ? fP[e] : 0.f;
    mx = fmaxf(mx, p[e]);
  }
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) {
    p[e] = e < experts ? expf(p[e] - mx) : 0.f;
    den += p[e];
  }
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) {
    p[e] /= den;
    fp += fr[e] * p[e];
  }
  const float scale = grad_scale * weight * static_cast<float>(experts) / static_cast<float>(rows);
  __nv_bfloat16* row = dlogits + static_cast<size_t>(r) * ldd;
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e)
    if (e < experts) row[e] = f2bf(bf2f(row[e]) + scale * p[e] * (fr[e] - fp));
}

}  // namespace sj

using namespace sj;

extern "C" int sj_route_capacity(int32_t* ids, int rows, int k, int experts, int capacity, void* stream) {
  if (rows <= 0 || k <= 0 || experts <= 0 || experts > kMaxExperts || capacity <= 0)
    return fail(SJ_ERR_SHAPE, "sj_route_capacity: rows=%d k=%d experts=%d (<= %d) capacity=%d", rows, k, experts,
                kMaxExperts, capacity);
  if (!ids) return fail(SJ_ERR_ARGUMENT, "sj_route_capacity: null ids");
  launch(route_capacity_kernel, 1, kPackThreads, 0, as_stream(stream), ids, rows, k, experts, capacity);
  SJ_LAUNCH_CHECK("route_capacity");
  return SJ_OK;
}

extern "C" size_t sj_moe_aux_workspace(int rows, int experts) {
  if (rows <= 0 || experts <= 0) return 0;
  return static_cast<size_t>((rows + kAuxThreads - 1) / kAuxThreads) * 2 * experts;
}

extern "C" int sj_moe_aux(const float* logits, int ld, int rows, int experts, int k, float weight, double loss_seed,
                          double* loss_sum, void* dlogits, int ldd, float grad_scale, float* workspace,
                          void* stream) {
  if (rows <= 0 || experts <= 0 || experts > kMaxExperts || k <= 0 || k > experts || ld < experts || ldd < experts)
    return fail(SJ_ERR_SHAPE, "sj_moe_aux: rows=%d experts=%d k=%d", rows, experts, k);
  if (!logits || !loss_sum || !dlogits || !workspace) return fail(SJ_ERR_ARGUMENT, "sj_moe_aux: null pointer");
  const int ctas = (rows + kAuxThreads - 1) / kAuxThreads;
  launch(moe_aux_stats_kernel, ctas, kAuxThreads, 0, as_stream(stream), logits, ld, rows, experts, k, workspace);
  SJ_LAUNCH_CHECK("moe_aux_stats");
  launch(moe_aux_grad_kernel, ctas, kAuxThreads, 0, as_stream(stream), logits, ld, rows, experts, k, ctas,
         static_cast<const float*>(workspace), weight, loss_seed, loss_sum, static_cast<__nv_bfloat16*>(dlogits), ldd,
         grad_scale);
  SJ_LAUNCH_CHECK("moe_aux_grad");
  return SJ_OK;
}

extern "C" int sj_moe_capacity(int rows, int k, int experts) {
  if (rows <= 0 || k <= 0 || experts <= 0) return 0;
  const long long need = static_cast<long long>(rows) * k + static_cast<long long>(experts) * (kSegment - 1);
  return static_cast<int>((need + kSegment - 1) / kSegment * kSegment);
}

extern "C" int sj_route_topk(const float* logits, int ld, int rows, int experts, int k, int32_t* ids, float* gates,
                             void* stream) {
  if (rows <= 0 || experts <= 0 || experts > kMaxExperts || k <= 0 || k > experts || ld < experts)
    return fail(SJ_ERR_SHAPE, "sj_route_topk: rows=%d experts=%d (<= %d) k=%d", rows, experts, kMaxExperts, k);
  if (!logits || !ids || !gates) return fail(SJ_ERR_ARGUMENT, "sj_route_topk: null pointer");
  launch(route_topk_kernel, (rows + 127) / 128, 128, 0, as_stream(stream), logits, ld, rows, experts, k, ids, gates);
  SJ_LAUNCH_CHECK("route_topk");
  return SJ_OK;
}

extern "C" int sj_route_pack(const int32_t* ids, int rows, int experts, int k, int32_t* group_rows, int32_t* pos,
                             int32_t* row_slot, int cap, void* stream) {
  if (rows <= 0 || experts <= 0 || experts > kMaxExperts || k <= 0)
    return fail(SJ_ERR_SHAPE, "sj_route_pack: rows=%d experts=%d (<= %d) k=%d", rows, experts, kMaxExperts, k);
  if (cap < sj_moe_capacity(rows, k, experts))
    return fail(SJ_ERR_CAPACITY, "sj_route_pack: capacity %d below sj_moe_capacity %d", cap,
                sj_moe_capacity(rows, k, experts));
  if (!ids || !group_rows || !pos || !row_slot) return fail(SJ_ERR_ARGUMENT, "sj_route_pack: null pointer");
  launch(route_pack_kernel, 1, kPackThreads, 0, as_stream(stream), ids, rows * k, experts, group_rows, pos, row_slot,
         cap);
  SJ_LAUNCH_CHECK("route_pack");
  return SJ_OK;
}

extern "C" int sj_moe_dispatch(const void* z, int ldz, const int32_t* row_slot, int cap, int k, int d, void* a,
                               void* stream) {
  if (cap <= 0 || k <= 0 || d <= 0 || d % 8 || ldz % 8) return fail(SJ_ERR_SHAPE, "sj_moe_dispatch: bad shape");
  if (!aligned16(z) || !aligned16(a) || !row_slot) return fail(SJ_ERR_ARGUMENT, "sj_moe_dispatch: aligned operands");
  const size_t n = static_cast<size_t>(cap) * (d / 8);
  launch(moe_dispatch_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream),
         static_cast<const __nv_bfloat16*>(z), ldz, row_slot, cap, k, d, static_cast<__nv_bfloat16*>(a));
  SJ_LAUNCH_CHECK("moe_dispatch");
  return SJ_OK;
}

extern "C" int sj_moe_combine(const void* out, const int32_t* pos, const float* gates, const float* x, float* y,
                              int rows, int k, int d, void* stream) {
  if (rows <= 0 || k <= 0 || d <= 0 || d % 8) return fail(SJ_ERR_SHAPE, "sj_moe_combine: bad shape");
  if (!aligned16(out) || !aligned16(x) || !aligned16(y) || !pos || !gates)
    return fail(SJ_ERR_ARGUMENT, "sj_moe_combine: aligned operands");
  const size_t n = static_cast<size_t>(rows) * (d / 8);
  launch(moe_combine_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream),
         static_cast<const __nv_bfloat16*>(out), pos, gates, x, y, rows, k, d);
  SJ_LAUNCH_CHECK("moe_combine");
  return SJ_OK;
}

extern "C" int sj_moe_combine_bwd(const void* out, const int32_t* row_slot, const float* gates, const float* dy,
                                  void* d_out, float* d_gates, int cap, int k, int d, void* stream) {
  if (cap <= 0 || k <= 0 || d <= 0 || d % 8) return fail(SJ_ERR_SHAPE, "sj_moe_combine_bwd: bad shape");
  if (!aligned16(out) || !aligned16(dy) || !aligned16(d_out) || !row_slot || !gates || !d_gates)
    return fail(SJ_ERR_ARGUMENT, "sj_moe_combine_bwd: aligned operands");
  launch(moe_combine_bwd_kernel, static_cast<unsigned>((static_cast<size_t>(cap) * 32 + 255) / 256), 256, 0,
         as_stream(stream), static_cast<const __nv_bfloat16*>(out), row_slot, gates, dy,
         static_cast<__nv_bfloat16*>(d_out), d_gates, cap, k, d);
  SJ_LAUNCH_CHECK("moe_combine_bwd");
  return SJ_OK;
}

extern "C" int sj_route_topk_bwd(const float* logits, int ld, const int32_t* ids, const float* gates,
                                 const float* d_gates, void* dlogits, int ldd, int rows, int experts, int k,
                                 void* stream) {
  if (rows <= 0 || experts <= 0 || experts > kMaxExperts || k <= 0 || k > experts || ld < experts || ldd < experts)
    return fail(SJ_ERR_SHAPE, "sj_route_topk_bwd: bad shape");
  if (!logits || !ids || !gates || !d_gates || !dlogits) return fail(SJ_ERR_ARGUMENT, "sj_route_topk_bwd: null");
  launch(route_topk_bwd_kernel, (rows + 127) / 128, 128, 0, as_stream(stream), logits, ld, ids, gates, d_gates,
         static_cast<__nv_bfloat16*>(dlogits), ldd, rows, experts, k);
  SJ_LAUNCH_CHECK("route_topk_bwd");
  return SJ_OK;
}

extern "C" int sj_moe_dispatch_bwd(const float* da, const int32_t* pos, float* dz, int ldz, int rows, int k, int d,
                                   void* stream) {
  if (rows <= 0 || k <= 0 || d <= 0 || d % 8 || ldz % 4) return fail(SJ_ERR_SHAPE, "sj_moe_dispatch_bwd: bad shape");
  if (!aligned16(da) || !aligned16(dz) || !pos) return fail(SJ_ERR_ARGUMENT, "sj_moe_dispatch_bwd: aligned operands");
  const size_t n = static_cast<size_t>(rows) * (d / 8);
  launch(moe_dispatch_bwd_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream), da, pos, dz, ldz,
         rows, k, d);
  SJ_LAUNCH_CHECK("moe_dispatch_bwd");
  return SJ_OK;
}
