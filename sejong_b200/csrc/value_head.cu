// The categorical value head of the NativeValue model (crates/sejong-model/src/native/value.rs:
// 111-160): the hidden state of each request's SEP row, gathered from the body's final-norm output,
// cast to f32 and sent through an f32 affine head (logits = h W + b, graph.rs affine = matmul +
// bias), then the cross entropy against the request's label (Engine::cross_entropy, lib.rs:
// 524-543, kernels.py:176-191) and its backward.  Small, latency-bound work (a few hundred
// requests, a few thousand values): plain f32 FMA kernels, one launch each.
#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {
constexpr int kHeadThreads = 256;
constexpr int kMaxHeadWidth = 4096;
}  // namespace

// One CTA per request b: h = f32(hidden[sel[b]]) staged in shared memory; logits[b, v] = sum_k
// h[k] W[k, v] + bias[v] (k ascending); then the softmax cross entropy over the values:
// dlogits = (softmax - onehot(label)) * seed, loss_sum += (lse - logit[label]) * weight.
__global__ void __launch_bounds__(kHeadThreads) value_head_fwd_kernel(
    const __nv_bfloat16* hidden, int ldh, int rows, const int32_t* sel, int d, const float* w, const float* bias,
    int nv, const int32_t* labels, float seed, float* logits, float* dlogits, double* loss_sum, double weight) {
  pdl_wait();
  __shared__ float hs[kMaxHeadWidth];
  __shared__ float red[kHeadThreads / 32];
  __shared__ float bcast;
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int row = sel[b], label = labels[b];
  if (row < 0 || row >= rows || label < 0 || label >= nv) {
    if (t == 0) record_error(SJ_DEV_BAD_INDEX);
    return;
  }
  for (int k = t; k < d; k += kHeadThreads) hs[k] = bf2f(hidden[static_cast<size_t>(row) * ldh + k]);
  __syncthreads();
  float* out = logits + static_cast<size_t>(b) * nv;
  float mx = -INFINITY;
  for (int v = t; v < nv; v += kHeadThreads) {
    float acc = 0.f;
    for (int k = 0; k < d; ++k) acc = fmaf(hs[k], w[static_cast<size_t>(k) * nv + v], acc);
    acc += bias[v];
    out[v] = acc;
    mx = fmaxf(mx, acc);
  }
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (t == 0) {
    float m = red[0];
    for (int i = 1; i < kHeadThreads / 32; ++i) m = fmaxf(m, red[i]);
    bcast = m;
  }
  __syncthreads();
  const float m = bcast;
  float s = 0.f;
  for (int v = t; v < nv; v += kHeadThreads) s += expf(out[v] - m);
  s = warp_sum(s);
  __syncthreads();
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (t == 0) {
    float total = 0.f;
    for (int i = 0; i < kHeadThreads / 32; ++i) total += red[i];
    bcast = total;
    const float loss = m + logf(total) - out[label];
    if (loss_sum) atomicAdd(loss_sum, static_cast<double>(loss) * weight);
  }
  __syncthreads();
  const float inv = 1.0f / bcast;
  if (dlogits) {
    float* g = dlogits + static_cast<size_t>(b) * nv;
    for (int v = t; v < nv; v += kHeadThreads) g[v] = (expf(out[v] - m) * inv - (v == label ? 1.0f : 0.0f)) * seed;
  }
}

// dW[k, v] += sum_b h_b[k] dlogits[b, v] (threads over (k, v), v fastest); the threads of row k == d
// accumulate dbias[v] += sum_b dlogits[b, v].
__global__ void value_head_wgrad_kernel(const __nv_bfloat16* hidden, int ldh, int rows, const int32_t* sel, int batch,
                                        int d, const float* dlogits, int nv, float* dw, float* dbias) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(d + 1) * nv) return;
  const int k = static_cast<int>(i / nv), v = static_cast<int>(i % nv);
  float acc = 0.f;
  if (k < d) {
    for (int b = 0; b < batch; ++b) {
      const int r = sel[b];
      if (r >= 0 && r < rows) acc = fmaf(bf2f(hidden[static_cast<size_t>(r) * ldh + k]), dlogits[static_cast<size_t>(b) * nv + v], acc);
    }
    dw[static_cast<size_t>(k) * nv + v] += acc;
  } else {
    for (int b = 0; b < batch; ++b) acc += dlogits[static_cast<size_t>(b) * nv + v];
    dbias[v] += acc;
  }
}

// dh[sel[b], k] = sum_v dlogits[b, v] W[k, v]: a warp per (b, k), lanes over v.
__global__ void value_head_dgrad_kernel(int rows, const int32_t* sel, int batch, int d, const float* w,
                                        const float* dlogits, int nv, float* dh, int ldd) {
  pdl_wait();
  const size_t wid = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<size_t>(batch) * d) return;
  const int b = static_cast<int>(wid / d), k = static_cast<int>(wid % d);
  if (sel[b] < 0 || sel[b] >= rows) return;
  const float* wr = w + static_cast<size_t>(k) * nv;
  const float* g = dlogits + static_cast<size_t>(b) * nv;
  float acc = 0.f;
  for (int v = lane; v < nv; v += 32) acc = fmaf(g[v], wr[v], acc);
  acc = warp_sum(acc);
  if (lane == 0) dh[static_cast<size_t>(sel[b]) * ldd + k] = acc;
}

}  // namespace sj

using namespace sj;

extern "C" int sj_value_head_fwd(const void* hidden, int ldh, int rows, const int32_t* sel, int batch, int d,
                                 const float* w, const float* bias, int nv, const int32_t* labels, float seed,
                                 float* logits, float* dlogits, double* loss_sum, double weight, void* stream) {
  if (batch <= 0 || d <= 0 || d > kMaxHeadWidth || nv <= 0 || rows <= 0 || ldh < d)
    return fail(SJ_ERR_SHAPE, "sj_value_head_fwd: batch=%d d=%d (<= %d) values=%d", batch, d, kMaxHeadWidth, nv);
  if (!hidden || !sel || !w || !bias || !labels || !logits) return fail(SJ_ERR_ARGUMENT, "sj_value_head_fwd: null");
  launch(value_head_fwd_kernel, batch, kHeadThreads, 0, as_stream(stream), static_cast<const __nv_bfloat16*>(hidden),
         ldh, rows, sel, d, w, bias, nv, labels, seed, logits, dlogits, loss_sum, weight);
  SJ_LAUNCH_CHECK("value_head_fwd");
  return SJ_OK;
}

extern "C" int sj_value_head_bwd(const void* hidden, int ldh, int rows, const int32_t* sel, int batch, int d,
                                 const float* w, const float* dlogits, int nv, float* dw, float* dbias, float* dh,
                                 int ldd, void* stream) {
  if (batch <= 0 || d <= 0 || nv <= 0 || rows <= 0 || ldh < d || ldd < d) return fail(SJ_ERR_SHAPE, "sj_value_head_bwd: bad shape");
  if (!hidden || !sel || !w || !dlogits || !dw || !dbias || !dh) return fail(SJ_ERR_ARGUMENT, "sj_value_head_bwd: null");
  const size_t n = static_cast<size_t>(d + 1) * nv;
  launch(value_head_wgrad_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream),
         static_cast<const __nv_bfloat16*>(hidden), ldh, rows, sel, batch, d, dlogits, nv, dw, dbias);
  SJ_LAUNCH_CHECK("value_head_wgrad");
  const size_t warps = static_cast<size_t>(batch) * d;
  launch(value_head_dgrad_kernel, static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, as_stream(stream), rows,
         sel, batch, d, w, dlogits, nv, dh, ldd);
  SJ_LAUNCH_CHECK("value_head_dgrad");
  return SJ_OK;
}
