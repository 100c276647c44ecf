// Fused next-byte cross entropy (forward + backward + FP64 loss summary) and the optimizer:
// FP64 gradient norm, device-side clip / LR / bias-correction bookkeeping, multi-tensor AdamW and
// SGD over one flat parameter buffer (one launch instead of one per tensor).
#include "common.cuh"
#include "internal.h"

namespace sj {

// ---------------------------------------------------------------- cross entropy
// One warp per row.  kernels.py:176-191 (forward, backward), kernels.py:254-262 (loss_summary).
SJ_DEVICE void store_grad(__nv_bfloat16* d, float g) { *d = f2bf(g); }
SJ_DEVICE void store_grad(float* d, float g) { *d = g; }

template <typename D>
__global__ void cross_entropy_kernel(const float* logits, int ld, const int32_t* targets,
                                     int rows, int vocab, float seed, float* loss_rows,
                                     D* dlogits, int ld_d, double* loss_sum,
                                     double weight) {
  pdl_wait();
  __shared__ double block_sum[8];
  const int warp_in_block = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_in_block;
  double contribution = 0.0;
  if (row < rows) {
    const float* x = logits + static_cast<size_t>(row) * ld;
    float m = -INFINITY;
    for (int j = lane; j < vocab; j += 32) m = fmaxf(m, x[j]);
    m = warp_max(m);
    float s = 0.f;
    for (int j = lane; j < vocab; j += 32) s += expf(x[j] - m);
    s = warp_sum(s);
    const int target = targets[row];
    const float lse = m + logf(s);
    const float loss = lse - x[target];
    if (lane == 0) {
      if (loss_rows) loss_rows[row] = loss;
      contribution = static_cast<double>(loss) * weight;
    }
    if (dlogits) {
      D* d = dlogits + static_cast<size_t>(row) * ld_d;
      const float inv = 1.0f / s;
      for (int j = lane; j < ld_d; j += 32) {
        float g = 0.f;
        if (j < vocab) g = (expf(x[j] - m) * inv - (j == target ? 1.0f : 0.0f)) * seed;
        store_grad(d + j, g);
      }
    }
  }
  if (lane == 0) block_sum[warp_in_block] = contribution;
  __syncthreads();
  if (threadIdx.x == 0 && loss_sum) {
    double t = 0.0;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += block_sum[w];
    atomicAdd(loss_sum, t);
  }
}

// ---------------------------------------------------------------- gradient norm (kernels.py:265-287)
constexpr int kSumsqThreads = 256;
__global__ void grad_sumsq_kernel(const float* g, size_t n, double* partials) {
  pdl_wait();
  __shared__ double red[kSumsqThreads / 32];
  double acc = 0.0;
  const size_t n4 = n / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 v = g4[i];
    acc += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
           static_cast<double>(v.w) * v.w;
  }
  if (blockIdx.x == 0)
    for (size_t i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) acc += static_cast<double>(g[i]) * g[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kSumsqThreads / 32; ++w) t += red[w];
    partials[blockIdx.x] = t;
  }
}

// hyper layout: [0] lr, [1] 1/(1-b1^t), [2] 1/(1-b2^t), [3] gradient scale, [4] norm, [5] step
__global__ void optim_prepare_kernel(const double* partials, int n_partials, double* state, float* hyper,
                                     float learning_rate, float min_learning_rate, int warmup_steps, int total_steps,
                                     float beta1, float beta2, float clip_norm, int clip_enabled, float loss_scale) {
  pdl_wait();
  __shared__ double red[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n_partials; i += blockDim.x) acc += partials[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x != 0) return;
  double total = 0.0;
  for (int w = 0; w < (blockDim.x >> 5); ++w) total += red[w];
  // max(0): the control-variate correction terms make the total a sum of signed parts, a squared
  // norm only up to rounding
  const double norm = sqrt(fmax(total, 0.0)) / static_cast<double>(loss_scale);
  const double clipping = (clip_enabled && norm > static_cast<double>(clip_norm)) ? clip_norm / norm : 1.0;
  const int step = static_cast<int>(state[0]);  // optimizer.step before the update
  // TrainConfig::lr (crates/sejong-core/src/lib.rs:422-433), f32 arithmetic as in the reference
  float lr;
  if (step < warmup_steps) {
    lr = learning_rate * static_cast<float>(step + 1) / static_cast<float>(warmup_steps);
  } else {
    const int span = max(total_steps - warmup_steps, 1);
    const float phase = fminf(static_cast<float>(max(step - warmup_steps, 0)) / static_cast<float>(span), 1.0f);
    lr = min_learning_rate + 0.5f * (learning_rate - min_learning_rate) * (1.0f + cosf(3.14159265358979323846f * phase));
  }
  const float t = static_cast<float>(step + 1);
  hyper[0] = lr;
  hyper[1] = 1.0f / (1.0f - powf(beta1, t));
  hyper[2] = 1.0f / (1.0f - powf(beta2, t));
  hyper[3] = static_cast<float>(clipping) / loss_scale;
  hyper[4] = static_cast<float>(norm);
  hyper[5] = t;
  state[0] = static_cast<double>(step + 1);
  state[1] = norm;
}

// kernels.py:193-202 per element; decay on [0, n_decay).
__global__ void adamw_kernel(float* w, const float* g, float* m,
                             float* v, __nv_bfloat16* wb, size_t n, size_t n_decay,
                             const float* hyper, float beta1, float beta2, float eps, float wd) {
  pdl_wait();
  const float lr = hyper[0], inv_b1 = hyper[1], inv_b2 = hyper[2], scale = hyper[3];
  const size_t n4 = n / 4;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (n + 3) / 4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (i < n4) {
      float4 w4 = reinterpret_cast<float4*>(w)[i];
      const float4 g4 = reinterpret_cast<const float4*>(g)[i];
      float4 m4 = reinterpret_cast<float4*>(m)[i];
      float4 v4 = reinterpret_cast<float4*>(v)[i];
      float* wp = &w4.x;
      const float* gp = &g4.x;
      float* mp = &m4.x;
      float* vp = &v4.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float decay = (4 * i + j) < n_decay ? wd : 0.f;
        const float gj = gp[j] * scale;
        mp[j] = beta1 * mp[j] + (1.f - beta1) * gj;
        vp[j] = beta2 * vp[j] + (1.f - beta2) * gj * gj;
        const float den = sqrtf(vp[j] * inv_b2) + eps;
        const float step = den > 0.f ? (mp[j] * inv_b1) / den : 0.f;
        wp[j] = wp[j] * (1.f - lr * decay) - lr * step;
      }
      reinterpret_cast<float4*>(w)[i] = w4;
      reinterpret_cast<float4*>(m)[i] = m4;
      reinterpret_cast<float4*>(v)[i] = v4;
      if (wb) {
        uint2 packed;
        packed.x = pack_bf16x2(w4.x, w4.y);
        packed.y = pack_bf16x2(w4.z, w4.w);
        reinterpret_cast<uint2*>(wb)[i] = packed;
      }
    } else {
      for (size_t e = 4 * i; e < n; ++e) {
        const float decay = e < n_decay ? wd : 0.f;
        const float gj = g[e] * scale;
        m[e] = beta1 * m[e] + (1.f - beta1) * gj;
        v[e] = beta2 * v[e] + (1.f - beta2) * gj * gj;
        const float den = sqrtf(v[e] * inv_b2) + eps;
        const float step = den > 0.f ? (m[e] * inv_b1) / den : 0.f;
        w[e] = w[e] * (1.f - lr * decay) - lr * step;
        if (wb) wb[e] = f2bf(w[e]);
      }
    }
  }
}

__global__ void sgd_kernel(float* w, const float* g, __nv_bfloat16* wb,
                           size_t n, size_t n_decay, const float* hyper, float wd) {
  pdl_wait();
  const float lr = hyper[0], scale = hyper[3];
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float decay = i < n_decay ? wd : 0.f;
    w[i] = w[i] * (1.f - lr * decay) - lr * scale * g[i];
    if (wb) wb[i] = f2bf(w[i]);
  }
}

}  // namespace sj

using namespace sj;

extern "C" int sj_cross_entropy(const float* logits, int ld, const int32_t* targets, int rows, int vocab, float seed,
                                float* loss_rows, void* dlogits, int ld_d, double* loss_sum, double weight,
                                void* stream) {
  if (rows <= 0 || vocab <= 0 || ld < vocab || (dlogits && ld_d < vocab))
    return fail(SJ_ERR_SHAPE, "sj_cross_entropy: bad shape");
  const int warps = 8;
  launch(cross_entropy_kernel<__nv_bfloat16>, (rows + warps - 1) / warps, warps * 32, 0, as_stream(stream),
      logits, ld, targets, rows, vocab, seed, loss_rows, static_cast<__nv_bfloat16*>(dlogits), ld_d, loss_sum, weight);
  SJ_LAUNCH_CHECK("cross_entropy");
  return SJ_OK;
}

extern "C" int sj_cross_entropy_f32(const float* logits, int ld, const int32_t* targets, int rows, int vocab,
                                    float seed, float* loss_rows, float* dlogits, int ld_d, double* loss_sum,
                                    double weight, void* stream) {
  if (rows <= 0 || vocab <= 0 || ld < vocab || (dlogits && ld_d < vocab))
    return fail(SJ_ERR_SHAPE, "sj_cross_entropy_f32: bad shape");
  const int warps = 8;
  launch(cross_entropy_kernel<float>, (rows + warps - 1) / warps, warps * 32, 0, as_stream(stream), logits, ld,
         targets, rows, vocab, seed, loss_rows, dlogits, ld_d, loss_sum, weight);
  SJ_LAUNCH_CHECK("cross_entropy_f32");
  return SJ_OK;
}

extern "C" int sj_sumsq_partials(size_t n) {
  const size_t blocks = (n / 4 + kSumsqThreads - 1) / kSumsqThreads;
  const size_t cap = static_cast<size_t>(sm_count()) * 4;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

extern "C" int sj_grad_sumsq(const float* g, size_t n, double* partials, void* stream) {
  if (!aligned16(g)) return fail(SJ_ERR_ARGUMENT, "sj_grad_sumsq: gradient buffer must be 16-byte aligned");
  launch(grad_sumsq_kernel, sj_sumsq_partials(n), kSumsqThreads, 0, as_stream(stream), g, n, partials);
  SJ_LAUNCH_CHECK("grad_sumsq");
  return SJ_OK;
}

extern "C" int sj_optim_prepare(const double* partials, int n_partials, double* state, float* hyper,
                                float learning_rate, float min_learning_rate, int warmup_steps, int total_steps,
                                float beta1, float beta2, float clip_norm, int clip_enabled, float loss_scale,
                                void* stream) {
  if (n_partials <= 0 || !partials || !state || !hyper) return fail(SJ_ERR_ARGUMENT, "sj_optim_prepare: bad argument");
  launch(optim_prepare_kernel, 1, 256, 0, as_stream(stream), partials, n_partials, state, hyper, learning_rate,
                                                        min_learning_rate, warmup_steps, total_steps, beta1, beta2,
                                                        clip_norm, clip_enabled, loss_scale);
  SJ_LAUNCH_CHECK("optim_prepare");
  return SJ_OK;
}

extern "C" int sj_adamw(float* w, const float* g, float* m, float* v, void* w_bf16, size_t n, size_t n_decay,
                        const float* hyper, float beta1, float beta2, float eps, float weight_decay, void* stream) {
  if (!aligned16(w) || !aligned16(g) || !aligned16(m) || !aligned16(v) || (w_bf16 && (reinterpret_cast<uintptr_t>(w_bf16) & 7)))
    return fail(SJ_ERR_ARGUMENT, "sj_adamw: buffers must be 16-byte aligned (bf16 copy 8-byte)");
  const size_t work = (n + 3) / 4;
  size_t blocks = (work + 255) / 256;
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  launch(adamw_kernel, static_cast<unsigned>(blocks), 256, 0, as_stream(stream), 
      w, g, m, v, static_cast<__nv_bfloat16*>(w_bf16), n, n_decay, hyper, beta1, beta2, eps, weight_decay);
  SJ_LAUNCH_CHECK("adamw");
  return SJ_OK;
}

extern "C" int sj_sgd(float* w, const float* g, void* w_bf16, size_t n, size_t n_decay, const float* hyper,
                      float weight_decay, void* stream) {
  size_t blocks = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  launch(sgd_kernel, static_cast<unsigned>(blocks), 256, 0, as_stream(stream), w, g, static_cast<__nv_bfloat16*>(w_bf16),
                                                                          n, n_decay, hyper, weight_decay);
  SJ_LAUNCH_CHECK("sgd");
  return SJ_OK;
}
