// Kernels of the control-variate SGD trainer (crates/sejong-train/src/control_variate.rs:236-877):
// orthonormal bases of the predicted matrices, coefficient transport at a basis refresh, the
// augmented observation feature, the norm terms of the low-rank correction, the deferred update,
// and the binding of a corrected weight.  The reference's Triton kernels for the first three are in
// python/sejong_kernels/ops/hierarchy.py:254-397 (hierarchy_orthogonal_column,
// hierarchy_coefficient_transport, hierarchy_row_mean); the rest restate control_variate.rs
// arithmetic.  All f32, as in the reference; norm terms are summed in FP64 into the optimizer's
// partials so that the gradient norm (and its clipping) includes the correction.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {
namespace {

constexpr int kCvThreads = 512;

// Block-wide f32 sum (every thread receives it); `red` holds kCvThreads / 32 floats.
SJ_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += red[i];
  return t;
}

// Two passes of modified Gram-Schmidt of column `col` of Q against the columns before it
// (hierarchy.py:356-368: the dot of each pass uses the column as updated by the previous one).
SJ_DEVICE void reorthogonalize(float* q, int rows, int cols, int col, float* red) {
  for (int rep = 0; rep < 2; ++rep) {
    for (int prev = 0; prev < col; ++prev) {
      float part = 0.f;
      for (int r = threadIdx.x; r < rows; r += blockDim.x)
        part += q[static_cast<size_t>(r) * cols + col] * q[static_cast<size_t>(r) * cols + prev];
      const float dot = block_sum(part, red);
      for (int r = threadIdx.x; r < rows; r += blockDim.x)
        q[static_cast<size_t>(r) * cols + col] -= dot * q[static_cast<size_t>(r) * cols + prev];
      __syncthreads();
    }
  }
}

SJ_DEVICE float column_sumsq(const float* q, int rows, int cols, int col, float* red) {
  float part = 0.f;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const float v = q[static_cast<size_t>(r) * cols + col];
    part += v * v;
  }
  return block_sum(part, red);
}

// One CTA: Q = the columns of X [rows, cols] orthonormalised in order (hierarchy_orthogonal_column),
// then (gram != null) gram = Q^T Q [cols, cols].  A column whose residual norm is below 1e-20 is
// replaced by the unit vector at the row the earlier columns occupy least (the first such row),
// orthogonalised the same way.
__global__ void __launch_bounds__(kCvThreads) cv_orthonormalize_kernel(const float* x, float* q, float* gram,
                                                                      int rows, int cols) {
  pdl_wait();
  __shared__ float red[kCvThreads / 32];
  __shared__ float sbest[kCvThreads / 32];
  __shared__ int spivot[kCvThreads / 32];
  for (size_t i = threadIdx.x; i < static_cast<size_t>(rows) * cols; i += blockDim.x) q[i] = x[i];
  __syncthreads();
  for (int col = 0; col < cols; ++col) {
    reorthogonalize(q, rows, cols, col, red);
    float norm = column_sumsq(q, rows, cols, col, red);
    if (norm < 1.0e-20f) {
      // score = 1 - occupancy of the earlier columns; the lowest row of the highest score
      float best = -2.f;
      int pivot = rows;
      for (int r = threadIdx.x; r < rows; r += blockDim.x) {
        float occ = 0.f;
        for (int prev = 0; prev < col; ++prev) {
          const float b = q[static_cast<size_t>(r) * cols + prev];
          occ += b * b;
        }
        const float score = 1.f - occ;
        if (score > best) {  // rows ascend within a thread: strict > keeps the lowest row
          best = score;
          pivot = r;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int op = __shfl_xor_sync(0xffffffffu, pivot, o);
        if (ob > best || (ob == best && op < pivot)) {
          best = ob;
          pivot = op;
        }
      }
      __syncthreads();
      if ((threadIdx.x & 31) == 0) {
        sbest[threadIdx.x >> 5] = best;
        spivot[threadIdx.x >> 5] = pivot;
      }
      __syncthreads();
      best = sbest[0];
      pivot = spivot[0];
      for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
        if (sbest[w] > best || (sbest[w] == best && spivot[w] < pivot)) {
          best = sbest[w];
          pivot = spivot[w];
        }
      for (int r = threadIdx.x; r < rows; r += blockDim.x) q[static_cast<size_t>(r) * cols + col] = r == pivot ? 1.f : 0.f;
      __syncthreads();
      reorthogonalize(q, rows, cols, col, red);
      norm = column_sumsq(q, rows, cols, col, red);
    }
    const float inv = rsqrtf(norm);
    for (int r = threadIdx.x; r < rows; r += blockDim.x) q[static_cast<size_t>(r) * cols + col] *= inv;
    __syncthreads();
  }
  if (gram == nullptr) return;
  for (int ij = 0; ij < cols * cols; ++ij) {
    const int i = ij / cols, j = ij % cols;
    float part = 0.f;
    for (int r = threadIdx.x; r < rows; r += blockDim.x)
      part += q[static_cast<size_t>(r) * cols + i] * q[static_cast<size_t>(r) * cols + j];
    const float v = block_sum(part, red);
    if (threadIdx.x == 0) gram[ij] = v;
  }
}

// Y_f = L^T H_f R for each feature row f of H (rows of `ld` floats, the r x r coefficient at column
// `col0`), hierarchy_coefficient_transport's two passes in one CTA per feature.
__global__ void cv_transport_kernel(const float* h, int ld, int col0, const float* left, const float* right, float* y,
                                    int features, int r) {
  pdl_wait();
  extern __shared__ float sm[];
  float* sh = sm;            // r x r
  float* sl = sh + r * r;    // r x r
  float* sr = sl + r * r;    // r x r
  float* st = sr + r * r;    // r x r: L^T H
  const int f = blockIdx.x;
  if (f >= features) return;
  const float* hf = h + static_cast<size_t>(f) * ld + col0;
  for (int i = threadIdx.x; i < r * r; i += blockDim.x) {
    sh[i] = hf[i];
    sl[i] = left[i];
    sr[i] = right[i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < r * r; i += blockDim.x) {
    const int a = i / r, b = i % r;
    float acc = 0.f;
    for (int k = 0; k < r; ++k) acc = fmaf(sl[k * r + a], sh[k * r + b], acc);
    st[i] = acc;
  }
  __syncthreads();
  float* yf = y + static_cast<size_t>(f) * ld + col0;
  for (int i = threadIdx.x; i < r * r; i += blockDim.x) {
    const int a = i / r, b = i % r;
    float acc = 0.f;
    for (int k = 0; k < r; ++k) acc = fmaf(st[a * r + k], sr[k * r + b], acc);
    yf[i] = acc;
  }
}

// augmented_feature (control_variate.rs:375-387): out = [row_mean(E), row_mean(T), row_mean(E * T), 1]
// with E the encoded rows (cast to f32) and T the f32 embedding rows of the targets; column sums run
// over the rows in order (hierarchy_row_mean).
template <typename T>
__global__ void cv_feature_kernel(const T* enc, int ld, const float* emb, int emb_ld, const int* labels, int rows,
                                  int width, int vocab, float* out) {
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c == 0 && blockIdx.y == 0) out[3 * width] = 1.f;
  if (c >= width) return;
  float se = 0.f, st = 0.f, sx = 0.f;
  for (int r = 0; r < rows; ++r) {
    const float e = static_cast<float>(enc[static_cast<size_t>(r) * ld + c]);
    const int lab = labels[r];
    const float t = (lab >= 0 && lab < vocab) ? emb[static_cast<size_t>(lab) * emb_ld + c] : 0.f;
    if (lab < 0 || lab >= vocab) record_error(SJ_DEV_BAD_INDEX);
    se += e;
    st += t;
    sx += e * t;
  }
  const float inv = static_cast<float>(rows);
  out[c] = se / inv;
  out[width + c] = st / inv;
  out[2 * width + c] = sx / inv;
}
template <>
__global__ void cv_feature_kernel<__nv_bfloat16>(const __nv_bfloat16* enc, int ld, const float* emb, int emb_ld,
                                                  const int* labels, int rows, int width, int vocab, float* out) {
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c == 0) out[3 * width] = 1.f;
  if (c >= width) return;
  float se = 0.f, st = 0.f, sx = 0.f;
  for (int r = 0; r < rows; ++r) {
    const float e = bf2f(enc[static_cast<size_t>(r) * ld + c]);
    const int lab = labels[r];
    const float t = (lab >= 0 && lab < vocab) ? emb[static_cast<size_t>(lab) * emb_ld + c] : 0.f;
    if (lab < 0 || lab >= vocab) record_error(SJ_DEV_BAD_INDEX);
    se += e;
    st += t;
    sx += e * t;
  }
  const float inv = static_cast<float>(rows);
  out[c] = se / inv;
  out[width + c] = st / inv;
  out[2 * width + c] = sx / inv;
}

// out[j] = scale * (<X_j, GU_j X_j GV_j> + t_weight <T_j, X_j>) in FP64 per block j (correction_norm
// and the cross term of control_variate.rs:365-373,699-713); one CTA per block.
__global__ void cv_block_terms_kernel(const float* gu, const float* gv, const float* x, const float* t, double* out,
                                      int r, float t_weight, double scale) {
  pdl_wait();
  extern __shared__ float sm[];
  const int j = blockIdx.x;
  const size_t rr = static_cast<size_t>(r) * r;
  float* su = sm;
  float* sv = su + rr;
  float* sx = sv + rr;
  for (int i = threadIdx.x; i < static_cast<int>(rr); i += blockDim.x) {
    su[i] = gu[j * rr + i];
    sv[i] = gv[j * rr + i];
    sx[i] = x[j * rr + i];
  }
  __syncthreads();
  double acc = 0.0;
  for (int i = threadIdx.x; i < static_cast<int>(rr); i += blockDim.x) {
    const int a = i / r, b = i % r;
    // (GU X GV)[a, b] = sum_k sum_l GU[a, k] X[k, l] GV[l, b]
    float v = 0.f;
    for (int k = 0; k < r; ++k) {
      float row = 0.f;
      for (int l = 0; l < r; ++l) row = fmaf(sx[k * r + l], sv[l * r + b], row);
      v = fmaf(su[a * r + k], row, v);
    }
    acc += static_cast<double>(sx[i]) * v;
    if (t != nullptr) acc += static_cast<double>(t_weight) * t[j * rr + i] * sx[i];
  }
  acc = warp_sum(acc);
  __shared__ double red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w];
    out[j] = s * scale;
  }
}

// A = A (1 - lr wd) - lr clip delta (control_variate.rs:796-806), lr = hyper[0], clip = hyper[3] *
// loss_scale (hyper[3] is the clipping factor over the loss scale).
__global__ void cv_deferred_kernel(float* a, const float* delta, const float* hyper, float wd, float loss_scale,
                                   size_t n) {
  pdl_wait();
  const float lr = hyper[0], clip = hyper[3] * loss_scale;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float v = a[i];
    v = v + (-lr * wd) * v;
    a[i] = v + (-lr * clip) * delta[i];
  }
}

// wb = bf16(master + correction): the bound compute weight of a corrected matrix.
__global__ void cv_bind_kernel(const float* master, const float* corr, __nv_bfloat16* wb, size_t n) {
  pdl_wait();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    wb[i] = f2bf(master[i] + corr[i]);
}

// out [out_rows, cols] = 0 except out[map[i], :] = v[i, :] (a member's rows placed in its fused block).
__global__ void cv_scatter_rows_kernel(const float* v, int rows, int cols, const int* map, float* out, int out_rows) {
  pdl_wait();
  const size_t n = static_cast<size_t>(out_rows) * cols;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = 0.f;
}
__global__ void cv_scatter_rows_fill_kernel(const float* v, int rows, int cols, const int* map, float* out,
                                            int out_rows) {
  pdl_wait();
  const size_t n = static_cast<size_t>(rows) * cols;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i % cols);
    const int dst = map[r];
    if (dst >= 0 && dst < out_rows) out[static_cast<size_t>(dst) * cols + c] = v[i];
    else record_error(SJ_DEV_BAD_INDEX);
  }
}
// out[i, :] = alpha * v[map[i], :] for i < rows.
__global__ void cv_gather_rows_kernel(const float* v, int v_rows, int cols, const int* map, float* out, int rows,
                                      float alpha) {
  pdl_wait();
  const size_t n = static_cast<size_t>(rows) * cols;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i % cols);
    const int src = map[r];
    if (src >= 0 && src < v_rows) out[i] = alpha * v[static_cast<size_t>(src) * cols + c];
    else {
      out[i] = 0.f;
      record_error(SJ_DEV_BAD_INDEX);
    }
  }
}

// out [f, n] += alpha * x[f] * (p[j] - beta * t[j]) for j < n: the predictor gradient's outer
// product feature^T (prediction - target) (control_variate.rs:718-725), with the residual formed
// in place.
__global__ void cv_outer_kernel(const float* x, int f, const float* p, const float* t, float beta, int n, float alpha,
                                float* out) {
  pdl_wait();
  const size_t total = static_cast<size_t>(f) * n;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / n), j = static_cast<int>(i % n);
    const float resid = p[j] - beta * t[j];
    out[i] += alpha * x[row] * resid;
  }
}

int grid_of(size_t n) { return static_cast<int>(std::min<size_t>((n + 255) / 256, 148 * 8)); }

}  // namespace
}  // namespace sj

using namespace sj;

extern "C" int sj_cv_orthonormalize(const float* x, float* q, float* gram, int rows, int cols, void* stream) {
  if (rows <= 0 || cols <= 0 || cols > rows)
    return fail(SJ_ERR_SHAPE, "sj_cv_orthonormalize: rows %d, cols %d (need 0 < cols <= rows)", rows, cols);
  if (!x || !q || x == q) return fail(SJ_ERR_ARGUMENT, "sj_cv_orthonormalize: x and q distinct and non-null");
  launch(cv_orthonormalize_kernel, 1, kCvThreads, 0, as_stream(stream), x, q, gram, rows, cols);
  SJ_LAUNCH_CHECK("cv_orthonormalize");
  return SJ_OK;
}

extern "C" int sj_cv_transport(const float* h, int ld, int col0, const float* left, const float* right, float* y,
                               int features, int rank, void* stream) {
  if (features <= 0 || rank <= 0 || rank > 64 || ld < col0 + rank * rank)
    return fail(SJ_ERR_SHAPE, "sj_cv_transport: features %d, rank %d (<= 64), ld %d", features, rank, ld);
  if (!h || !left || !right || !y || h == y) return fail(SJ_ERR_ARGUMENT, "sj_cv_transport: operands");
  const int smem = 4 * rank * rank * 4;
  if (smem > 48 * 1024) return fail(SJ_ERR_CAPACITY, "sj_cv_transport: rank %d needs %d bytes", rank, smem);
  launch(cv_transport_kernel, features, 256, smem, as_stream(stream), h, ld, col0, left, right, y, features, rank);
  SJ_LAUNCH_CHECK("cv_transport");
  return SJ_OK;
}

extern "C" int sj_cv_feature(const void* encoded, int dtype, int ld, const float* embedding, int emb_ld,
                             const int* labels, int rows, int width, int vocab, float* out, void* stream) {
  if (rows <= 0 || width <= 0 || ld < width || emb_ld < width || vocab <= 0)
    return fail(SJ_ERR_SHAPE, "sj_cv_feature: rows %d width %d ld %d", rows, width, ld);
  if (!encoded || !embedding || !labels || !out) return fail(SJ_ERR_ARGUMENT, "sj_cv_feature: null");
  const dim3 grid((width + 127) / 128);
  if (dtype == SJ_BF16)
    launch(cv_feature_kernel<__nv_bfloat16>, grid, 128, 0, as_stream(stream),
           static_cast<const __nv_bfloat16*>(encoded), ld, embedding, emb_ld, labels, rows, width, vocab, out);
  else if (dtype == SJ_F32)
    launch(cv_feature_kernel<float>, grid, 128, 0, as_stream(stream), static_cast<const float*>(encoded), ld,
           embedding, emb_ld, labels, rows, width, vocab, out);
  else
    return fail(SJ_ERR_UNSUPPORTED, "sj_cv_feature: dtype %d", dtype);
  SJ_LAUNCH_CHECK("cv_feature");
  return SJ_OK;
}

extern "C" int sj_cv_block_terms(const float* gram_u, const float* gram_v, const float* x, const float* t,
                                 double* out, int blocks, int rank, float t_weight, double scale, void* stream) {
  if (blocks <= 0 || rank <= 0 || rank > 64) return fail(SJ_ERR_SHAPE, "sj_cv_block_terms: %d blocks, rank %d", blocks, rank);
  if (!gram_u || !gram_v || !x || !out) return fail(SJ_ERR_ARGUMENT, "sj_cv_block_terms: null");
  const int smem = 3 * rank * rank * 4;
  launch(cv_block_terms_kernel, blocks, 256, smem, as_stream(stream), gram_u, gram_v, x, t, out, rank, t_weight,
         scale);
  SJ_LAUNCH_CHECK("cv_block_terms");
  return SJ_OK;
}

extern "C" int sj_cv_deferred_update(float* a, const float* delta, const float* hyper, float weight_decay,
                                     float loss_scale, size_t n, void* stream) {
  if (!a || !delta || !hyper) return fail(SJ_ERR_ARGUMENT, "sj_cv_deferred_update: null");
  if (n == 0) return SJ_OK;
  launch(cv_deferred_kernel, grid_of(n), 256, 0, as_stream(stream), a, delta, hyper, weight_decay, loss_scale, n);
  SJ_LAUNCH_CHECK("cv_deferred_update");
  return SJ_OK;
}

extern "C" int sj_cv_bind(const float* master, const float* correction, void* wb, size_t n, void* stream) {
  if (!master || !correction || !wb) return fail(SJ_ERR_ARGUMENT, "sj_cv_bind: null");
  if (n == 0) return SJ_OK;
  launch(cv_bind_kernel, grid_of(n), 256, 0, as_stream(stream), master, correction,
         static_cast<__nv_bfloat16*>(wb), n);
  SJ_LAUNCH_CHECK("cv_bind");
  return SJ_OK;
}

extern "C" int sj_cv_scatter_rows(const float* v, int rows, int cols, const int* map, float* out, int out_rows,
                                  void* stream) {
  if (rows <= 0 || cols <= 0 || out_rows < rows) return fail(SJ_ERR_SHAPE, "sj_cv_scatter_rows: %d -> %d rows", rows, out_rows);
  if (!v || !map || !out) return fail(SJ_ERR_ARGUMENT, "sj_cv_scatter_rows: null");
  cudaStream_t s = as_stream(stream);
  launch(cv_scatter_rows_kernel, grid_of(static_cast<size_t>(out_rows) * cols), 256, 0, s, v, rows, cols, map, out,
         out_rows);
  launch(cv_scatter_rows_fill_kernel, grid_of(static_cast<size_t>(rows) * cols), 256, 0, s, v, rows, cols, map, out,
         out_rows);
  SJ_LAUNCH_CHECK("cv_scatter_rows");
  return SJ_OK;
}

extern "C" int sj_cv_gather_rows(const float* v, int v_rows, int cols, const int* map, float* out, int rows,
                                 float alpha, void* stream) {
  if (rows <= 0 || cols <= 0 || v_rows <= 0) return fail(SJ_ERR_SHAPE, "sj_cv_gather_rows: shape");
  if (!v || !map || !out) return fail(SJ_ERR_ARGUMENT, "sj_cv_gather_rows: null");
  launch(cv_gather_rows_kernel, grid_of(static_cast<size_t>(rows) * cols), 256, 0, as_stream(stream), v, v_rows, cols,
         map, out, rows, alpha);
  SJ_LAUNCH_CHECK("cv_gather_rows");
  return SJ_OK;
}

extern "C" int sj_cv_outer(const float* x, int f, const float* p, const float* t, float beta, int n, float alpha,
                           float* out, void* stream) {
  if (f <= 0 || n <= 0) return fail(SJ_ERR_SHAPE, "sj_cv_outer: %d x %d", f, n);
  if (!x || !p || !t || !out) return fail(SJ_ERR_ARGUMENT, "sj_cv_outer: null");
  launch(cv_outer_kernel, grid_of(static_cast<size_t>(f) * n), 256, 0, as_stream(stream), x, f, p, t, beta, n, alpha,
         out);
  SJ_LAUNCH_CHECK("cv_outer");
  return SJ_OK;
}
