// Parameter VJP: a weight gradient as low-rank factors from a forward basis plus the exact
// gradient of a random selection of feature rows.
//
// Restates crates/sejong-gpu/src/parameter_vjp.rs:152-321 and python/sejong_kernels/ops/
// parameter.py:25-244.  For a weight gradient dW = X^T dY (X [n, a], dY [n, b]) the reference
// forms an orthonormal basis Q [n, r] of r selected columns of a donor output Y = X W_donor and
//   left = X^T Q [a, r],  E = [Q^T ; (X - Q left^T)[:, selected rows]^T * NB/S]  [(r+k), n],
//   (right ; tail) = E dY,  G = left right + scatterRows(tail).
// Work split on the B200:
//   * sj_param_indices: the single-program partial Fisher-Yates of parameter.py:25-62, bit-exact.
//     Its seed is one next_u64 of a device-resident SplitMix64 state (the host draw of
//     parameter_vjp.rs:190), so a training step that uses it never synchronises with the host.
//   * sj_param_basis: the selected donor columns recomputed as X W[:, columns] (so the donor may be
//     a projection whose stored output already had RoPE applied), their FP64 Gram matrix, and the
//     CGS2 of parameter.py:65-129 carried out in coefficient space: Q = Ys T with T upper
//     triangular, built by the same two classical projection passes and the same small-norm cutoff
//     (|v|^2 <= eps^2 |y|^2 gives a zero column).  In exact arithmetic this is the reference's CGS2
//     and, unlike column-by-column CGS2 over n rows, every row-sized pass is fully parallel.
//   * sj_param_prepare: left (f32) and E (bf16: the A operand of the coefficient GEMM, which runs
//     on sj_gemm with split-K).
//   * sj_param_materialize: G (+)= left right + scatterRows(tail) into the flat f32 gradient.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace sj {

constexpr int kMaxRank = 32;

SJ_DEVICE uint64_t splitmix_next(uint64_t& state) {
  state += 0x9e3779b97f4a7c15ull;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Rejection with threshold (2^64 - size) mod size, as crates/sejong-core/src/lib.rs:609-618.
SJ_DEVICE uint64_t splitmix_index(uint64_t& state, uint64_t size) {
  const uint64_t threshold = (0ull - size) % size;
  while (true) {
    const uint64_t x = splitmix_next(state);
    if (x >= threshold) return x % size;
  }
}

// One thread: the draws are sequential by definition.  scratch holds b + nb ints.
__global__ void param_indices_kernel(unsigned long long* rng_state, int a, int b, int nb, int s, int r, int group,
                                     int32_t* scratch, int32_t* columns, int32_t* rows, int32_t* row_map) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  uint64_t outer = *rng_state;
  uint64_t state = splitmix_next(outer);  // seed = rng.next_u64(); the kernel's generator starts there
  *rng_state = outer;
  for (int i = 0; i < b; ++i) scratch[i] = i;
  for (int i = 0; i < nb; ++i) scratch[b + i] = i;
  for (int i = 0; i < a; ++i) row_map[i] = -1;
  for (int i = 0; i < r; ++i) {
    const int j = i + static_cast<int>(splitmix_index(state, static_cast<uint64_t>(b - i)));
    const int value = scratch[j];
    scratch[j] = scratch[i];
    scratch[i] = value;
    columns[i] = value;
  }
  for (int i = 0; i < s; ++i) {
    const int j = i + static_cast<int>(splitmix_index(state, static_cast<uint64_t>(nb - i)));
    const int value = scratch[b + j];
    scratch[b + j] = scratch[b + i];
    scratch[b + i] = value;
    for (int o = 0; o < group; ++o) {
      const int index = value * group + o, position = i * group + o;
      rows[position] = index < a ? index : -1;
      if (index < a) row_map[index] = position;
    }
  }
}

// Physical column of logical column c of a member: plain, or the second ("up") half of a
// gate/up weight whose columns are interleaved in blocks of `interleave`.
SJ_DEVICE int member_column(int c, int interleave) {
  return interleave > 0 ? (c / interleave) * 2 * interleave + interleave + (c % interleave) : c;
}

// ys[row, j] = sum_f x[row, f] w[f, col_j]; the r selected weight columns are staged in shared
// memory as f32 [a][r]; one thread per row, 16-byte loads of x.
__global__ void __launch_bounds__(256) param_ys_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int n, int a,
                                                       const __nv_bfloat16* __restrict__ w, int ldw, int interleave,
                                                       const int32_t* __restrict__ columns, int r,
                                                       float* __restrict__ ys) {
  extern __shared__ float wsel[];  // [a][r]
  for (int idx = threadIdx.x; idx < a * r; idx += blockDim.x) {
    const int f = idx / r, j = idx % r;
    wsel[idx] = bf2f(w[static_cast<size_t>(f) * ldw + member_column(columns[j], interleave)]);
  }
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  float acc[kMaxRank];
#pragma unroll
  for (int j = 0; j < kMaxRank; ++j) acc[j] = 0.f;
  const __nv_bfloat16* xr = x + static_cast<size_t>(row) * ldx;
  for (int f0 = 0; f0 < a; f0 += 8) {
    const uint4 packed = *reinterpret_cast<const uint4*>(xr + f0);
    const uint32_t words[4] = {packed.x, packed.y, packed.z, packed.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 xv = unpack_bf16x2(words[h]);
      const float* w0 = wsel + (f0 + 2 * h) * r;
      const float* w1 = w0 + r;
#pragma unroll
      for (int j = 0; j < kMaxRank; ++j)
        if (j < r) acc[j] = fmaf(xv.x, w0[j], fmaf(xv.y, w1[j], acc[j]));
    }
  }
#pragma unroll
  for (int j = 0; j < kMaxRank; ++j)
    if (j < r) ys[static_cast<size_t>(row) * r + j] = acc[j];
}

// gram[i, j] += sum over this CTA's 256 rows of ys[row, i] ys[row, j], in FP64.
constexpr int kGramRows = 256;
__global__ void __launch_bounds__(256) param_gram_kernel(const float* __restrict__ ys, int n, int r,
                                                         double* __restrict__ gram) {
  __shared__ float tile[kGramRows * kMaxRank];
  const int row0 = blockIdx.x * kGramRows;
  const int rows = min(kGramRows, n - row0);
  for (int idx = threadIdx.x; idx < rows * r; idx += blockDim.x) tile[idx] = ys[static_cast<size_t>(row0) * r + idx];
  __syncthreads();
  for (int pair = threadIdx.x; pair < r * r; pair += blockDim.x) {
    const int i = pair / r, j = pair % r;
    double acc = 0.0;
    for (int t = 0; t < rows; ++t) acc += static_cast<double>(tile[t * r + i]) * static_cast<double>(tile[t * r + j]);
    atomicAdd(&gram[pair], acc);
  }
}

// CGS2 in coefficient space.  Column c of T (t[k * r + c]) gives q_c = Ys t_c.  For the current
// column u starts as e_c; each pass takes all projections coef_i = q_i . v = t_i^T G u from the same
// v and then subtracts them (classical Gram-Schmidt), twice; |v|^2 = u^T G u.
__global__ void param_cgs2_kernel(const double* __restrict__ gram, int r, float eps, double* __restrict__ t) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int i = 0; i < r * r; ++i) t[i] = 0.0;
  const double e = static_cast<double>(eps);
  for (int cur = 0; cur < r; ++cur) {
    double u[kMaxRank], gu[kMaxRank], coef[kMaxRank];
    for (int k = 0; k < r; ++k) u[k] = k == cur ? 1.0 : 0.0;
    const double original = gram[cur * r + cur];
    for (int pass = 0; pass < 2; ++pass) {
      for (int k = 0; k < r; ++k) {
        double acc = 0.0;
        for (int l = 0; l < r; ++l) acc += gram[k * r + l] * u[l];
        gu[k] = acc;
      }
      for (int i = 0; i < cur; ++i) {
        double acc = 0.0;
        for (int k = 0; k < r; ++k) acc += t[k * r + i] * gu[k];
        coef[i] = acc;
      }
      for (int i = 0; i < cur; ++i)
        for (int k = 0; k < r; ++k) u[k] -= coef[i] * t[k * r + i];
    }
    double magnitude = 0.0;
    for (int k = 0; k < r; ++k) {
      double acc = 0.0;
      for (int l = 0; l < r; ++l) acc += gram[k * r + l] * u[l];
      magnitude += u[k] * acc;
    }
    const double inverse = magnitude > e * e * original ? 1.0 / sqrt(magnitude) : 0.0;
    for (int k = 0; k < r; ++k) t[k * r + cur] = u[k] * inverse;
  }
}

// q = ys T (T upper triangular).
__global__ void __launch_bounds__(256) param_apply_t_kernel(const float* __restrict__ ys,
                                                            const double* __restrict__ t, int n, int r,
                                                            float* __restrict__ q) {
  __shared__ float ts[kMaxRank * kMaxRank];
  for (int i = threadIdx.x; i < r * r; i += blockDim.x) ts[i] = static_cast<float>(t[i]);
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  float yv[kMaxRank];
#pragma unroll
  for (int k = 0; k < kMaxRank; ++k) yv[k] = k < r ? ys[static_cast<size_t>(row) * r + k] : 0.f;
  for (int j = 0; j < r; ++j) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxRank; ++k)
      if (k <= j) acc = fmaf(yv[k], ts[k * r + j], acc);
    q[static_cast<size_t>(row) * r + j] = acc;
  }
}

// left[a, r] += x^T q over a chunk of kPrepRows rows; thread f owns features f, f + 256, ...
constexpr int kPrepRows = 128;
__global__ void __launch_bounds__(256) param_left_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int n, int a,
                                                         const float* __restrict__ q, int r,
                                                         float* __restrict__ left) {
  __shared__ float qs[kPrepRows * kMaxRank];
  const int row0 = blockIdx.x * kPrepRows;
  const int rows = min(kPrepRows, n - row0);
  for (int i = threadIdx.x; i < rows * r; i += blockDim.x) qs[i] = q[static_cast<size_t>(row0) * r + i];
  __syncthreads();
  for (int f = threadIdx.x; f < a; f += blockDim.x) {
    float acc[kMaxRank];
#pragma unroll
    for (int j = 0; j < kMaxRank; ++j) acc[j] = 0.f;
    for (int t = 0; t < rows; ++t) {
      const float xv = bf2f(x[static_cast<size_t>(row0 + t) * ldx + f]);
#pragma unroll
      for (int j = 0; j < kMaxRank; ++j)
        if (j < r) acc[j] = fmaf(xv, qs[t * r + j], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < kMaxRank; ++j)
      if (j < r) atomicAdd(&left[static_cast<size_t>(f) * r + j], acc[j]);
  }
}

// E [(r + k), n] bf16: rows [0, r) = q^T; row r + pos = (x[:, rows[pos]] - q left[rows[pos]]^T) * inverse,
// zero where rows[pos] < 0 (a padded block past the last feature).
__global__ void __launch_bounds__(256) param_e_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int n,
                                                      const float* __restrict__ q, int r,
                                                      const float* __restrict__ left,
                                                      const int32_t* __restrict__ rows, int k, float inverse,
                                                      __nv_bfloat16* __restrict__ e) {
  const int token = blockIdx.x * blockDim.x + threadIdx.x;
  if (token >= n) return;
  float qv[kMaxRank];
#pragma unroll
  for (int j = 0; j < kMaxRank; ++j) {
    qv[j] = j < r ? q[static_cast<size_t>(token) * r + j] : 0.f;
    if (j < r) e[static_cast<size_t>(j) * n + token] = f2bf(qv[j]);
  }
  const __nv_bfloat16* xr = x + static_cast<size_t>(token) * ldx;
  for (int pos = 0; pos < k; ++pos) {
    const int row = rows[pos];
    float v = 0.f;
    if (row >= 0) {
      float proj = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxRank; ++j)
        if (j < r) proj = fmaf(qv[j], left[static_cast<size_t>(row) * r + j], proj);
      v = (bf2f(xr[row]) - proj) * inverse;
    }
    e[static_cast<size_t>(r + pos) * n + token] = f2bf(v);
  }
}

// g[i, j] (+)= sum_k left[i, k] coeff[k, j] + (row_map[i] >= 0 ? coeff[r + row_map[i], j] : 0)
// over columns [0, b) of coeff and g (both offset by the caller to the member's first column).
__global__ void __launch_bounds__(256) param_materialize_kernel(const float* __restrict__ left,
                                                                const float* __restrict__ coeff, int ldc,
                                                                const int32_t* __restrict__ row_map, int a, int b,
                                                                int r, float* __restrict__ g, int ldg,
                                                                int accumulate) {
  __shared__ float lrow[kMaxRank];
  __shared__ int mapped;
  const int i = blockIdx.y;
  if (threadIdx.x < r) lrow[threadIdx.x] = left[static_cast<size_t>(i) * r + threadIdx.x];
  if (threadIdx.x == 0) mapped = row_map[i];
  __syncthreads();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= b) return;
  float v = 0.f;
  for (int k = 0; k < r; ++k) v = fmaf(lrow[k], coeff[static_cast<size_t>(k) * ldc + j], v);
  if (mapped >= 0) v += coeff[static_cast<size_t>(r + mapped) * ldc + j];
  float* dst = g + static_cast<size_t>(i) * ldg + j;
  *dst = accumulate ? *dst + v : v;
}

}  // namespace sj

using namespace sj;

extern "C" int sj_param_indices_host(uint64_t seed, int a, int b, int nb, int s, int r, int group, int32_t* columns,
                                     int32_t* rows, int32_t* row_map) {
  if (a < 0 || b < 0 || nb < 0 || s < 0 || r < 0 || group <= 0 || r > b || s > nb)
    return fail(SJ_ERR_ARGUMENT, "sj_param_indices_host: bad sizes a=%d b=%d nb=%d s=%d r=%d", a, b, nb, s, r);
  if ((r && !columns) || (s && !rows) || (a && !row_map))
    return fail(SJ_ERR_ARGUMENT, "sj_param_indices_host: null output");
  std::vector<int32_t> scratch(static_cast<size_t>(b) + nb);
  for (int i = 0; i < b; ++i) scratch[i] = i;
  for (int i = 0; i < nb; ++i) scratch[b + i] = i;
  for (int i = 0; i < a; ++i) row_map[i] = -1;
  uint64_t state = seed;
  for (int i = 0; i < r; ++i) {
    const int j = i + static_cast<int>(sj_rng_index(&state, static_cast<uint64_t>(b - i)));
    std::swap(scratch[i], scratch[j]);
    columns[i] = scratch[i];
  }
  for (int i = 0; i < s; ++i) {
    const int j = i + static_cast<int>(sj_rng_index(&state, static_cast<uint64_t>(nb - i)));
    std::swap(scratch[b + i], scratch[b + j]);
    const int value = scratch[b + i];
    for (int o = 0; o < group; ++o) {
      const int index = value * group + o, position = i * group + o;
      rows[position] = index < a ? index : -1;
      if (index < a) row_map[index] = position;
    }
  }
  return SJ_OK;
}

extern "C" int sj_param_indices(uint64_t* rng_state, int a, int b, int nb, int s, int r, int group, int32_t* scratch,
                                int32_t* columns, int32_t* rows, int32_t* row_map, void* stream) {
  if (!rng_state || !scratch || a < 0 || b < 0 || nb < 0 || s < 0 || r < 0 || group <= 0 || r > b || s > nb)
    return fail(SJ_ERR_ARGUMENT, "sj_param_indices: bad sizes a=%d b=%d nb=%d s=%d r=%d", a, b, nb, s, r);
  if ((r && !columns) || (s && !rows) || (a && !row_map))
    return fail(SJ_ERR_ARGUMENT, "sj_param_indices: null output");
  param_indices_kernel<<<1, 32, 0, as_stream(stream)>>>(reinterpret_cast<unsigned long long*>(rng_state), a, b, nb,
                                                        s, r, group, scratch, columns, rows, row_map);
  SJ_LAUNCH_CHECK("param_indices");
  return SJ_OK;
}

extern "C" size_t sj_param_basis_workspace(int n, int r) {
  if (n <= 0 || r <= 0) return 0;
  return 2 * static_cast<size_t>(r) * r * sizeof(double) + static_cast<size_t>(n) * r * sizeof(float);
}

extern "C" int sj_param_basis(const void* x, int ldx, int n, int a, const void* w, int ldw, int interleave,
                              const int32_t* columns, int r, float eps, float* q, void* workspace, void* stream) {
  if (!x || !w || !columns || !q || !workspace || n <= 0 || a <= 0 || r <= 0 || r > kMaxRank)
    return fail(SJ_ERR_ARGUMENT, "sj_param_basis: bad arguments (1 <= rank <= %d)", kMaxRank);
  if (a % 8 || ldx % 8 || !aligned16(x) || (reinterpret_cast<uintptr_t>(workspace) & 7))
    return fail(SJ_ERR_ARGUMENT, "sj_param_basis: x rows must be 16-byte aligned multiples of 8 features");
  const size_t smem = static_cast<size_t>(a) * r * sizeof(float);
  if (smem > 200 * 1024) return fail(SJ_ERR_SHAPE, "sj_param_basis: a*r = %d too large", a * r);
  cudaStream_t s = as_stream(stream);
  double* gram = static_cast<double*>(workspace);
  double* t = gram + r * r;
  float* ys = reinterpret_cast<float*>(t + r * r);
  // the shared-memory opt-in is per device; set once, on the first call (make it before any capture)
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(param_ys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return cuda_check(e, "param_ys shared-memory attribute");
    configured_device = dev;
  }
  cudaError_t e = cudaMemsetAsync(gram, 0, sizeof(double) * r * r, s);
  if (e != cudaSuccess) return cuda_check(e, "param_basis memset");
  const int blocks = (n + 255) / 256;
  param_ys_kernel<<<blocks, 256, smem, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, n, a,
                                            static_cast<const __nv_bfloat16*>(w), ldw, interleave, columns, r, ys);
  SJ_LAUNCH_CHECK("param_ys");
  param_gram_kernel<<<(n + kGramRows - 1) / kGramRows, 256, 0, s>>>(ys, n, r, gram);
  SJ_LAUNCH_CHECK("param_gram");
  param_cgs2_kernel<<<1, 32, 0, s>>>(gram, r, eps, t);
  SJ_LAUNCH_CHECK("param_cgs2");
  param_apply_t_kernel<<<blocks, 256, 0, s>>>(ys, t, n, r, q);
  SJ_LAUNCH_CHECK("param_apply_t");
  return SJ_OK;
}

extern "C" int sj_param_prepare(const void* x, int ldx, int n, int a, const float* q, int r, const int32_t* rows,
                                int k, float inverse, float* left, void* e, void* stream) {
  if (!x || !q || !left || !e || (k && !rows) || n <= 0 || a <= 0 || r <= 0 || r > kMaxRank || k < 0)
    return fail(SJ_ERR_ARGUMENT, "sj_param_prepare: bad arguments");
  cudaStream_t s = as_stream(stream);
  cudaError_t err = cudaMemsetAsync(left, 0, sizeof(float) * a * r, s);
  if (err != cudaSuccess) return cuda_check(err, "param_prepare memset");
  param_left_kernel<<<(n + kPrepRows - 1) / kPrepRows, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, n, a,
                                                                     q, r, left);
  SJ_LAUNCH_CHECK("param_left");
  param_e_kernel<<<(n + 255) / 256, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, n, q, r, left, rows, k,
                                                 inverse, static_cast<__nv_bfloat16*>(e));
  SJ_LAUNCH_CHECK("param_e");
  return SJ_OK;
}

extern "C" int sj_param_materialize(const float* left, const float* coeff, int ldc, const int32_t* row_map, int a,
                                    int b, int r, float* g, int ldg, int accumulate, void* stream) {
  if (!left || !coeff || !row_map || !g || a <= 0 || b <= 0 || r <= 0 || r > kMaxRank || ldc < b || ldg < b)
    return fail(SJ_ERR_ARGUMENT, "sj_param_materialize: bad arguments");
  if (a > 65535) return fail(SJ_ERR_SHAPE, "sj_param_materialize: a=%d above 65535", a);
  const dim3 grid((b + 255) / 256, a);
  param_materialize_kernel<<<grid, 256, 0, as_stream(stream)>>>(left, coeff, ldc, row_map, a, b, r, g, ldg,
                                                                accumulate);
  SJ_LAUNCH_CHECK("param_materialize");
  return SJ_OK;
}
