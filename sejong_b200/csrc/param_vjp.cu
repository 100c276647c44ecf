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

// The draws themselves are sequential by definition and run on thread 0; the initialisation of
// the permutation scratch (shared memory), of the row map and the expansion of the selected
// blocks into rows use the whole block.
__global__ void __launch_bounds__(256) param_indices_kernel(unsigned long long* rng_state, int a, int b, int nb,
                                                            int s, int r, int group, int32_t* columns,
                                                            int32_t* rows, int32_t* row_map) {
  pdl_wait();
  extern __shared__ int32_t scratch[];  // [b + nb] permutation, then [s] chosen blocks
  int32_t* chosen = scratch + b + nb;
  for (int i = threadIdx.x; i < b + nb; i += blockDim.x) scratch[i] = i < b ? i : i - b;
  for (int i = threadIdx.x; i < a; i += blockDim.x) row_map[i] = -1;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t outer = *rng_state;
    uint64_t state = splitmix_next(outer);  // seed = rng.next_u64(); the draw's generator starts there
    *rng_state = outer;
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
      chosen[i] = value;
    }
  }
  __syncthreads();
  for (int position = threadIdx.x; position < s * group; position += blockDim.x) {
    const int index = chosen[position / group] * group + position % group;
    rows[position] = index < a ? index : -1;
    if (index < a) row_map[index] = position;
  }
}

// Physical column of logical column c of a member: plain, or the second ("up") half of a
// gate/up weight whose columns are interleaved in blocks of `interleave`.
SJ_DEVICE int member_column(int c, int interleave) {
  return interleave > 0 ? (c / interleave) * 2 * interleave + interleave + (c % interleave) : c;
}

// wsel[f, j] = w[f, column j] in f32: the r donor columns of the weight, gathered once.
__global__ void param_wsel_kernel(const __nv_bfloat16* w, int ldw, int interleave,
                                  const int32_t* columns, int a, int r, float* wsel) {
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= a * r) return;
  const int f = idx / r, j = idx % r;
  wsel[idx] = bf2f(w[static_cast<size_t>(f) * ldw + member_column(columns[j], interleave)]);
}

// Donor columns ys = x wsel [n, R] and their FP64 Gram matrix.  A CTA takes 64 rows: lane l owns
// rows l and l + 32, warp w a slice of the features; the 8 slices are summed in shared memory,
// then the CTA's 64 x R tile adds its R x R Gram contribution.
constexpr int kYsRows = 64;
template <int R>
__global__ void __launch_bounds__(256) param_ys_gram_kernel(const __nv_bfloat16* x, int ldx, int n,
                                                            int a, const float* wsel_g, int r,
                                                            float* ys, double* gram) {
  pdl_wait();
  extern __shared__ __align__(16) float smem[];
  float* wsel = smem;                        // [a][R] (columns >= r zero)
  float* part = smem + a * R;                // [8][kYsRows][R]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int idx = threadIdx.x; idx < a * R; idx += blockDim.x) {
    const int f = idx / R, j = idx % R;
    wsel[idx] = j < r ? wsel_g[f * r + j] : 0.f;
  }
  __syncthreads();
  const int slice = ((a + 63) / 64) * 8;     // features per warp, a multiple of 8
  const int f_begin = warp * slice, f_end = min(a, f_begin + slice);
  const int row0 = blockIdx.x * kYsRows + lane, row1 = row0 + 32;
  float acc0[R], acc1[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc0[j] = acc1[j] = 0.f;
  const __nv_bfloat16* x0 = x + static_cast<size_t>(min(row0, n - 1)) * ldx;
  const __nv_bfloat16* x1 = x + static_cast<size_t>(min(row1, n - 1)) * ldx;
  for (int f = f_begin; f < f_end; f += 8) {
    const uint4 p0 = *reinterpret_cast<const uint4*>(x0 + f);
    const uint4 p1 = *reinterpret_cast<const uint4*>(x1 + f);
    const uint32_t w0[4] = {p0.x, p0.y, p0.z, p0.w}, w1[4] = {p1.x, p1.y, p1.z, p1.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 a0 = unpack_bf16x2(w0[h]), a1 = unpack_bf16x2(w1[h]);
      const float4* ws0 = reinterpret_cast<const float4*>(wsel + (f + 2 * h) * R);
      const float4* ws1 = reinterpret_cast<const float4*>(wsel + (f + 2 * h + 1) * R);
#pragma unroll
      for (int j4 = 0; j4 < R / 4; ++j4) {
        const float4 u = ws0[j4], v = ws1[j4];
        acc0[4 * j4 + 0] = fmaf(a0.x, u.x, fmaf(a0.y, v.x, acc0[4 * j4 + 0]));
        acc0[4 * j4 + 1] = fmaf(a0.x, u.y, fmaf(a0.y, v.y, acc0[4 * j4 + 1]));
        acc0[4 * j4 + 2] = fmaf(a0.x, u.z, fmaf(a0.y, v.z, acc0[4 * j4 + 2]));
        acc0[4 * j4 + 3] = fmaf(a0.x, u.w, fmaf(a0.y, v.w, acc0[4 * j4 + 3]));
        acc1[4 * j4 + 0] = fmaf(a1.x, u.x, fmaf(a1.y, v.x, acc1[4 * j4 + 0]));
        acc1[4 * j4 + 1] = fmaf(a1.x, u.y, fmaf(a1.y, v.y, acc1[4 * j4 + 1]));
        acc1[4 * j4 + 2] = fmaf(a1.x, u.z, fmaf(a1.y, v.z, acc1[4 * j4 + 2]));
        acc1[4 * j4 + 3] = fmaf(a1.x, u.w, fmaf(a1.y, v.w, acc1[4 * j4 + 3]));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < R; ++j) {
    part[(warp * kYsRows + lane) * R + j] = acc0[j];
    part[(warp * kYsRows + lane + 32) * R + j] = acc1[j];
  }
  __syncthreads();
  // slice sums -> ys (global) and the CTA's tile (kept in part[0])
  for (int idx = threadIdx.x; idx < kYsRows * R; idx += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += part[w * kYsRows * R + idx];
    const int row = blockIdx.x * kYsRows + idx / R, j = idx % R;
    if (row >= n) v = 0.f;
    part[idx] = v;
    if (row < n && j < r) ys[static_cast<size_t>(row) * r + j] = v;
  }
  __syncthreads();
  for (int pair = threadIdx.x; pair < r * r; pair += blockDim.x) {
    const int i = pair / r, j = pair % r;
    double g0 = 0.0, g1 = 0.0;
    for (int t = 0; t < kYsRows; t += 2) {
      g0 += static_cast<double>(part[t * R + i]) * static_cast<double>(part[t * R + j]);
      g1 += static_cast<double>(part[(t + 1) * R + i]) * static_cast<double>(part[(t + 1) * R + j]);
    }
    atomicAdd(&gram[pair], g0 + g1);
  }
}

SJ_DEVICE double shfl_d(double v, int src) { return __shfl_sync(0xffffffffu, v, src); }

// CGS2 in coefficient space on one warp.  Column c of T gives q_c = Ys t_c.  Lane k holds row k of
// the Gram matrix and row k of T; lane i also keeps column i of T.  For the current column, u
// starts as e_c; each pass takes all projections coef_i = q_i . v = t_i^T (G u) from the same v and
// then subtracts them (classical Gram-Schmidt), twice; |v|^2 = u^T G u.  t[k * r + c] on output.
__global__ void __launch_bounds__(32) param_cgs2_kernel(const double* gram, int r, float eps,
                                                        double* t) {
  pdl_wait();
  const int lane = threadIdx.x;
  double grow[kMaxRank], trow[kMaxRank], tcol[kMaxRank];
#pragma unroll
  for (int l = 0; l < kMaxRank; ++l) {
    grow[l] = (lane < r && l < r) ? gram[lane * r + l] : 0.0;
    trow[l] = 0.0;
    tcol[l] = 0.0;
  }
  const double e2 = static_cast<double>(eps) * static_cast<double>(eps);
  for (int cur = 0; cur < r; ++cur) {
    double u = lane == cur ? 1.0 : 0.0;
    double diagonal = 0.0;                     // G[lane][cur]; lane cur's copy is |y_cur|^2
#pragma unroll
    for (int l = 0; l < kMaxRank; ++l)
      if (l == cur) diagonal = grow[l];
    const double original = shfl_d(diagonal, cur);
    for (int pass = 0; pass < 2; ++pass) {
      double gu = 0.0;                         // (G u)[lane]
#pragma unroll
      for (int l = 0; l < kMaxRank; ++l) gu = fma(grow[l], shfl_d(u, l), gu);
      double coef = 0.0;                       // coef[lane] = t_lane . (G u), lane < cur
#pragma unroll
      for (int k = 0; k < kMaxRank; ++k) coef = fma(tcol[k], shfl_d(gu, k), coef);
      if (lane >= cur) coef = 0.0;
      double update = 0.0;                     // sum_i coef_i T[lane][i]
#pragma unroll
      for (int i = 0; i < kMaxRank; ++i) update = fma(shfl_d(coef, i), trow[i], update);
      u -= update;
    }
    double gu = 0.0;
#pragma unroll
    for (int l = 0; l < kMaxRank; ++l) gu = fma(grow[l], shfl_d(u, l), gu);
    double magnitude = lane < r ? u * gu : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) magnitude += __shfl_xor_sync(0xffffffffu, magnitude, o);
    const double inverse = magnitude > e2 * original ? 1.0 / sqrt(magnitude) : 0.0;
    const double value = lane < r ? u * inverse : 0.0;
#pragma unroll
    for (int i = 0; i < kMaxRank; ++i)
      if (i == cur) trow[i] = value;
#pragma unroll
    for (int k = 0; k < kMaxRank; ++k) {
      const double vk = shfl_d(value, k);
      if (lane == cur) tcol[k] = vk;
    }
  }
  if (lane < r) {
#pragma unroll
    for (int c = 0; c < kMaxRank; ++c)
      if (c < r) t[lane * r + c] = trow[c];
  }
}

// q = ys T (T upper triangular), thread per row.
template <int R>
__global__ void __launch_bounds__(256) param_apply_t_kernel(const float* ys,
                                                            const double* t, int n, int r,
                                                            float* q) {
  pdl_wait();
  __shared__ float ts[R * R];
  for (int i = threadIdx.x; i < R * R; i += blockDim.x) {
    const int k = i / R, j = i % R;
    ts[i] = (k < r && j < r) ? static_cast<float>(t[k * r + j]) : 0.f;
  }
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  float yv[R];
#pragma unroll
  for (int k = 0; k < R; ++k) yv[k] = k < r ? ys[static_cast<size_t>(row) * r + k] : 0.f;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    if (j >= r) break;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k <= j; ++k) acc = fmaf(yv[k], ts[k * R + j], acc);
    q[static_cast<size_t>(row) * r + j] = acc;
  }
}

// left[a, r] += x^T q.  A CTA covers 64 features (lane l: features 2l, 2l + 1) and up to
// 256 tokens (128 at rank > 16), split over its 8 warps.  The CTA's q rows are first copied to shared memory
// (one coalesced read), so the inner loop is one x load per token and warp plus shared-memory
// broadcasts; the warps' partial sums meet in shared memory and the CTA adds its 64 x r block with
// one atomic per value.
template <int R>
constexpr int left_tokens() { return R <= 16 ? 256 : 128; }  // keeps q + partial sums within 48 KB
template <int R>
__global__ void __launch_bounds__(256) param_left_kernel(const __nv_bfloat16* x, int ldx, int n, int a,
                                                         const float* q, int r,
                                                         float* left) {
  pdl_wait();
  constexpr int kTokens = left_tokens<R>();
  __shared__ __align__(16) float qs[kTokens * R];
  __shared__ float red[8][32][R];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.y * 64 + 2 * lane;
  const int t_begin = blockIdx.x * kTokens;
  const int tokens = min(kTokens, n - t_begin);
  if (r == R) {
    // q rows are R floats: the block's tokens x R floats are one contiguous run, staged as 16-byte
    // vectors whose loads are all issued before the shared-memory stores
    constexpr int kVec = kTokens * R / 4 / 256;  // vectors per thread (4 for both ranks)
    const float4* src = reinterpret_cast<const float4*>(q + static_cast<size_t>(t_begin) * R);
    float4* dst = reinterpret_cast<float4*>(qs);
    const int n4 = tokens * R / 4;
    float4 v[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int i = threadIdx.x + u * 256;
      v[u] = i < n4 ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int i = threadIdx.x + u * 256;
      if (i < n4) dst[i] = v[u];
    }
  } else {
    for (int idx = threadIdx.x; idx < tokens * R; idx += blockDim.x) {
      const int t = idx / R, j = idx % R;
      qs[idx] = j < r ? q[static_cast<size_t>(t_begin + t) * r + j] : 0.f;
    }
  }
  __syncthreads();
  float acc0[R], acc1[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc0[j] = acc1[j] = 0.f;
  if (f0 < a) {
    // each warp owns kTokens / 8 consecutive tokens of the block and issues all their loads first
    constexpr int kU = kTokens / 8;
    const int t0 = warp * kU;
    {
      uint32_t xw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        xw[u] = t0 + u < tokens
                    ? *reinterpret_cast<const uint32_t*>(x + static_cast<size_t>(t_begin + t0 + u) * ldx + f0)
                    : 0u;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const float2 xv = unpack_bf16x2(xw[u]);   // zero past the last token
        const float4* q4 = reinterpret_cast<const float4*>(qs + (t0 + u < tokens ? t0 + u : 0) * R);
#pragma unroll
        for (int j4 = 0; j4 < R / 4; ++j4) {
          const float4 qv = q4[j4];
          acc0[4 * j4] = fmaf(xv.x, qv.x, acc0[4 * j4]);
          acc0[4 * j4 + 1] = fmaf(xv.x, qv.y, acc0[4 * j4 + 1]);
          acc0[4 * j4 + 2] = fmaf(xv.x, qv.z, acc0[4 * j4 + 2]);
          acc0[4 * j4 + 3] = fmaf(xv.x, qv.w, acc0[4 * j4 + 3]);
          acc1[4 * j4] = fmaf(xv.y, qv.x, acc1[4 * j4]);
          acc1[4 * j4 + 1] = fmaf(xv.y, qv.y, acc1[4 * j4 + 1]);
          acc1[4 * j4 + 2] = fmaf(xv.y, qv.z, acc1[4 * j4 + 2]);
          acc1[4 * j4 + 3] = fmaf(xv.y, qv.w, acc1[4 * j4 + 3]);
        }
      }
    }
  }
  // two rounds (even, then odd features) through an [8 warps][32 lanes][R] buffer
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int j = 0; j < R; ++j) red[warp][lane][j] = h == 0 ? acc0[j] : acc1[j];
    __syncthreads();
    for (int idx = threadIdx.x; idx < 32 * R; idx += blockDim.x) {
      const int fl = idx / R, j = idx % R;
      const int f = blockIdx.y * 64 + 2 * fl + h;
      if (f < a && j < r) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += red[w][fl][j];
        atomicAdd(&left[static_cast<size_t>(f) * r + j], v);
      }
    }
    __syncthreads();
  }
}

// E [(r + k), n] bf16.  blockIdx.y < ceil(k / 32): 32 residual rows r + pos of E,
// (x[:, rows[pos]] - q left[rows[pos]]^T) * inverse (zero where rows[pos] < 0); the last y-slice
// writes rows [0, r) = q^T.  Thread per token; the slice's left rows sit in shared memory.
template <int R>
__global__ void __launch_bounds__(128) param_e_kernel(const __nv_bfloat16* x, int ldx, int n,
                                                      const float* q, int r,
                                                      const float* left,
                                                      const int32_t* rows, int k, float inverse,
                                                      __nv_bfloat16* e) {
  pdl_wait();
  __shared__ __align__(16) float ls[32][R];
  __shared__ int rs[32];
  __shared__ int contiguous;
  const int token = blockIdx.x * blockDim.x + threadIdx.x;
  const int slices = (k + 31) / 32;
  const bool head = blockIdx.y == slices;
  if (!head) {
    for (int idx = threadIdx.x; idx < 32 * R; idx += blockDim.x) {
      const int p = idx / R, j = idx % R, pos = blockIdx.y * 32 + p;
      const int row = pos < k ? rows[pos] : -1;
      ls[p][j] = (row >= 0 && j < r) ? left[static_cast<size_t>(row) * r + j] : 0.f;
      if (j == 0) rs[p] = pos < k ? row : -2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      bool ok = rs[0] >= 0 && (rs[0] & 7) == 0 && (ldx & 7) == 0;
      for (int p = 1; p < 32 && ok; ++p) ok = rs[p] == rs[0] + p;
      contiguous = ok;
    }
    __syncthreads();
  }
  if (token >= n) return;
  float qv[R];
#pragma unroll
  for (int j = 0; j < R; ++j) qv[j] = j < r ? q[static_cast<size_t>(token) * r + j] : 0.f;
  if (head) {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (j < r) e[static_cast<size_t>(j) * n + token] = f2bf(qv[j]);
    return;
  }
  const __nv_bfloat16* xr = x + static_cast<size_t>(token) * ldx;
  // gather the slice's 32 x values first (independent loads), then form the residuals
  float xs[32];
  if (contiguous) {   // 64 contiguous bytes of the token's row: four 16-byte loads
    const uint4* src = reinterpret_cast<const uint4*>(xr + rs[0]);
#pragma unroll
    for (int v4 = 0; v4 < 4; ++v4) {
      const uint4 w = src[v4];
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(words[h]);
        xs[8 * v4 + 2 * h] = f.x;
        xs[8 * v4 + 2 * h + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int p = 0; p < 32; ++p) {
      const int row = rs[p];
      xs[p] = row >= 0 ? bf2f(xr[row]) : 0.f;
    }
  }
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    const int row = rs[p];
    if (row == -2) break;
    float v = 0.f;
    if (row >= 0) {
      float proj = 0.f;
      const float4* l4 = reinterpret_cast<const float4*>(ls[p]);
#pragma unroll
      for (int j4 = 0; j4 < R / 4; ++j4) {
        const float4 lv = l4[j4];
        proj = fmaf(qv[4 * j4], lv.x, proj);
        proj = fmaf(qv[4 * j4 + 1], lv.y, proj);
        proj = fmaf(qv[4 * j4 + 2], lv.z, proj);
        proj = fmaf(qv[4 * j4 + 3], lv.w, proj);
      }
      v = (xs[p] - proj) * inverse;
    }
    e[static_cast<size_t>(r + blockIdx.y * 32 + p) * n + token] = f2bf(v);
  }
}

// g[i, j] (+)= sum_k left[i, k] coeff[k, j] + (row_map[i] >= 0 ? coeff[r + row_map[i], j] : 0),
// j < b (coeff and g offset by the caller to the member's first column).  A CTA owns kMatRows rows x
// 128 columns: each thread keeps its column's r coefficients in registers and walks the rows.
constexpr int kMatRows = 8;
template <int R>
__global__ void __launch_bounds__(128) param_materialize_kernel(const float* left,
                                                                const float* coeff, int ldc,
                                                                const int32_t* row_map, int a, int b,
                                                                int r, float* g, int ldg,
                                                                int accumulate) {
  pdl_wait();
  __shared__ float ls[kMatRows][R];
  __shared__ int ms[kMatRows];
  const int i0 = blockIdx.y * kMatRows;
  for (int idx = threadIdx.x; idx < kMatRows * R; idx += blockDim.x) {
    const int i = idx / R, kk = idx % R;
    ls[i][kk] = (i0 + i < a && kk < r) ? left[static_cast<size_t>(i0 + i) * r + kk] : 0.f;
    if (kk == 0) ms[i] = i0 + i < a ? row_map[i0 + i] : -1;
  }
  __syncthreads();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= b) return;
  float c[R];
#pragma unroll
  for (int kk = 0; kk < R; ++kk) c[kk] = kk < r ? coeff[static_cast<size_t>(kk) * ldc + j] : 0.f;
  // all loads of the row tile first (g and the selected-row tails), then the arithmetic
  float gv[kMatRows], tv[kMatRows];
#pragma unroll
  for (int i = 0; i < kMatRows; ++i) {
    const bool valid = i0 + i < a;
    gv[i] = (valid && accumulate) ? g[static_cast<size_t>(i0 + i) * ldg + j] : 0.f;
    const int m = valid ? ms[i] : -1;
    tv[i] = m >= 0 ? coeff[static_cast<size_t>(r + m) * ldc + j] : 0.f;
  }
#pragma unroll
  for (int i = 0; i < kMatRows; ++i) {
    if (i0 + i >= a) break;
    float v = tv[i];
#pragma unroll
    for (int kk = 0; kk < R; ++kk) v = fmaf(ls[i][kk], c[kk], v);
    g[static_cast<size_t>(i0 + i) * ldg + j] = gv[i] + v;
  }
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

extern "C" int sj_param_indices(uint64_t* rng_state, int a, int b, int nb, int s, int r, int group,
                                int32_t* columns, int32_t* rows, int32_t* row_map, void* stream) {
  if (!rng_state || a < 0 || b < 0 || nb < 0 || s < 0 || r < 0 || group <= 0 || r > b || s > nb)
    return fail(SJ_ERR_ARGUMENT, "sj_param_indices: bad sizes a=%d b=%d nb=%d s=%d r=%d", a, b, nb, s, r);
  if ((r && !columns) || (s && !rows) || (a && !row_map))
    return fail(SJ_ERR_ARGUMENT, "sj_param_indices: null output");
  const size_t smem = (static_cast<size_t>(b) + nb + s) * sizeof(int32_t);
  if (smem > 48 * 1024) return fail(SJ_ERR_SHAPE, "sj_param_indices: b + nb + s = %zu above 12288", smem / 4);
  launch(param_indices_kernel, 1, 256, smem, as_stream(stream), reinterpret_cast<unsigned long long*>(rng_state), a, b,
                                                            nb, s, r, group, columns, rows, row_map);
  SJ_LAUNCH_CHECK("param_indices");
  return SJ_OK;
}

namespace {

// 8-byte aligned pieces of the basis workspace: Gram and T (f64), gathered weights and ys (f32).
struct BasisWorkspace {
  double* gram;
  double* t;
  float* wsel;
  float* ys;
};

BasisWorkspace basis_workspace(void* base, int n, int a, int r) {
  BasisWorkspace w;
  w.gram = static_cast<double*>(base);
  w.t = w.gram + r * r;
  w.wsel = reinterpret_cast<float*>(w.t + r * r);
  w.ys = w.wsel + ((static_cast<size_t>(a) * r + 3) & ~size_t(3));
  (void)n;
  return w;
}

template <int R>
int launch_basis(const __nv_bfloat16* x, int ldx, int n, int a, const __nv_bfloat16* w, int ldw, int interleave,
                 const int32_t* columns, int r, float eps, float* q, const BasisWorkspace& ws, cudaStream_t s) {
  static KernelAttrOnce attr_once;  // one per template instance
  const int attr_rc = ensure_max_smem(attr_once, reinterpret_cast<const void*>(param_ys_gram_kernel<R>), 200 * 1024,
                                      "param_ys_gram shared-memory attribute");
  if (attr_rc != SJ_OK) return attr_rc;
  const size_t smem = (static_cast<size_t>(a) * R + 8 * kYsRows * R) * sizeof(float);
  if (smem > 200 * 1024) return fail(SJ_ERR_SHAPE, "sj_param_basis: a = %d too wide for rank %d", a, r);
  const int zs = zero_async(ws.gram, sizeof(double) * r * r, s);
  if (zs != SJ_OK) return zs;
  launch(param_wsel_kernel, (a * r + 255) / 256, 256, 0, s, w, ldw, interleave, columns, a, r, ws.wsel);
  SJ_LAUNCH_CHECK("param_wsel");
  launch(param_ys_gram_kernel<R>, (n + kYsRows - 1) / kYsRows, 256, smem, s, x, ldx, n, a, ws.wsel, r, ws.ys, ws.gram);
  SJ_LAUNCH_CHECK("param_ys_gram");
  launch(param_cgs2_kernel, 1, 32, 0, s, ws.gram, r, eps, ws.t);
  SJ_LAUNCH_CHECK("param_cgs2");
  launch(param_apply_t_kernel<R>, (n + 255) / 256, 256, 0, s, ws.ys, ws.t, n, r, q);
  SJ_LAUNCH_CHECK("param_apply_t");
  return SJ_OK;
}

}  // namespace

extern "C" size_t sj_param_basis_workspace(int n, int a, int r) {
  if (n <= 0 || a <= 0 || r <= 0) return 0;
  return 2 * static_cast<size_t>(r) * r * sizeof(double) +
         (((static_cast<size_t>(a) * r + 3) & ~size_t(3)) + static_cast<size_t>(n) * r) * sizeof(float);
}

extern "C" int sj_param_basis(const void* x, int ldx, int n, int a, const void* w, int ldw, int interleave,
                              const int32_t* columns, int r, float eps, float* q, void* workspace, void* stream) {
  if (!x || !w || !columns || !q || !workspace || n <= 0 || a <= 0 || r <= 0 || r > kMaxRank)
    return fail(SJ_ERR_ARGUMENT, "sj_param_basis: bad arguments (1 <= rank <= %d)", kMaxRank);
  if (a % 8 || ldx % 8 || !aligned16(x) || !aligned16(workspace))
    return fail(SJ_ERR_ARGUMENT, "sj_param_basis: x rows and the workspace must be 16-byte aligned, a % 8 == 0");
  const BasisWorkspace ws = basis_workspace(workspace, n, a, r);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  if (r <= 16) return launch_basis<16>(xb, ldx, n, a, wb, ldw, interleave, columns, r, eps, q, ws, as_stream(stream));
  return launch_basis<32>(xb, ldx, n, a, wb, ldw, interleave, columns, r, eps, q, ws, as_stream(stream));
}

namespace {

template <int R>
int launch_prepare(const __nv_bfloat16* x, int ldx, int n, int a, const float* q, int r, const int32_t* rows, int k,
                   float inverse, float* left, __nv_bfloat16* e, cudaStream_t s) {
  const int zs = zero_async(left, sizeof(float) * a * r, s);
  if (zs != SJ_OK) return zs;
  const dim3 grid_left((n + left_tokens<R>() - 1) / left_tokens<R>(), (a + 63) / 64);
  launch(param_left_kernel<R>, grid_left, 256, 0, s, x, ldx, n, a, q, r, left);
  SJ_LAUNCH_CHECK("param_left");
  const dim3 grid_e((n + 127) / 128, (k + 31) / 32 + 1);
  launch(param_e_kernel<R>, grid_e, 128, 0, s, x, ldx, n, q, r, left, rows, k, inverse, e);
  SJ_LAUNCH_CHECK("param_e");
  return SJ_OK;
}

template <int R>
int launch_materialize(const float* left, const float* coeff, int ldc, const int32_t* row_map, int a, int b, int r,
                       float* g, int ldg, int accumulate, cudaStream_t s) {
  const dim3 grid((b + 127) / 128, (a + kMatRows - 1) / kMatRows);
  launch(param_materialize_kernel<R>, grid, 128, 0, s, left, coeff, ldc, row_map, a, b, r, g, ldg, accumulate);
  SJ_LAUNCH_CHECK("param_materialize");
  return SJ_OK;
}

}  // namespace

extern "C" int sj_param_prepare(const void* x, int ldx, int n, int a, const float* q, int r, const int32_t* rows,
                                int k, float inverse, float* left, void* e, void* stream) {
  if (!x || !q || !left || !e || (k && !rows) || n <= 0 || a <= 0 || r <= 0 || r > kMaxRank || k < 0)
    return fail(SJ_ERR_ARGUMENT, "sj_param_prepare: bad arguments");
  if (a % 2 || ldx % 2 || (reinterpret_cast<uintptr_t>(x) & 3) || (reinterpret_cast<uintptr_t>(q) & 15))
    return fail(SJ_ERR_ARGUMENT, "sj_param_prepare: x rows must hold feature pairs (a, ldx even), q 16-byte aligned");
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* eb = static_cast<__nv_bfloat16*>(e);
  if (r <= 16) return launch_prepare<16>(xb, ldx, n, a, q, r, rows, k, inverse, left, eb, as_stream(stream));
  return launch_prepare<32>(xb, ldx, n, a, q, r, rows, k, inverse, left, eb, as_stream(stream));
}

extern "C" int sj_param_materialize(const float* left, const float* coeff, int ldc, const int32_t* row_map, int a,
                                    int b, int r, float* g, int ldg, int accumulate, void* stream) {
  if (!left || !coeff || !row_map || !g || a <= 0 || b <= 0 || r <= 0 || r > kMaxRank || ldc < b || ldg < b)
    return fail(SJ_ERR_ARGUMENT, "sj_param_materialize: bad arguments");
  if ((a + kMatRows - 1) / kMatRows > 65535) return fail(SJ_ERR_SHAPE, "sj_param_materialize: a=%d too large", a);
  if (r <= 16) return launch_materialize<16>(left, coeff, ldc, row_map, a, b, r, g, ldg, accumulate, as_stream(stream));
  return launch_materialize<32>(left, coeff, ldc, row_map, a, b, r, g, ldg, accumulate, as_stream(stream));
}
