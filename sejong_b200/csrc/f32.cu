// The f32 arithmetic variant of the byte-model step ("one training step in
// fp32", the reference's F32 precision, crates/sejong-core/src/lib.rs DType::F32): the same ops as
// the bf16 path with every activation, operand and gradient in f32 and f32 FMA accumulation.
//
//   sgemm_kernel      C = A B with the bf16 GEMM's epilogues (STORE, ACCUM, RESIDUAL, ROPE,
//                     SWIGLU; gemm.cu) -- kernels.py:23-39 / projection.py in f32.  CUDA-core FMA:
//                     the tensor cores' f32-input kind (tf32) keeps 10 mantissa bits, which is not
//                     the reference's f32 arithmetic.  128 x 128 (or, for grids under two waves,
//                     64 x 64) output tiles, 8 x 8 (4 x 4) per thread, double-buffered 8-deep K
//                     slices in shared memory; accumulating products with few tiles split K.
//   attn_f32_fwd      causal GQA with optional window, online softmax, LSE (natural log)
//                     (hierarchy.py:7-39), one CTA per (64-query block, head, sequence).
//   attn_f32_delta / attn_f32_bwd / attn_f32_dq_finish   the backward (hierarchy.py:43-104): Delta =
//                     rowsum(dO O); per (64-key block, kv head) recompute P, dP, dS for every query
//                     head of the group, dK / dV in registers (inverse RoPE on dK at the store), dQ
//                     accumulated with f32 atomics, then rotated back by the finish kernel.
//   swiglu_bwd_f32    lib.rs:711-733 on the interleaved gate/up layout of the SWIGLU epilogue.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {
constexpr int kSBM = 128, kSBN = 128, kSBK = 8, kSThreads = 256;
constexpr int kAB = 64, kAD = 64, kAThreads = 256, kAPad = kAD + 1;

struct SgemmParams {
  const float* a;
  const float* b;
  float* c;
  float* aux;          // RESIDUAL: the residual (ld_aux); SWIGLU: h [M, N/2] (ld_aux)
  const float* rope;   // ROPE: [rope_t, 64] (cos, sin) pairs
  int lda, ldb, ldc, ld_aux;
  int a_trans, b_trans;
  int m, n, k;
  int epilogue;
  int rope_cols, rope_t;
};

SJ_DEVICE float silu_f32(float g) { return g / (1.0f + expf(-g)); }
}  // namespace

// Tile BM x BN (128 x 128 or 64 x 64), 256 threads as 16 x 16: thread (tx, ty) owns the rows
// (i >> 2) * BM/2 + ty * 4 + (i & 3) and the columns (j >> 2) * BN/2 + tx * 4 + (j & 3).  With
// gridDim.z > 1 (ACCUM only) CTA z reduces the K slice [z * kslice, (z + 1) * kslice) and adds its
// partial product with f32 atomics.
template <int BM, int BN>
__global__ void __launch_bounds__(kSThreads) sgemm_kernel(SgemmParams p, int kslice) {
  pdl_wait();
  constexpr int TM = BM / 16, TN = BN / 16;
  constexpr int LA = BM * kSBK / kSThreads, LB = BN * kSBK / kSThreads;  // elements each thread stages
  __shared__ __align__(16) float As[2][kSBK][BM + 4];
  __shared__ __align__(16) float Bs[2][kSBK][BN + 4];
  const int t = threadIdx.x, tx = t % 16, ty = t / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int kb = blockIdx.z * kslice, ke = min(p.k, kb + kslice);
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  float ra[LA], rb[LB];
  auto load = [&](int k0) {
#pragma unroll
    for (int j = 0; j < LA; ++j) {
      const int e = t + kSThreads * j;
      int mm, kk;
      if (p.a_trans) { mm = e % BM; kk = e / BM; } else { kk = e % kSBK; mm = e / kSBK; }
      const int gm = m0 + mm, gk = k0 + kk;
      ra[j] = (gm < p.m && gk < ke) ? (p.a_trans ? p.a[static_cast<size_t>(gk) * p.lda + gm]
                                                 : p.a[static_cast<size_t>(gm) * p.lda + gk])
                                    : 0.f;
    }
#pragma unroll
    for (int j = 0; j < LB; ++j) {
      const int e = t + kSThreads * j;
      int nn, kk;
      if (p.b_trans) { kk = e % kSBK; nn = e / kSBK; } else { nn = e % BN; kk = e / BN; }
      const int gn = n0 + nn, gk = k0 + kk;
      rb[j] = (gn < p.n && gk < ke) ? (p.b_trans ? p.b[static_cast<size_t>(gn) * p.ldb + gk]
                                                 : p.b[static_cast<size_t>(gk) * p.ldb + gn])
                                    : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int j = 0; j < LA; ++j) {
      const int e = t + kSThreads * j;
      if (p.a_trans) As[buf][e / BM][e % BM] = ra[j]; else As[buf][e % kSBK][e / kSBK] = ra[j];
    }
#pragma unroll
    for (int j = 0; j < LB; ++j) {
      const int e = t + kSThreads * j;
      if (p.b_trans) Bs[buf][e % kSBK][e / kSBK] = rb[j]; else Bs[buf][e / BN][e % BN] = rb[j];
    }
  };
  const int ktiles = ke > kb ? (ke - kb + kSBK - 1) / kSBK : 0;
  if (ktiles > 0) {
    load(kb);
    store(0);
  }
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load(kb + (kt + 1) * kSBK);
#pragma unroll
    for (int kk = 0; kk < kSBK; ++kk) {
      float av[TM], bv[TN];
#pragma unroll
      for (int h = 0; h < TM / 4; ++h) {
        const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][kk][h * (BM / 2) + ty * 4]);
        av[4 * h] = a4.x; av[4 * h + 1] = a4.y; av[4 * h + 2] = a4.z; av[4 * h + 3] = a4.w;
      }
#pragma unroll
      for (int h = 0; h < TN / 4; ++h) {
        const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][kk][h * (BN / 2) + tx * 4]);
        bv[4 * h] = b4.x; bv[4 * h + 1] = b4.y; bv[4 * h + 2] = b4.z; bv[4 * h + 3] = b4.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store(buf ^ 1);
    __syncthreads();
  }
  const bool split = gridDim.z > 1;
  // epilogue
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int gr = m0 + (i >> 2) * (BM / 2) + ty * 4 + (i & 3);
    if (gr >= p.m) continue;
#pragma unroll
    for (int j = 0; j < TN; j += 2) {
      const int gc = n0 + (j >> 2) * (BN / 2) + tx * 4 + (j & 3);  // even: (gc, gc + 1) is a RoPE pair
      if (gc >= p.n) continue;
      float v0 = acc[i][j], v1 = acc[i][j + 1];
      float* c = p.c + static_cast<size_t>(gr) * p.ldc + gc;
      if (p.epilogue == SJ_EPI_ROPE && gc < p.rope_cols) {
        const float* tab = p.rope + static_cast<size_t>(gr % p.rope_t) * 64 + (gc % 64);
        const float cs = tab[0], sn = tab[1];
        const float a = v0, b = v1;
        v0 = a * cs - b * sn;
        v1 = a * sn + b * cs;
      } else if (p.epilogue == SJ_EPI_RESIDUAL) {
        const float* r = p.aux + static_cast<size_t>(gr) * p.ld_aux + gc;
        v0 += r[0];
        if (gc + 1 < p.n) v1 += r[1];
      }
      if (split) {
        atomicAdd(c, v0);
        if (gc + 1 < p.n) atomicAdd(c + 1, v1);
      } else if (p.epilogue == SJ_EPI_ACCUM) {
        c[0] += v0;
        if (gc + 1 < p.n) c[1] += v1;
      } else {
        c[0] = v0;
        if (gc + 1 < p.n) c[1] = v1;
      }
    }
  }
  if (p.epilogue == SJ_EPI_SWIGLU) {
    // the tile's blocks of (16 gate | 16 up) columns are in global memory now: h = silu(g) * u
    __syncthreads();
    for (int e = t; e < BM * (BN / 2); e += kSThreads) {
      const int r = e / (BN / 2), f = e % (BN / 2);
      const int gr = m0 + r, gcol = n0 + (f / 16) * 32 + (f % 16);
      if (gr >= p.m || gcol + 16 >= p.n) continue;
      const float g = p.c[static_cast<size_t>(gr) * p.ldc + gcol];
      const float u = p.c[static_cast<size_t>(gr) * p.ldc + gcol + 16];
      p.aux[static_cast<size_t>(gr) * p.ld_aux + n0 / 2 + f] = silu_f32(g) * u;
    }
  }
}

// dg = dh u s (1 + g (1 - s)), du = dh g s with s = sigmoid(g); thread per feature.
__global__ void swiglu_bwd_f32_kernel(const float* gu, const float* dh, float* dgu, int rows, int f) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * f) return;
  const int row = static_cast<int>(i / f), x = static_cast<int>(i % f);
  const size_t gc = static_cast<size_t>(row) * 2 * f + (x / 16) * 32 + (x % 16);
  const float g = gu[gc], u = gu[gc + 16], d = dh[static_cast<size_t>(row) * f + x];
  const float s = 1.0f / (1.0f + expf(-g));
  dgu[gc] = d * u * s * (1.0f + g * (1.0f - s));
  dgu[gc + 16] = d * g * s;
}

namespace {
// key `key` is visible from query `query` (causal, optional window)
SJ_DEVICE bool visible(int query, int key, int window) {
  return key <= query && (window <= 0 || key >= query + 1 - window);
}
// thread c0 (0..3) of a row owns the head dims {8 jj + 2 c0 + e : jj < 8, e < 2}: RoPE pairs stay local
SJ_DEVICE int own_dim(int c0, int q) { return 8 * (q >> 1) + 2 * c0 + (q & 1); }
}  // namespace

// grid (query blocks, hq, batch); dynamic shared memory 4 * 64 * 65 floats
__global__ void __launch_bounds__(kAThreads) attn_f32_fwd_kernel(const float* q, int ldq, const float* k, int ldk,
                                                                 const float* v, int ldv, float* o, int ldo,
                                                                 float* lse, int t, int hq, int hk, int window) {
  pdl_wait();
  extern __shared__ float sm[];
  float* Qs = sm;
  float* Ks = Qs + kAB * kAPad;
  float* Vs = Ks + kAB * kAPad;
  float* Ps = Vs + kAB * kAPad;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (hq / hk);
  const int tid = threadIdx.x, r = tid >> 2, c0 = tid & 3;
  const int q0 = qb * kAB;
  const size_t base = static_cast<size_t>(b) * t;
  const float scale = rsqrtf(static_cast<float>(kAD));
  for (int e = tid; e < kAB * kAD; e += kAThreads) {
    const int rr = e / kAD, d = e % kAD;
    Qs[rr * kAPad + d] = q0 + rr < t ? q[(base + q0 + rr) * ldq + h * kAD + d] : 0.f;
  }
  const int query = q0 + r;
  float m_i = -INFINITY, l_i = 0.f, acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
  const int kb_hi = min((q0 + kAB - 1) / kAB, (t - 1) / kAB);
  const int kb_lo = window > 0 ? max(0, q0 + 1 - window) / kAB : 0;
  for (int kb = kb_lo; kb <= kb_hi; ++kb) {
    __syncthreads();
    for (int e = tid; e < kAB * kAD; e += kAThreads) {
      const int rr = e / kAD, d = e % kAD, key = kb * kAB + rr;
      Ks[rr * kAPad + d] = key < t ? k[(base + key) * ldk + kvh * kAD + d] : 0.f;
      Vs[rr * kAPad + d] = key < t ? v[(base + key) * ldv + kvh * kAD + d] : 0.f;
    }
    __syncthreads();
    float s[16], mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int c = c0 + 4 * j, key = kb * kAB + c;
      float dot = 0.f;
      for (int d = 0; d < kAD; ++d) dot = fmaf(Qs[r * kAPad + d], Ks[c * kAPad + d], dot);
      s[j] = (query < t && key < t && visible(query, key, window)) ? dot * scale : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_i, mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float pj = m_new == -INFINITY ? 0.f : expf(s[j] - m_new);
      Ps[r * kAPad + c0 + 4 * j] = pj;
      sum += pj;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float alpha = m_i == -INFINITY ? 0.f : expf(m_i - m_new);
    l_i = l_i * alpha + sum;
    m_i = m_new;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = own_dim(c0, j);
      float a = acc[j] * alpha;
      for (int c = 0; c < kAB; ++c) a = fmaf(Ps[r * kAPad + c], Vs[c * kAPad + d], a);
      acc[j] = a;
    }
  }
  if (query < t) {
    const float inv = l_i > 0.f ? 1.0f / l_i : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) o[(base + query) * ldo + h * kAD + own_dim(c0, j)] = acc[j] * inv;
    if (c0 == 0) lse[(base + query) * hq + h] = m_i + logf(l_i);
  }
}

// Delta[row, h] = sum_d dO O; zeroes the dq accumulator (the q columns of dqkv).  Warp per (row, h).
__global__ void attn_f32_delta_kernel(const float* o, int ldo, const float* dout, int lddo, float* delta, float* dq,
                                      int lddq, int rows, int hq) {
  pdl_wait();
  const size_t w = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<size_t>(rows) * hq) return;
  const int row = static_cast<int>(w / hq), h = static_cast<int>(w % hq);
  float s = 0.f;
  for (int d = lane; d < kAD; d += 32) {
    s = fmaf(o[static_cast<size_t>(row) * ldo + h * kAD + d], dout[static_cast<size_t>(row) * lddo + h * kAD + d], s);
    dq[static_cast<size_t>(row) * lddq + h * kAD + d] = 0.f;
  }
  s = warp_sum(s);
  if (lane == 0) delta[w] = s;
}

// grid (key blocks, hk, batch); dynamic shared memory 5 * 64 * 65 + 128 floats
__global__ void __launch_bounds__(kAThreads) attn_f32_bwd_kernel(
    const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, const float* lse, const float* delta,
    const float* dout, int lddo, float* dq, int lddq, float* dk, int lddk, float* dv, int lddv, int t, int hq, int hk,
    int window, const float* rope) {
  pdl_wait();
  extern __shared__ float sm[];
  float* Ks = sm;
  float* Vs = Ks + kAB * kAPad;
  float* Qs = Vs + kAB * kAPad;
  float* dOs = Qs + kAB * kAPad;
  float* Ss = dOs + kAB * kAPad;  // P^T, then dS^T: [key][query]
  float* Ls = Ss + kAB * kAPad;   // LSE of the query block
  float* Ds = Ls + kAB;           // Delta of the query block
  const int kb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = hq / hk;
  const int tid = threadIdx.x, r = tid >> 2, c0 = tid & 3;
  const int k0 = kb * kAB;
  const size_t base = static_cast<size_t>(b) * t;
  const float scale = rsqrtf(static_cast<float>(kAD));
  for (int e = tid; e < kAB * kAD; e += kAThreads) {
    const int rr = e / kAD, d = e % kAD, key = k0 + rr;
    Ks[rr * kAPad + d] = key < t ? k[(base + key) * ldk + kvh * kAD + d] : 0.f;
    Vs[rr * kAPad + d] = key < t ? v[(base + key) * ldv + kvh * kAD + d] : 0.f;
  }
  float dkr[16], dvr[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) dkr[j] = dvr[j] = 0.f;
  const int key = k0 + r;
  const int qb_last = window > 0 ? min((t - 1) / kAB, (k0 + kAB - 1 + window - 1) / kAB) : (t - 1) / kAB;
  for (int gi = 0; gi < group; ++gi) {
    const int h = kvh * group + gi;
    for (int qb = kb; qb <= qb_last; ++qb) {
      const int q0 = qb * kAB;
      __syncthreads();
      for (int e = tid; e < kAB * kAD; e += kAThreads) {
        const int rr = e / kAD, d = e % kAD, query = q0 + rr;
        Qs[rr * kAPad + d] = query < t ? q[(base + query) * ldq + h * kAD + d] : 0.f;
        dOs[rr * kAPad + d] = query < t ? dout[(base + query) * lddo + h * kAD + d] : 0.f;
      }
      if (tid < kAB) {
        const int query = q0 + tid;
        Ls[tid] = query < t ? lse[(base + query) * hq + h] : 0.f;
        Ds[tid] = query < t ? delta[(base + query) * hq + h] : 0.f;
      }
      __syncthreads();
      // thread (key r, queries c0 + 4 j): P^T and dS^T
      float pj[16], dsj[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = c0 + 4 * j, query = q0 + c;
        float s = 0.f, dp = 0.f;
        for (int d = 0; d < kAD; ++d) {
          s = fmaf(Ks[r * kAPad + d], Qs[c * kAPad + d], s);
          dp = fmaf(Vs[r * kAPad + d], dOs[c * kAPad + d], dp);
        }
        const bool ok = key < t && query < t && visible(query, key, window);
        pj[j] = ok ? expf(s * scale - Ls[c]) : 0.f;
        dsj[j] = pj[j] * (dp - Ds[c]);
        Ss[r * kAPad + c] = pj[j];
      }
      __syncwarp();
      // dV[key] += sum_c P^T[key, c] dO[c]
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int d = own_dim(c0, j);
        float a = dvr[j];
        for (int c = 0; c < kAB; ++c) a = fmaf(Ss[r * kAPad + c], dOs[c * kAPad + d], a);
        dvr[j] = a;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 16; ++j) Ss[r * kAPad + c0 + 4 * j] = dsj[j];
      __syncwarp();
      // dK[key] += scale sum_c dS^T[key, c] Q[c]
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int d = own_dim(c0, j);
        float a = 0.f;
        for (int c = 0; c < kAB; ++c) a = fmaf(Ss[r * kAPad + c], Qs[c * kAPad + d], a);
        dkr[j] = fmaf(a, scale, dkr[j]);
      }
      __syncthreads();
      // dQ[query r'] += scale sum_keys dS^T[key, r'] K[key]: thread (query r, dims of c0)
      const int query = q0 + r;
      if (query < t) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int d = own_dim(c0, j);
          float a = 0.f;
          for (int kk = 0; kk < kAB; ++kk) a = fmaf(Ss[kk * kAPad + r], Ks[kk * kAPad + d], a);
          atomicAdd(&dq[(base + query) * lddq + h * kAD + d], a * scale);
        }
      }
    }
  }
  if (key < t) {
    const float* tab = rope + static_cast<size_t>(key % t) * 64;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {  // dims (d, d + 1) are a RoPE pair: dk = R^T dk_rot
      const int d = own_dim(c0, j);
      const float cs = tab[d], sn = tab[d + 1];
      const float x = dkr[j], y = dkr[j + 1];
      dk[(base + key) * lddk + kvh * kAD + d] = x * cs + y * sn;
      dk[(base + key) * lddk + kvh * kAD + d + 1] = -x * sn + y * cs;
      dv[(base + key) * lddv + kvh * kAD + d] = dvr[j];
      dv[(base + key) * lddv + kvh * kAD + d + 1] = dvr[j + 1];
    }
  }
}

// dq = R^T dq_rot in place (thread per pair)
__global__ void attn_f32_dq_finish_kernel(float* dq, int lddq, int rows, int hq, int t, const float* rope) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int pairs = hq * kAD / 2;
  if (i >= static_cast<size_t>(rows) * pairs) return;
  const int row = static_cast<int>(i / pairs), pr = static_cast<int>(i % pairs);
  const int col = 2 * pr, d = col % kAD;
  const float* tab = rope + static_cast<size_t>(row % t) * 64 + d;
  float* x = dq + static_cast<size_t>(row) * lddq + col;
  const float a = x[0], b = x[1];
  x[0] = a * tab[0] + b * tab[1];
  x[1] = -a * tab[1] + b * tab[0];
}

}  // namespace sj

using namespace sj;

extern "C" int sj_sgemm(const float* a, int lda, int a_trans, const float* b, int ldb, int b_trans, float* c, int ldc,
                        int m, int n, int k, int epilogue, float* aux, int ld_aux, const float* rope_table,
                        int rope_cols, int rope_t, void* stream) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(SJ_ERR_SHAPE, "sj_sgemm: m=%d n=%d k=%d", m, n, k);
  if (!a || !b || !c) return fail(SJ_ERR_ARGUMENT, "sj_sgemm: null operand");
  if (lda < (a_trans ? m : k) || ldb < (b_trans ? k : n) || ldc < n)
    return fail(SJ_ERR_SHAPE, "sj_sgemm: leading dimension smaller than the matrix width");
  switch (epilogue) {
    case SJ_EPI_STORE:
    case SJ_EPI_ACCUM:
      break;
    case SJ_EPI_RESIDUAL:
      if (!aux || ld_aux < n) return fail(SJ_ERR_ARGUMENT, "sj_sgemm: RESIDUAL needs aux");
      break;
    case SJ_EPI_SWIGLU:
      if (!aux || n % 32 || ld_aux < n / 2) return fail(SJ_ERR_ARGUMENT, "sj_sgemm: SWIGLU needs aux and N %% 32 == 0");
      break;
    case SJ_EPI_ROPE:
      if (!rope_table || rope_t <= 0 || rope_cols % 64 || rope_cols > n)
        return fail(SJ_ERR_ARGUMENT, "sj_sgemm: ROPE needs a table, rope_t > 0 and rope_cols %% 64 == 0");
      break;
    default:
      return fail(SJ_ERR_ARGUMENT, "sj_sgemm: epilogue %d not available in f32", epilogue);
  }
  SgemmParams p{a, b, c, aux, rope_table, lda, ldb, ldc, ld_aux, a_trans, b_trans, m, n, k, epilogue, rope_cols,
                rope_t > 0 ? rope_t : 1};
  // 128 x 128 tiles when they fill two waves of the SMs, else 64 x 64; an accumulating product whose
  // tiles still leave SMs idle (a weight gradient: small M x N, K = the rows) splits K as well
  const int sms = sm_count();
  const long long big = static_cast<long long>((m + kSBM - 1) / kSBM) * ((n + kSBN - 1) / kSBN);
  const bool large = big >= 2LL * sms;
  const int bm = large ? kSBM : 64, bn = large ? kSBN : 64;
  const long long tiles = static_cast<long long>((m + bm - 1) / bm) * ((n + bn - 1) / bn);
  int splits = 1;
  if (epilogue == SJ_EPI_ACCUM && tiles < 2LL * sms) {
    splits = static_cast<int>((2LL * sms + tiles - 1) / tiles);
    splits = std::max(1, std::min(splits, k / 256));
  }
  const int kslice = (((k + splits - 1) / splits) + kSBK - 1) / kSBK * kSBK;
  splits = (k + kslice - 1) / kslice;
  const dim3 grid((n + bn - 1) / bn, (m + bm - 1) / bm, splits);
  if (large)
    launch(sgemm_kernel<kSBM, kSBN>, grid, kSThreads, 0, as_stream(stream), p, kslice);
  else
    launch(sgemm_kernel<64, 64>, grid, kSThreads, 0, as_stream(stream), p, kslice);
  SJ_LAUNCH_CHECK("sgemm");
  return SJ_OK;
}

extern "C" int sj_swiglu_bwd_f32(const float* gu, const float* dh, float* dgu, int rows, int f, void* stream) {
  if (rows <= 0 || f <= 0 || f % 16) return fail(SJ_ERR_SHAPE, "sj_swiglu_bwd_f32: f=%d must be a multiple of 16", f);
  if (!gu || !dh || !dgu) return fail(SJ_ERR_ARGUMENT, "sj_swiglu_bwd_f32: null");
  const size_t n = static_cast<size_t>(rows) * f;
  launch(swiglu_bwd_f32_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream), gu, dh, dgu, rows,
         f);
  SJ_LAUNCH_CHECK("swiglu_bwd_f32");
  return SJ_OK;
}

static int attn_f32_check(int batch, int t, int hq, int hk, int head_dim, int window) {
  if (head_dim != kAD) return fail(SJ_ERR_UNSUPPORTED, "attention f32: head_dim %d (this build: 64)", head_dim);
  if (batch <= 0 || t <= 0 || hq <= 0 || hk <= 0 || hq % hk || window < 0)
    return fail(SJ_ERR_SHAPE, "attention f32: bad shape batch=%d t=%d hq=%d hk=%d window=%d", batch, t, hq, hk, window);
  return SJ_OK;
}

extern "C" int sj_attn_f32_fwd(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* o,
                               int ldo, float* lse, int batch, int t, int hq, int hk, int head_dim, int window,
                               void* stream) {
  int rc = attn_f32_check(batch, t, hq, hk, head_dim, window);
  if (rc != SJ_OK) return rc;
  if (!q || !k || !v || !o || !lse) return fail(SJ_ERR_ARGUMENT, "sj_attn_f32_fwd: null");
  const size_t smem = 4 * kAB * kAPad * sizeof(float);
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    rc = cuda_check(cudaFuncSetAttribute(attn_f32_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)), "sj_attn_f32_fwd: shared memory");
    if (rc != SJ_OK) return rc;
    configured = dev;
  }
  const dim3 grid((t + kAB - 1) / kAB, hq, batch);
  launch(attn_f32_fwd_kernel, grid, kAThreads, smem, as_stream(stream), q, ldq, k, ldk, v, ldv, o, ldo, lse, t, hq, hk,
         window);
  SJ_LAUNCH_CHECK("attn_f32_fwd");
  return SJ_OK;
}

extern "C" size_t sj_attn_f32_workspace(int batch, int t, int hq) {
  return static_cast<size_t>(batch) * t * hq;  // floats: Delta
}

extern "C" int sj_attn_f32_bwd(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv,
                               const float* o, int ldo, const float* lse, const float* dout, int lddo, float* dq,
                               int lddq, float* dk, int lddk, float* dv, int lddv, float* workspace, int batch, int t,
                               int hq, int hk, int head_dim, int window, const float* rope_table, void* stream) {
  int rc = attn_f32_check(batch, t, hq, hk, head_dim, window);
  if (rc != SJ_OK) return rc;
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv || !workspace || !rope_table)
    return fail(SJ_ERR_ARGUMENT, "sj_attn_f32_bwd: null");
  const int rows = batch * t;
  cudaStream_t s = as_stream(stream);
  const size_t warps = static_cast<size_t>(rows) * hq;
  launch(attn_f32_delta_kernel, static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, s, o, ldo, dout, lddo,
         workspace, dq, lddq, rows, hq);
  SJ_LAUNCH_CHECK("attn_f32_delta");
  const size_t smem = (5 * kAB * kAPad + 2 * kAB) * sizeof(float);
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    rc = cuda_check(cudaFuncSetAttribute(attn_f32_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)), "sj_attn_f32_bwd: shared memory");
    if (rc != SJ_OK) return rc;
    configured = dev;
  }
  const dim3 grid((t + kAB - 1) / kAB, hk, batch);
  launch(attn_f32_bwd_kernel, grid, kAThreads, smem, s, q, ldq, k, ldk, v, ldv, lse, workspace, dout, lddo, dq, lddq,
         dk, lddk, dv, lddv, t, hq, hk, window, rope_table);
  SJ_LAUNCH_CHECK("attn_f32_bwd");
  const size_t pairs = static_cast<size_t>(rows) * hq * kAD / 2;
  launch(attn_f32_dq_finish_kernel, static_cast<unsigned>((pairs + 255) / 256), 256, 0, s, dq, lddq, rows, hq, t,
         rope_table);
  SJ_LAUNCH_CHECK("attn_f32_dq_finish");
  return SJ_OK;
}
