// Causal grouped-query attention with an optional sliding window, backward, head dim 64 (the forward
// is the tcgen05 kernel of attention_fwd.cu).
//
// Restates python/sejong_kernels/ops/hierarchy.py:42-104 (hierarchy_attention _dq, _dkv): query
// (b, t, h) attends keys s of kv head h / (HQ/HK) with max(0, t+1-W) <= s <= t, scale 64^-1/2,
// LSE in natural log.  The reference launches one program per (row, head) and re-reads K/V for
// every query; here a CTA owns a 64-query (or 64-key) tile, K/V (or Q/dO) tiles are staged once in
// swizzled shared memory with cp.async double buffering and shared by the CTA's four warps, and the
// products run on bf16 mma.sync tensor-core tiles with f32 accumulation and an online softmax.
// dQ is one pass over key tiles; dK/dV is one CTA per (key tile, query head) so the causal
// critical path is a single head long, and for grouped heads a small kernel sums the group's f32
// partials (no atomics) and applies the inverse RoPE.
#include "common.cuh"
#include "internal.h"

namespace sj {

constexpr int kAttnD = 64;
constexpr int kAttnTile = 64;
constexpr int kAttnThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnParams {
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  __nv_bfloat16 *out, *dq, *dk, *dv;
  const float* lse_in;
  float* lse_out;
  float* delta;
  int ldq, ldk, ldv, ldo, lddo, lddq, lddk, lddv;
  int t, hq, hk, window;
  float scale;       // head_dim^-1/2
  float rope_log_theta;  // > 0: apply the inverse RoPE rotation to dq / dk before the store
  const float2* rope_tab;  // optional (cos, sin) table [t][32]; preferred over rope_log_theta
};

// 64 x 64 bf16 tile, 128-byte rows, 16-byte chunks XOR-swizzled by (row & 7).
SJ_DEVICE uint32_t tile_addr(uint32_t base, int row, int col) {
  return base + row * 128 + ((((col >> 3) ^ (row & 7))) << 4);
}

SJ_DEVICE void load_tile_async(__nv_bfloat16* s, const __nv_bfloat16* g, int ld, int row0, int t) {
  for (int i = threadIdx.x; i < kAttnTile * 8; i += kAttnThreads) {
    const int r = i >> 3, c = i & 7;
    const bool valid = row0 + r < t;
    const __nv_bfloat16* src = g + static_cast<size_t>(valid ? row0 + r : 0) * ld + c * 8;
    cp_async16(reinterpret_cast<uint8_t*>(s) + r * 128 + ((c ^ (r & 7)) << 4), src, valid);
  }
}

// A fragments (16 rows x 64) of rows [r0, r0+16) of a swizzled tile: frag[kstep][4].
SJ_DEVICE void load_a_frags(uint32_t (&f)[4][4], uint32_t base, int r0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) ldmatrix_x4(f[ks], tile_addr(base, r0 + (lane & 15), ks * 16 + (lane >> 4) * 8));
}

// acc[16 x 64] += A(frags, k = 64 feature columns) * B^T where B is a [64 rows][64 cols] tile whose
// rows are the output columns (n) and whose columns are the contraction (k): S = Q K^T form.
SJ_DEVICE void mma_abt(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t b_base) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldmatrix_x4(b, tile_addr(b_base, np * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 16 + ((lane >> 3) & 1) * 8));
      mma_bf16_16816(acc[2 * np], a[ks], b[0], b[1]);
      mma_bf16_16816(acc[2 * np + 1], a[ks], b[2], b[3]);
    }
  }
}

// acc[16 x 64] += P(frags from a 16 x 64 C-layout matrix, k = 64 tile rows) * B where B is a
// [64 rows = k][64 cols = n] tile: O = P V form.
SJ_DEVICE void mma_ab(float (&acc)[8][4], const uint32_t (&p)[4][4], uint32_t b_base) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int dp = 0; dp < 4; ++dp) {
      uint32_t b[4];
      ldmatrix_x4_trans(b, tile_addr(b_base, ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
      mma_bf16_16816(acc[2 * dp], p[ks], b[0], b[1]);
      mma_bf16_16816(acc[2 * dp + 1], p[ks], b[2], b[3]);
    }
  }
}

// C-layout 16 x 64 f32 -> bf16 A fragments with k = the 64 columns.
SJ_DEVICE void c_to_a_frags(uint32_t (&a)[4][4], const float (&c)[8][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a[j][0] = pack_bf16x2(c[2 * j][0], c[2 * j][1]);
    a[j][1] = pack_bf16x2(c[2 * j][2], c[2 * j][3]);
    a[j][2] = pack_bf16x2(c[2 * j + 1][0], c[2 * j + 1][1]);
    a[j][3] = pack_bf16x2(c[2 * j + 1][2], c[2 * j + 1][3]);
  }
}

SJ_DEVICE void zero(float (&c)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.f;
}

// Store a warp's 16 x 64 C-layout tile (rows r0.., head columns) as bf16, optionally rotating the
// (2i, 2i+1) pairs back by the RoPE angle of position (row mod t).
SJ_DEVICE void store_rows(__nv_bfloat16* dst, int ld, const float (&c)[8][4], int r0, int t_limit, int pos_base,
                          float rope_log_theta, const float2* rope_tab) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = r0 + g + half * 8;
    if (r >= t_limit) continue;
    const float pos = static_cast<float>(pos_base + r);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = nt * 8 + 2 * tq;
      float a = c[nt][2 * half], b = c[nt][2 * half + 1];
      if (rope_tab != nullptr || rope_log_theta > 0.f) {
        float s, co;
        if (rope_tab != nullptr) {
          const float2 cs = rope_tab[static_cast<size_t>(pos_base + r) * 32 + (col >> 1)];
          co = cs.x;
          s = cs.y;
        } else {
          const float inv_freq = expf((-2.0f * static_cast<float>(col >> 1) / 64.0f) * rope_log_theta);
          sincosf(pos * inv_freq, &s, &co);
        }
        const float na = a * co + b * s, nb = -a * s + b * co;  // inverse rotation
        a = na;
        b = nb;
      }
      *reinterpret_cast<uint32_t*>(dst + static_cast<size_t>(r) * ld + col) = pack_bf16x2(a, b);
    }
  }
}

// ------------------------------------------------------------------------------------ forward
constexpr int kTileElems = kAttnTile * kAttnD;
constexpr int kDqSmem = 6 * kTileElems * 2;
constexpr int kDkvSmem = 6 * kTileElems * 2 + 4 * kAttnTile * 4;

// ------------------------------------------------------------------------------------ backward
// Delta[row*hq + h] = sum_d dO * O (hierarchy.py:53-57).
__global__ void attn_delta_kernel(const AttnParams p, int rows) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= rows * p.hq) return;
  const int row = w / p.hq, h = w % p.hq;
  const float2 a = unpack_bf16x2(
      *reinterpret_cast<const uint32_t*>(p.dout + static_cast<size_t>(row) * p.lddo + h * kAttnD + 2 * lane));
  const float2 c = unpack_bf16x2(
      *reinterpret_cast<const uint32_t*>(p.o + static_cast<size_t>(row) * p.ldo + h * kAttnD + 2 * lane));
  const float s = warp_sum(a.x * c.x + a.y * c.y);
  if (lane == 0) p.delta[w] = s;
}

// dQ for one 64-query tile of head h (hierarchy.py:42-70).
__global__ void __launch_bounds__(kAttnThreads, 3) attn_dq_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  // smem: Q, dO, then K stages 0/1, then V stages 0/1
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(attn_smem);
  __nv_bfloat16* sdo = sq + kTileElems;
  __nv_bfloat16* sk0 = sq + 2 * kTileElems;
  __nv_bfloat16* sv0 = sq + 4 * kTileElems;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.hq / p.hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int q0 = qb * kAttnTile;
  const size_t brow = static_cast<size_t>(b) * p.t;
  const __nv_bfloat16* kg = p.k + brow * p.ldk + kvh * kAttnD;
  const __nv_bfloat16* vg = p.v + brow * p.ldv + kvh * kAttnD;
  const int kb_lo = p.window > 0 ? max(0, q0 - p.window + 1) / kAttnTile : 0;
  const int kb_hi = min((q0 + kAttnTile - 1) / kAttnTile, (p.t - 1) / kAttnTile);

  load_tile_async(sq, p.q + brow * p.ldq + h * kAttnD, p.ldq, q0, p.t);
  load_tile_async(sdo, p.dout + brow * p.lddo + h * kAttnD, p.lddo, q0, p.t);
  load_tile_async(sk0, kg, p.ldk, kb_lo * kAttnTile, p.t);
  load_tile_async(sv0, vg, p.ldv, kb_lo * kAttnTile, p.t);
  cp_async_commit();

  const int row_lo = q0 + warp * 16 + g;
  float lse2[2], dl[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = min(row_lo + 8 * i, p.t - 1);
    lse2[i] = p.lse_in[(brow + r) * p.hq + h] * kLog2e;
    dl[i] = p.delta[(brow + r) * p.hq + h];
  }
  const float sl2 = p.scale * kLog2e;
  uint32_t qf[4][4], df[4][4];
  float dq[8][4];
  zero(dq);
  for (int kb = kb_lo; kb <= kb_hi; ++kb) {
    const int st = (kb - kb_lo) & 1;
    if (kb < kb_hi) {
      load_tile_async(sk0 + (st ^ 1) * kTileElems, kg, p.ldk, (kb + 1) * kAttnTile, p.t);
      load_tile_async(sv0 + (st ^ 1) * kTileElems, vg, p.ldv, (kb + 1) * kAttnTile, p.t);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == kb_lo) {
      load_a_frags(qf, smem_u32(sq), warp * 16);
      load_a_frags(df, smem_u32(sdo), warp * 16);
    }
    float s[8][4], dp[8][4];
    zero(s);
    zero(dp);
    mma_abt(s, qf, smem_u32(sk0 + st * kTileElems));
    mma_abt(dp, df, smem_u32(sv0 + st * kTileElems));
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qpos = row_lo + (e >> 1) * 8;
        const int kpos = kb * kAttnTile + nt * 8 + 2 * tq + (e & 1);
        const bool ok = kpos <= qpos && kpos < p.t && qpos < p.t && (p.window <= 0 || qpos - kpos < p.window);
        const float pr = ok ? exp2f(s[nt][e] * sl2 - lse2[e >> 1]) : 0.f;
        s[nt][e] = pr * (dp[nt][e] - dl[e >> 1]) * p.scale;  // dS
      }
    uint32_t sf[4][4];
    c_to_a_frags(sf, s);
    mma_ab(dq, sf, smem_u32(sk0 + st * kTileElems));
    __syncthreads();
  }
  store_rows(p.dq + brow * p.lddq + h * kAttnD, p.lddq, dq, q0 + warp * 16, p.t, 0, p.rope_log_theta, p.rope_tab);
}

// dK, dV of one 64-key tile against ONE query head h (hierarchy.py:73-104 sums the query group in
// one program; here each query head is its own CTA so the causal critical path is one head long).
// With a single query head per kv head the result is stored directly (bf16, inverse RoPE on dK);
// otherwise the f32 partial goes to part_dk / part_dv [rows, hq*64] and attn_dkv_reduce_kernel
// sums the group.
__global__ void __launch_bounds__(kAttnThreads, 3) attn_dkv_kernel(const AttnParams p, float* part_dk,
                                                                    float* part_dv) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  // smem: K, V, then Q stages 0/1, dO stages 0/1, LSE stages 0/1, Delta stages 0/1
  __nv_bfloat16* skk = reinterpret_cast<__nv_bfloat16*>(attn_smem);
  __nv_bfloat16* svv = skk + kTileElems;
  __nv_bfloat16* sq0 = skk + 2 * kTileElems;
  __nv_bfloat16* sdo0 = skk + 4 * kTileElems;
  float* slse0 = reinterpret_cast<float*>(skk + 6 * kTileElems);
  float* sdl0 = slse0 + 2 * kAttnTile;
  const int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int group = p.hq / p.hk;
  const int kvh = h / group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int k0 = kb * kAttnTile;
  const size_t brow = static_cast<size_t>(b) * p.t;
  const int nqb = (p.t + kAttnTile - 1) / kAttnTile;
  const int qb_lo = k0 / kAttnTile;
  const int qb_hi = p.window > 0 ? min(nqb - 1, (k0 + kAttnTile - 1 + p.window - 1) / kAttnTile) : nqb - 1;
  const __nv_bfloat16* qg = p.q + brow * p.ldq + h * kAttnD;
  const __nv_bfloat16* dog = p.dout + brow * p.lddo + h * kAttnD;

  load_tile_async(skk, p.k + brow * p.ldk + kvh * kAttnD, p.ldk, k0, p.t);
  load_tile_async(svv, p.v + brow * p.ldv + kvh * kAttnD, p.ldv, k0, p.t);
  auto issue = [&](int qb, int st) {
    load_tile_async(sq0 + st * kTileElems, qg, p.ldq, qb * kAttnTile, p.t);
    load_tile_async(sdo0 + st * kTileElems, dog, p.lddo, qb * kAttnTile, p.t);
    for (int i = threadIdx.x; i < kAttnTile; i += kAttnThreads) {
      const int r = min(qb * kAttnTile + i, p.t - 1);
      slse0[st * kAttnTile + i] = p.lse_in[(brow + r) * p.hq + h] * kLog2e;
      sdl0[st * kAttnTile + i] = p.delta[(brow + r) * p.hq + h];
    }
  };
  issue(qb_lo, 0);
  cp_async_commit();

  const float sl2 = p.scale * kLog2e;
  const int key_lo = k0 + warp * 16 + g;  // keys key_lo and key_lo + 8
  uint32_t kf[4][4], vf[4][4];
  float dk[8][4], dv[8][4];
  zero(dk);
  zero(dv);
  for (int qb = qb_lo; qb <= qb_hi; ++qb) {
    const int st = (qb - qb_lo) & 1;
    if (qb < qb_hi) {
      issue(qb + 1, st ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (qb == qb_lo) {
      load_a_frags(kf, smem_u32(skk), warp * 16);
      load_a_frags(vf, smem_u32(svv), warp * 16);
    }
    const float* slse = slse0 + st * kAttnTile;
    const float* sdl = sdl0 + st * kAttnTile;
    const uint32_t q_tile = smem_u32(sq0 + st * kTileElems);
    const uint32_t do_tile = smem_u32(sdo0 + st * kTileElems);
    float s[8][4];
    zero(s);
    mma_abt(s, kf, q_tile);  // S^T = K Q^T   [keys x queries]
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kpos = key_lo + (e >> 1) * 8;
        const int qi = nt * 8 + 2 * tq + (e & 1);
        const int qpos = qb * kAttnTile + qi;
        const bool ok = qpos >= kpos && qpos < p.t && kpos < p.t && (p.window <= 0 || qpos - kpos < p.window);
        s[nt][e] = ok ? exp2f(s[nt][e] * sl2 - slse[qi]) : 0.f;  // P^T
      }
    {
      uint32_t pf[4][4];
      c_to_a_frags(pf, s);
      mma_ab(dv, pf, do_tile);  // dV += P^T dO
    }
    float dp[8][4];
    zero(dp);
    mma_abt(dp, vf, do_tile);  // dP^T = V dO^T
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + 2 * tq + (e & 1);
        dp[nt][e] = s[nt][e] * (dp[nt][e] - sdl[qi]) * p.scale;  // dS^T
      }
    {
      uint32_t sf[4][4];
      c_to_a_frags(sf, dp);
      mma_ab(dk, sf, q_tile);  // dK += dS^T Q
    }
    __syncthreads();
  }
  if (group == 1) {
    store_rows(p.dk + brow * p.lddk + kvh * kAttnD, p.lddk, dk, k0 + warp * 16, p.t, 0, p.rope_log_theta,
               p.rope_tab);
    store_rows(p.dv + brow * p.lddv + kvh * kAttnD, p.lddv, dv, k0 + warp * 16, p.t, 0, 0.f, nullptr);
    return;
  }
  // f32 partials of this query head: [rows, hq*64]
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = k0 + warp * 16 + g + half * 8;
    if (r >= p.t) continue;
    float* pk = part_dk + (brow + r) * (static_cast<size_t>(p.hq) * kAttnD) + h * kAttnD;
    float* pv = part_dv + (brow + r) * (static_cast<size_t>(p.hq) * kAttnD) + h * kAttnD;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = nt * 8 + 2 * tq;
      *reinterpret_cast<float2*>(pk + col) = make_float2(dk[nt][2 * half], dk[nt][2 * half + 1]);
      *reinterpret_cast<float2*>(pv + col) = make_float2(dv[nt][2 * half], dv[nt][2 * half + 1]);
    }
  }
}

// Sum the query-group partials of dK / dV, apply the inverse RoPE to dK, store bf16.
// One thread per (row, kv head, column pair).
__global__ void attn_dkv_reduce_kernel(const AttnParams p, const float* __restrict__ part_dk,
                                       const float* __restrict__ part_dv, int rows) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int pairs = p.hk * (kAttnD / 2);
  if (i >= static_cast<size_t>(rows) * pairs) return;
  const int row = static_cast<int>(i / pairs);
  const int kvh = static_cast<int>(i % pairs) / (kAttnD / 2);
  const int col = (static_cast<int>(i % pairs) % (kAttnD / 2)) * 2;
  const int group = p.hq / p.hk;
  float2 k = make_float2(0.f, 0.f), v = make_float2(0.f, 0.f);
  const size_t base = static_cast<size_t>(row) * p.hq * kAttnD;
  for (int j = 0; j < group; ++j) {
    const int h = kvh * group + j;
    const float2 a = *reinterpret_cast<const float2*>(part_dk + base + h * kAttnD + col);
    const float2 c = *reinterpret_cast<const float2*>(part_dv + base + h * kAttnD + col);
    k.x += a.x;
    k.y += a.y;
    v.x += c.x;
    v.y += c.y;
  }
  if (p.rope_tab != nullptr || p.rope_log_theta > 0.f) {
    const int pos = row % p.t;
    float s, co;
    if (p.rope_tab != nullptr) {
      const float2 cs = p.rope_tab[static_cast<size_t>(pos) * 32 + (col >> 1)];
      co = cs.x;
      s = cs.y;
    } else {
      sincosf(static_cast<float>(pos) * expf((-2.0f * static_cast<float>(col >> 1) / 64.0f) * p.rope_log_theta), &s,
              &co);
    }
    const float na = k.x * co + k.y * s, nb = -k.x * s + k.y * co;
    k.x = na;
    k.y = nb;
  }
  *reinterpret_cast<uint32_t*>(p.dk + static_cast<size_t>(row) * p.lddk + kvh * kAttnD + col) = pack_bf16x2(k.x, k.y);
  *reinterpret_cast<uint32_t*>(p.dv + static_cast<size_t>(row) * p.lddv + kvh * kAttnD + col) = pack_bf16x2(v.x, v.y);
}

static int configure_attention() {
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured == dev) return SJ_OK;
  cudaError_t e = cudaFuncSetAttribute(attn_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDkvSmem);
  if (e != cudaSuccess) return cuda_check(e, "attention shared-memory attribute");
  configured = dev;
  return SJ_OK;
}

static int check_common(int batch, int t, int hq, int hk, int head_dim, int window) {
  if (head_dim != kAttnD) return fail(SJ_ERR_UNSUPPORTED, "attention: head_dim %d (this build: 64)", head_dim);
  if (batch <= 0 || t <= 0 || hq <= 0 || hk <= 0 || hq % hk || window < 0)
    return fail(SJ_ERR_SHAPE, "attention: bad shape batch=%d t=%d hq=%d hk=%d window=%d", batch, t, hq, hk, window);
  return SJ_OK;
}

}  // namespace sj

using namespace sj;

extern "C" size_t sj_attn_workspace(int batch, int t, int hq, int hk) {
  if (batch <= 0 || t <= 0 || hq <= 0 || hk <= 0) return 0;
  const size_t rows = static_cast<size_t>(batch) * t;
  return rows * hq + (hq != hk ? 2 * rows * hq * kAttnD : 0);
}

extern "C" int sj_attn_gqa_bwd(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv, const void* o,
                               int ldo, const float* lse, const void* dout, int lddo, void* dq, int lddq, void* dk,
                               int lddk, void* dv, int lddv, float* workspace, int batch, int t, int hq, int hk,
                               int head_dim, int window, float rope_theta, const float* rope_table, void* stream) {
  int rc = check_common(batch, t, hq, hk, head_dim, window);
  if (rc) return rc;
  if ((rc = configure_attention())) return rc;
  if ((ldq | ldk | ldv | ldo | lddo | lddq | lddk | lddv) % 8)
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: strides must be multiples of 8");
  if (!workspace || !aligned16(workspace)) return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: workspace must be aligned");
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.o = static_cast<const __nv_bfloat16*>(o);
  p.dout = static_cast<const __nv_bfloat16*>(dout);
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.lse_in = lse;
  p.ldq = ldq;
  p.ldk = ldk;
  p.ldv = ldv;
  p.ldo = ldo;
  p.lddo = lddo;
  p.lddq = lddq;
  p.lddk = lddk;
  p.lddv = lddv;
  p.t = t;
  p.hq = hq;
  p.hk = hk;
  p.window = window;
  p.scale = 0.125f;
  p.rope_log_theta = rope_theta > 0.f ? logf(rope_theta) : 0.f;
  p.rope_tab = reinterpret_cast<const float2*>(rope_table);
  if (rope_table && (reinterpret_cast<uintptr_t>(rope_table) & 7))
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: rope table must be 8-byte aligned");
  const int rows = batch * t;
  // workspace: delta [rows*hq], then (GQA only) f32 dK / dV partials [rows, hq*64] each
  p.delta = workspace;
  float* part_dk = workspace + ((static_cast<size_t>(rows) * hq + 3) / 4) * 4;
  float* part_dv = part_dk + static_cast<size_t>(rows) * hq * kAttnD;
  cudaStream_t s = as_stream(stream);
  const long long warps = static_cast<long long>(rows) * hq;
  attn_delta_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, s>>>(p, rows);
  SJ_LAUNCH_CHECK("attn_delta");
  attn_dq_kernel<<<dim3((t + kAttnTile - 1) / kAttnTile, hq, batch), kAttnThreads, kDqSmem, s>>>(p);
  SJ_LAUNCH_CHECK("attn_dq");
  attn_dkv_kernel<<<dim3((t + kAttnTile - 1) / kAttnTile, hq, batch), kAttnThreads, kDkvSmem, s>>>(p, part_dk,
                                                                                                  part_dv);
  SJ_LAUNCH_CHECK("attn_dkv");
  if (hq != hk) {
    const size_t n = static_cast<size_t>(rows) * hk * (kAttnD / 2);
    attn_dkv_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(p, part_dk, part_dv, rows);
    SJ_LAUNCH_CHECK("attn_dkv_reduce");
  }
  return SJ_OK;
}
