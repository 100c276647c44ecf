// tcgen05 GEMM for sm_100a: C[M,N] = op(A) * op(B), bf16 operands, f32 accumulation in TMEM.
//
// Replaces the reference's `matmul`, `projection_qkv` and `projection_gate_up` Triton kernels
// (python/sejong_kernels/ops/kernels.py:23-39, projection.py:6-73) and the tape's backward GEMMs
// dA = dY*B^T (NT) and dB = A^T*dY (TN) (crates/sejong-gpu/src/graph.rs:817-853).
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte swizzle,
//               STAGES-deep ring guarded by full/empty mbarriers.
//   warp 1      allocates TMEM (2 x BN f32 columns = two accumulators) and one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, fused epilogue, global stores, while
//               the MMA warp already fills the other accumulator.
// A and B may each be K-major or MN-major in global memory (the UMMA descriptor's major bit), so
// forward (A K-major, B N-major), input-gradient (A K-major, B K-major) and weight-gradient
// (A M-major, B N-major) products all read their operands in place.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace sj {

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, kb_total;
  void* c;
  int ldc;
  int c_f32;
  int epilogue;
  float alpha;
  void* aux;
  int ld_aux;
  int rope_cols, rope_t;
  float rope_log_theta;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // 256 or 512: powers of two
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

SJ_DEVICE void store_row_bf16(__nv_bfloat16* dst, int col0, int n, const float* v, int count) {
  // count = 32 consecutive columns starting at col0; 16-byte vector stores when fully in range.
  if (col0 + count <= n && (reinterpret_cast<uintptr_t>(dst + col0) & 15u) == 0) {
    uint4* d = reinterpret_cast<uint4*>(dst + col0);
#pragma unroll
    for (int j = 0; j < count / 8; ++j) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      d[j] = w;
    }
  } else {
    for (int j = 0; j < count; ++j)
      if (col0 + j < n) dst[col0 + j] = f2bf(v[j]);
  }
}

SJ_DEVICE void epilogue_chunk(const GemmParams& p, int row, int col0, float (&v)[32], bool atomic) {
  if (row >= p.M) return;
  const float alpha = p.alpha;
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] *= alpha;
  switch (p.epilogue) {
    case SJ_EPI_STORE: {
      if (p.c_f32) {
        float* dst = reinterpret_cast<float*>(p.c) + static_cast<size_t>(row) * p.ldc;
        if (col0 + 32 <= p.N && (reinterpret_cast<uintptr_t>(dst + col0) & 15u) == 0) {
          float4* d = reinterpret_cast<float4*>(dst + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.N) dst[col0 + j] = v[j];
        }
      } else {
        store_row_bf16(reinterpret_cast<__nv_bfloat16*>(p.c) + static_cast<size_t>(row) * p.ldc, col0, p.N, v, 32);
      }
      break;
    }
    case SJ_EPI_ACCUM: {
      float* dst = reinterpret_cast<float*>(p.c) + static_cast<size_t>(row) * p.ldc;
      if (atomic) {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) atomicAdd(dst + col0 + j, v[j]);
      } else if (col0 + 32 <= p.N && (reinterpret_cast<uintptr_t>(dst + col0) & 15u) == 0) {
        float4* d = reinterpret_cast<float4*>(dst + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 o = d[j];
          o.x += v[4 * j];
          o.y += v[4 * j + 1];
          o.z += v[4 * j + 2];
          o.w += v[4 * j + 3];
          d[j] = o;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) dst[col0 + j] += v[j];
      }
      break;
    }
    case SJ_EPI_RESIDUAL: {
      if (p.c_f32) {  // f32 residual stream: C = aux + acc, both f32
        const float* res = reinterpret_cast<const float*>(p.aux) + static_cast<size_t>(row) * p.ld_aux;
        float* dst = reinterpret_cast<float*>(p.c) + static_cast<size_t>(row) * p.ldc;
        if (col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(res + col0) | reinterpret_cast<uintptr_t>(dst + col0)) & 15u) == 0) {
          const float4* r4 = reinterpret_cast<const float4*>(res + col0);
          float4* d4 = reinterpret_cast<float4*>(dst + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 r = r4[j];
            d4[j] = make_float4(v[4 * j] + r.x, v[4 * j + 1] + r.y, v[4 * j + 2] + r.z, v[4 * j + 3] + r.w);
          }
        } else {
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.N) dst[col0 + j] = v[j] + res[col0 + j];
        }
        break;
      }
      const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(p.aux) + static_cast<size_t>(row) * p.ld_aux;
      if (col0 + 32 <= p.N && (reinterpret_cast<uintptr_t>(res + col0) & 15u) == 0) {
        const uint4* r4 = reinterpret_cast<const uint4*>(res + col0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w = r4[j];
          float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
          v[8 * j + 0] += a.x;
          v[8 * j + 1] += a.y;
          v[8 * j + 2] += b.x;
          v[8 * j + 3] += b.y;
          v[8 * j + 4] += c.x;
          v[8 * j + 5] += c.y;
          v[8 * j + 6] += d.x;
          v[8 * j + 7] += d.y;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) v[j] += bf2f(res[col0 + j]);
      }
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(p.c) + static_cast<size_t>(row) * p.ldc, col0, p.N, v, 32);
      break;
    }
    case SJ_EPI_SWIGLU: {
      // columns [col0, col0+16) are gate features f0..f0+15, [col0+16, col0+32) the matching up features.
      // g and u are rounded to bf16 before h = silu(g)*u (projection.py:464-470).
      float h[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float g = round_bf16(v[j]);
        const float u = round_bf16(v[16 + j]);
        h[j] = g / (1.0f + __expf(-g)) * u;
      }
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(p.c) + static_cast<size_t>(row) * p.ldc, col0, p.N, v, 32);
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(p.aux) + static_cast<size_t>(row) * p.ld_aux, col0 / 2,
                     p.N / 2, h, 16);
      break;
    }
    case SJ_EPI_ROPE: {
      if (col0 < p.rope_cols) {
        const float pos = static_cast<float>(row % p.rope_t);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const int pair = ((col0 + j) & 63) >> 1;
          const float inv_freq = expf((-2.0f * static_cast<float>(pair) / 64.0f) * p.rope_log_theta);
          float s, c;
          sincosf(pos * inv_freq, &s, &c);
          const float a = v[j], b = v[j + 1];
          v[j] = a * c - b * s;
          v[j + 1] = a * s + b * c;
        }
      }
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(p.c) + static_cast<size_t>(row) * p.ldc, col0, p.N, v, 32);
      break;
    }
    default:
      break;
  }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = umma_idesc_bf16(kBM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = p.m_tiles * p.n_tiles * p.splits;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        const int ks = tile % p.splits;
        const int nb = (tile / p.splits) % p.n_tiles;
        const int mb = tile / (p.splits * p.n_tiles);
        const int m0 = mb * kBM, n0 = nb * BN;
        const int kb_begin = ks * p.kb_per_split;
        const int kb_end = min(kb_begin + p.kb_per_split, p.kb_total);
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = static_cast<uint32_t>(it / STAGES);
          if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort_flag, SJ_DEV_GEMM_PRODUCER_WAIT)) break;
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          const int k0 = kb * kBK;
          if (A_MN) {
            tma_load_2d(sa, &map_a, &full[s], m0, k0);
            tma_load_2d(sa + 8192, &map_a, &full[s], m0 + 64, k0);
          } else {
            tma_load_2d(sa, &map_a, &full[s], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * 8192, &map_b, &full[s], n0 + 64 * c, k0);
          } else {
            tma_load_2d(sb, &map_b, &full[s], k0, n0);
          }
        }
      }
      // drain: wait (bounded) for the copies still in flight into the most recent stages
      for (int j = max(0, it - STAGES); j < it; ++j)
        mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1u, nullptr, SJ_DEV_GEMM_DRAIN_WAIT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++local) {
        const int ks = tile % p.splits;
        const int kb_begin = ks * p.kb_per_split;
        const int kb_end = min(kb_begin + p.kb_per_split, p.kb_total);
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag, SJ_DEV_GEMM_MMA_WAIT)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = static_cast<uint32_t>(it / STAGES);
          if (!mbar_wait(&full[s], round & 1u, abort_flag, SJ_DEV_GEMM_MMA_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = A_MN ? umma_desc(a_base + kk * 2048, 8192, 1024) : umma_desc(a_base + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? umma_desc(b_base + kk * 2048, 8192, 1024) : umma_desc(b_base + kk * 32, 16, 1024);
            umma_f16(d_tmem, da, db, IDESC, (kb > kb_begin || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      // all issued MMAs must retire before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, SJ_DEV_GEMM_DRAIN_WAIT);
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32) belong to this warp
    int local = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++local) {
      const int ks = tile % p.splits;
      const int nb = (tile / p.splits) % p.n_tiles;
      const int mb = tile / (p.splits * p.n_tiles);
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&acc_full[buf], use & 1u, abort_flag, SJ_DEV_GEMM_EPILOGUE_WAIT)) break;
      tc_fence_after();
      const int row = mb * kBM + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      const bool atomic = p.splits > 1;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        const int col0 = nb * BN + c * 32;
        if (col0 < p.N) epilogue_chunk(p, row, col0, v, atomic);
      }
      (void)ks;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map: `inner` contiguous elements per row, `outer` rows, row stride `ld` elements.
static int make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                    uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SJ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SJ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SJ_OK;
}

template <int BN, bool A_MN, bool B_MN>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p, int grid,
                       cudaStream_t stream) {
  auto kernel = gemm_tcgen05_kernel<BN, A_MN, B_MN>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM);
    if (e != cudaSuccess) return cuda_check(e, "gemm shared-memory attribute");
    configured_device = dev;
  }
  kernel<<<grid, kThreads, GemmCfg<BN>::SMEM, stream>>>(ma, mb, p);
  SJ_LAUNCH_CHECK("gemm launch");
  return SJ_OK;
}

template <int BN>
static int dispatch_majors(bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p,
                           int grid, cudaStream_t s) {
  if (!a_mn && b_mn) return launch_gemm<BN, false, true>(ma, mb, p, grid, s);
  if (!a_mn && !b_mn) return launch_gemm<BN, false, false>(ma, mb, p, grid, s);
  if (a_mn && b_mn) return launch_gemm<BN, true, true>(ma, mb, p, grid, s);
  return launch_gemm<BN, true, false>(ma, mb, p, grid, s);
}

}  // namespace sj

extern "C" int sj_gemm(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c, int ldc,
                       int c_dtype, int m, int n, int k, int epilogue, float alpha, void* aux, int ld_aux,
                       int rope_cols, int rope_t, float rope_theta, int split_k, void* stream) {
  using namespace sj;
  if (m <= 0 || n <= 0 || k <= 0) return fail(SJ_ERR_SHAPE, "sj_gemm: empty problem %dx%dx%d", m, n, k);
  if (!a || !b || !c) return fail(SJ_ERR_ARGUMENT, "sj_gemm: null operand");
  if (!aligned16(a) || !aligned16(b)) return fail(SJ_ERR_ARGUMENT, "sj_gemm: A/B must be 16-byte aligned");
  if ((lda % 8) || (ldb % 8)) return fail(SJ_ERR_ARGUMENT, "sj_gemm: lda/ldb must be multiples of 8 elements");
  const int a_rows_min = a_trans ? m : k, b_rows_min = b_trans ? k : n;
  if (lda < a_rows_min || ldb < b_rows_min || ldc < n)
    return fail(SJ_ERR_SHAPE, "sj_gemm: leading dimension smaller than the matrix width");
  if (c_dtype != SJ_BF16 && c_dtype != SJ_F32) return fail(SJ_ERR_ARGUMENT, "sj_gemm: C must be bf16 or f32");
  switch (epilogue) {
    case SJ_EPI_STORE:
      break;
    case SJ_EPI_ACCUM:
      if (c_dtype != SJ_F32) return fail(SJ_ERR_ARGUMENT, "sj_gemm: ACCUM needs an f32 C");
      break;
    case SJ_EPI_RESIDUAL:
      if (!aux) return fail(SJ_ERR_ARGUMENT, "sj_gemm: RESIDUAL needs aux (same dtype as C)");
      break;
    case SJ_EPI_SWIGLU:
      if (c_dtype != SJ_BF16 || !aux || (n % 32))
        return fail(SJ_ERR_ARGUMENT, "sj_gemm: SWIGLU needs bf16 C, aux and N %% 32 == 0");
      break;
    case SJ_EPI_ROPE:
      if (c_dtype != SJ_BF16 || rope_t <= 0 || (rope_cols % 64) || rope_theta <= 0.f)
        return fail(SJ_ERR_ARGUMENT, "sj_gemm: ROPE needs bf16 C, rope_t > 0, rope_cols %% 64 == 0");
      break;
    default:
      return fail(SJ_ERR_ARGUMENT, "sj_gemm: unknown epilogue %d", epilogue);
  }
  if (split_k > 1 && epilogue != SJ_EPI_ACCUM) return fail(SJ_ERR_ARGUMENT, "sj_gemm: split_k needs ACCUM");

  const int sms = sm_count();
  const int m_tiles = (m + kBM - 1) / kBM;
  const int kb_total = (k + kBK - 1) / kBK;
  int bn = 128;
  if (n > 128 && m_tiles * ((n + 255) / 256) >= sms) bn = 256;
  const int n_tiles = (n + bn - 1) / bn;
  int splits = 1;
  if (epilogue == SJ_EPI_ACCUM) {
    if (split_k > 0) {
      splits = split_k;
    } else {
      const int tiles = m_tiles * n_tiles;
      splits = tiles >= sms ? 1 : (2 * sms + tiles - 1) / tiles;
      splits = std::min(splits, std::max(1, kb_total / 4));
    }
    splits = std::max(1, std::min(splits, kb_total));
  }
  const int kb_per_split = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per_split - 1) / kb_per_split;  // no empty split

  CUtensorMap ma, mb;
  int rc;
  if (!a_trans)
    rc = make_map(&ma, a, static_cast<uint64_t>(k), static_cast<uint64_t>(m), lda, 64, 128);
  else
    rc = make_map(&ma, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k), lda, 64, 64);
  if (rc) return rc;
  if (b_trans)
    rc = make_map(&mb, b, static_cast<uint64_t>(k), static_cast<uint64_t>(n), ldb, 64, static_cast<uint32_t>(bn));
  else
    rc = make_map(&mb, b, static_cast<uint64_t>(n), static_cast<uint64_t>(k), ldb, 64, 64);
  if (rc) return rc;

  GemmParams p;
  p.M = m;
  p.N = n;
  p.K = k;
  p.m_tiles = m_tiles;
  p.n_tiles = n_tiles;
  p.splits = splits;
  p.kb_per_split = kb_per_split;
  p.kb_total = kb_total;
  p.c = c;
  p.ldc = ldc;
  p.c_f32 = c_dtype == SJ_F32;
  p.epilogue = epilogue;
  p.alpha = alpha;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.rope_cols = rope_cols;
  p.rope_t = rope_t > 0 ? rope_t : 1;
  p.rope_log_theta = rope_theta > 0.f ? logf(rope_theta) : 0.f;
  const int total = m_tiles * n_tiles * splits;
  const int grid = std::min(total, sms);
  const bool a_mn = a_trans != 0;   // A stored [K, M]
  const bool b_mn = b_trans == 0;   // B stored [K, N]
  if (bn == 256) return dispatch_majors<256>(a_mn, b_mn, ma, mb, p, grid, as_stream(stream));
  return dispatch_majors<128>(a_mn, b_mn, ma, mb, p, grid, as_stream(stream));
}
