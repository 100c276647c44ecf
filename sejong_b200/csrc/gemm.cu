// tcgen05 GEMM for sm_100a: C[M,N] = op(A) * op(B), bf16 operands, f32 accumulation in TMEM.
//
// Replaces the reference's `matmul`, `projection_qkv` and `projection_gate_up` Triton kernels
// (python/sejong_kernels/ops/kernels.py:23-39, projection.py:6-73) and the tape's backward GEMMs
// dA = dY*B^T (NT) and dB = A^T*dY (TN) (crates/sejong-gpu/src/graph.rs:817-853).
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte swizzle, a
//               `stages`-deep ring (sized at launch to the shared memory left) guarded by
//               full/empty mbarriers.
//   warp 1      allocates TMEM (2 x BN f32 columns = two accumulators); one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, fused epilogue math, then each warp
//               stages its 32-row slab (128 bytes per row) in 128-byte-swizzled shared memory and
//               one lane writes it with a TMA bulk-tensor store -- or a TMA reduce-add for
//               accumulating (split-K) weight gradients -- while the MMA warp already fills the
//               other accumulator.
// A and B may each be K-major or MN-major in global memory (the UMMA descriptor's major bit), so
// forward (A K-major, B N-major), input-gradient (A K-major, B K-major) and weight-gradient
// (A M-major, B N-major) products all read their operands in place.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace sj {

// tcgen05.wait::ld that also names the registers the pending load writes, so no use of them can be
// scheduled above the wait.
SJ_DEVICE void tmem_wait_ld_dep(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, kb_total;
  int stages;
  int c_f32;
  int epilogue;
  float alpha;
  const void* aux;  // residual source (same dtype as C)
  int ld_aux;
  int rope_cols, rope_t;
  float rope_log_theta;
  const float* bias;  // [N] f32 (SJ_EPI_BIAS*), else null
  // Grouped products (one launch over all groups, e.g. the experts of an MoE layer); group_rows
  // is a device array [groups + 1] of row offsets, each a multiple of 128:
  //   group_mode 1 (grouped rows): the rows of A and C are packed by group; rows [group_rows[g],
  //     group_rows[g+1]) use B rows offset by g * b_group_rows (B's stored outer dimension);
  //   group_mode 2 (grouped reduction): C_g (rows offset by g * c_group_rows) = A_g^T B_g over
  //     the reduction rows [group_rows[g], group_rows[g+1]).
  const int* group_rows;
  int groups, group_mode, b_group_rows, c_group_rows;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpilogueWarps = 8;  // two per TMEM lane quarter, alternating 128-byte column units
constexpr int kThreads = 64 + 32 * kEpilogueWarps;
constexpr int kSmemLimit = 232448;          // 227 KB: the sm_100 per-block opt-in maximum
constexpr int kStagingC = kEpilogueWarps * 4096;  // one 32 rows x 128 B slab per epilogue warp
constexpr int kStagingH = kEpilogueWarps * 2048;  // SwiGLU h output: 32 rows x 64 B per warp
constexpr int kBarrierBytes = 512;  // barriers, then (grouped products) the group offsets
constexpr int kMaxGroups = 63;
constexpr int kPairStages = 6;  // a pair CTA's stage is 32 KB at BN = 256

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = BN == 128 ? 256 : 512;  // two accumulators, rounded to a power of two
};

SJ_DEVICE void tma_store_2d(const CUtensorMap* map, const void* smem, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem)), "r"(x), "r"(y)
               : "memory");
}
SJ_DEVICE void tma_reduce_add_2d(const CUtensorMap* map, const void* smem, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem)), "r"(x), "r"(y)
               : "memory");
}
// erf GELU, kernels.py:227-232: 0.5 x (1 + erf(x / sqrt 2))
SJ_DEVICE float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }
SJ_DEVICE float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// ---- CTA pairs (tcgen05 cta_group::2): two CTAs of a cluster compute one 256-row tile.  Each loads
// its own 128 rows of A and half of the tile's B into its own shared memory, the even CTA issues
// the M = 256 products for both, and each CTA's tensor memory holds the accumulator rows it owns.
SJ_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of this CTA's shared-memory variable `p` in the shared memory of cluster CTA `rank`.
SJ_DEVICE uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Bounded wait with cluster-scope acquire: the barrier receives arrivals released by the other CTA.
SJ_DEVICE bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const uint64_t start = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (try_once()) return true;
    if (abort != nullptr && *abort) return false;
    if (globaltimer() - start > kWaitLimitNs) {
      record_error(code);
      if (abort != nullptr) *abort = 1;
      return false;
    }
  }
}
SJ_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of a cluster CTA (address from cluster_addr), releasing at cluster scope.
SJ_DEVICE void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Tile load whose completion is counted on the pair's even-CTA barrier `cluster_bar`; the data lands
// in this CTA's shared memory.
SJ_DEVICE void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t cluster_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}
SJ_DEVICE void umma_f16_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` (same offset) in both CTAs of the pair when this thread's pair products complete.
SJ_DEVICE void umma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
// Arrive once on this CTA's `bar` when this thread's pair products complete.
SJ_DEVICE void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
SJ_DEVICE void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
SJ_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
SJ_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

SJ_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
SJ_DEVICE void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
SJ_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
SJ_DEVICE void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Row `lane` of a 32 x 128-byte slab in the SWIZZLE_128B layout: 16-byte chunk j of row r lives
// at r*128 + ((j ^ (r & 7)) * 16).  Writes of 8 consecutive rows hit 8 distinct chunks.
SJ_DEVICE void stage_row128(uint8_t* buf, int lane, const uint32_t (&w)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}
// Half `hb` (chunks 4 hb .. 4 hb + 3) of row `lane` of a 32 x 128-byte SWIZZLE_128B slab.
SJ_DEVICE void stage_half128(uint8_t* buf, int lane, int hb, const uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(buf + lane * 128 + (((4 * hb + j) ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}
// Chunk j of row `lane` of a 32 x 64-byte SWIZZLE_64B slab: r*64 + ((j ^ ((r >> 1) & 3)) * 16).
SJ_DEVICE void stage_chunk64(uint8_t* buf, int lane, int j, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = make_uint4(a, b, c, d);
}
// Row `lane` of a 32 x 64-byte slab in the SWIZZLE_64B layout: chunk j of row r at
// r*64 + ((j ^ ((r >> 1) & 3)) * 16).
SJ_DEVICE void stage_row64(uint8_t* buf, int lane, const uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// One output tile: its rows / columns, reduction k-blocks, and the outer-coordinate offsets of B
// and C (grouped products).
struct Unit {
  int mb, nb, kb_begin, kb_end, b_off, c_off;
};
SJ_DEVICE Unit unit_of(const GemmParams& p, const int* grp, int tile) {
  Unit u;
  const int tiles_mn = p.m_tiles * p.n_tiles;
  if (p.group_mode == 2) {
    const int g = tile / tiles_mn;
    const int rest = tile % tiles_mn;
    u.mb = rest / p.n_tiles;
    u.nb = rest % p.n_tiles;
    u.kb_begin = grp[g] / kBK;
    u.kb_end = grp[g + 1] / kBK;
    u.b_off = 0;
    u.c_off = g * p.c_group_rows;
  } else if (p.group_mode == 1) {
    u.mb = tile / p.n_tiles;
    u.nb = tile % p.n_tiles;
    const int m0 = u.mb * kBM;
    int g = 0;
    while (g + 1 < p.groups && grp[g + 1] <= m0) ++g;
    u.kb_begin = 0;
    u.kb_end = p.kb_total;
    u.b_off = g * p.b_group_rows;
    u.c_off = 0;
  } else {
    const int ks = tile / tiles_mn;
    u.mb = (tile % tiles_mn) / p.n_tiles;
    u.nb = tile % p.n_tiles;
    u.kb_begin = ks * p.kb_per_split;
    u.kb_end = min(u.kb_begin + p.kb_per_split, p.kb_total);
    u.b_off = 0;
    u.c_off = 0;
  }
  return u;
}

// Epilogue kinds, each its own kernel instance (a kernel that carried every epilogue missed in the
// instruction cache on a quarter of its fetches): plain (store, split-K accumulate), SwiGLU,
// residual (with an optional bias), RoPE, bias (with an optional GELU).
constexpr int kEkPlain = 0, kEkSwiglu = 1, kEkResidual = 2, kEkRope = 3, kEkBias = 4;

__host__ __device__ constexpr int epilogue_kind(int epilogue) {
  return epilogue == SJ_EPI_SWIGLU                                            ? kEkSwiglu
         : (epilogue == SJ_EPI_RESIDUAL || epilogue == SJ_EPI_BIAS_RESIDUAL) ? kEkResidual
         : epilogue == SJ_EPI_ROPE                                            ? kEkRope
         : (epilogue == SJ_EPI_BIAS || epilogue == SJ_EPI_BIAS_GELU)         ? kEkBias
                                                                              : kEkPlain;
}

// OPS (residual, RoPE, bias): the epilogue reads operands from global memory (a residual, the RoPE
// table, a bias), which it prefetches into registers before the accumulator is ready; without them
// (plain store, split-K accumulate, SwiGLU) those registers go to overlapping a unit's second TMEM
// read with the arithmetic of its first half (local SwiGLU product 51.5 -> 45.4 us).  CF32: C is f32.
// PAIR: a CTA pair computes 256 x BN tiles (cta_group::2); each CTA holds 128 rows of A and BN / 2
// rows of B per stage, so a stage is a third smaller at BN = 256 and more of them fit.
template <int BN, bool A_MN, bool B_MN, int EK, bool CF32, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_h,
                        const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  static_assert(!PAIR || !A_MN, "CTA pairs take a K-major A");
  constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows (K-major) or columns (MN-major) of B this CTA loads
  constexpr uint32_t B_BYTES = B_ROWS * kBK * 2;
  constexpr uint32_t STAGE_BYTES = Cfg::A_BYTES + B_BYTES;
  constexpr int TILE_M = PAIR ? 2 * kBM : kBM;
  constexpr uint32_t IDESC = umma_idesc_bf16(TILE_M, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
  const int stages = p.stages;
  constexpr bool OPS = EK == kEkResidual || EK == kEkRope || EK == kEkBias;
  constexpr bool swiglu = EK == kEkSwiglu;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging_c = smem + stages * STAGE_BYTES;
  uint8_t* staging_h = staging_c + kStagingC;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging_c + kStagingC + (swiglu ? kStagingH : 0));
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* grp = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(full) + 256);  // [groups + 1]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_mn = p.m_tiles * p.n_tiles;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;       // 0: the CTA that issues the pair's products
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int unit_stride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], (PAIR ? 2 : 1) * kEpilogueWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_c);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  pdl_wait();  // operands may come from the previous kernel
  if (p.group_mode != 0) {
    for (int i = threadIdx.x; i <= p.groups; i += blockDim.x) grp[i] = p.group_rows[i];
    __syncthreads();
  }
  const uint32_t tmem_base = *tmem_slot;
  // work unit -> (split, m tile, n tile); the split index is slowest so that concurrently running
  // CTAs share the K range of their A and B tiles in L2.  Grouped rows: the tile count follows
  // the device-side group offsets.
  const int total_tiles = p.group_mode == 1   ? (grp[p.groups] / kBM) * p.n_tiles
                          : p.group_mode == 2 ? p.groups * tiles_mn
                                              : tiles_mn * p.splits;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = unit0; tile < total_tiles && !*abort_flag; tile += unit_stride) {
        const Unit u = unit_of(p, grp, tile);
        const int m0 = u.mb * TILE_M + static_cast<int>(rank) * kBM;
        const int n0 = u.nb * BN + static_cast<int>(rank) * B_ROWS;
        for (int kb = u.kb_begin; kb < u.kb_end; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t round = static_cast<uint32_t>(it / stages);
          if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort_flag, SJ_DEV_GEMM_PRODUCER_WAIT)) break;
          uint8_t* sa = smem + s * STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          const int k0 = kb * kBK;
          if constexpr (PAIR) {
            // both CTAs' copies complete on the even CTA's barrier, which expects the bytes of both
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
            const uint32_t bar = cluster_addr(&full[s], 0);
            tma_load_2d_pair(sa, &map_a, bar, k0, m0);
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < B_ROWS / 64; ++c) tma_load_2d_pair(sb + c * 8192, &map_b, bar, n0 + 64 * c, k0);
            } else {
              tma_load_2d_pair(sb, &map_b, bar, k0, n0);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            if (A_MN) {
              tma_load_2d(sa, &map_a, &full[s], m0, k0);
              tma_load_2d(sa + 8192, &map_a, &full[s], m0 + 64, k0);
            } else {
              tma_load_2d(sa, &map_a, &full[s], k0, m0);
            }
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < BN / 64; ++c)
                tma_load_2d(sb + c * 8192, &map_b, &full[s], n0 + 64 * c, k0 + u.b_off);
            } else {
              tma_load_2d(sb, &map_b, &full[s], k0, n0 + u.b_off);
            }
          }
        }
      }
      // drain: wait (bounded) for the copies still in flight into the most recent stages (a pair's
      // odd CTA cannot see its copies complete: they are counted on the even CTA's barriers, whose
      // MMA thread waits for every stage before the CTAs meet at the closing cluster barrier)
      if (!PAIR || rank == 0)
        for (int j = max(0, it - stages); j < it; ++j)
          mbar_wait(&full[j % stages], static_cast<uint32_t>(j / stages) & 1u, nullptr, SJ_DEV_GEMM_DRAIN_WAIT);
    }
  } else if (warp == 1) {
    if (lane == 0 && (!PAIR || rank == 0)) {
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = unit0; tile < total_tiles && ok; tile += unit_stride, ++local) {
        const Unit u = unit_of(p, grp, tile);
        const int kb_begin = u.kb_begin, kb_end = u.kb_end;
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        const bool acc_free = PAIR ? mbar_wait_cluster(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag, SJ_DEV_GEMM_MMA_WAIT)
                                   : mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag, SJ_DEV_GEMM_MMA_WAIT);
        if (!acc_free) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t round = static_cast<uint32_t>(it / stages);
          if (!mbar_wait(&full[s], round & 1u, abort_flag, SJ_DEV_GEMM_MMA_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = A_MN ? umma_desc(a_base + kk * 2048, 8192, 1024) : umma_desc(a_base + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? umma_desc(b_base + kk * 2048, 8192, 1024) : umma_desc(b_base + kk * 32, 16, 1024);
            if constexpr (PAIR)
              umma_f16_pair(d_tmem, da, db, IDESC, (kb > kb_begin || kk > 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, da, db, IDESC, (kb > kb_begin || kk > 0) ? 1u : 0u);
          }
          if constexpr (PAIR)
            umma_commit_pair_both(&empty[s]);  // the stage is free in both CTAs
          else
            umma_commit(&empty[s]);
        }
        if (!ok) break;
        if constexpr (PAIR)
          umma_commit_pair_both(&acc_full[buf]);
        else
          umma_commit(&acc_full[buf]);
      }
      // all issued MMAs must retire before TMEM is released
      if constexpr (PAIR)
        umma_commit_pair(drain);
      else
        umma_commit(drain);
      mbar_wait(drain, 0, nullptr, SJ_DEV_GEMM_DRAIN_WAIT);
    }
  } else {
    const int quarter = warp & 3;       // TMEM lanes [32*quarter, 32*quarter+32) belong to this warp
    const int ew = warp - 2;            // epilogue warp 0..7
    const int half = ew >> 2;           // takes column units c with c % 2 == half
    uint8_t* my_c = staging_c + ew * 4096;  // one 32 x 128 B slab per warp
    uint8_t* my_h = staging_h + ew * 2048;
    constexpr bool residual = EK == kEkResidual;
    constexpr bool rope = EK == kEkRope;
    const bool gelu = EK == kEkBias && p.epilogue == SJ_EPI_BIAS_GELU;
    const float* bias = (EK == kEkBias || EK == kEkResidual) ? p.bias : nullptr;
    int local = 0;
    // a pair's epilogue warps release the accumulator on the even CTA's barrier
    const uint32_t acc_empty_bar0 = PAIR ? cluster_addr(&acc_empty[0], 0) : 0u;
    for (int tile = unit0; tile < total_tiles; tile += unit_stride, ++local) {
      const Unit u = unit_of(p, grp, tile);
      const int mb = u.mb, nb = u.nb;
      const bool empty_unit = u.kb_end <= u.kb_begin;  // a group without reduction rows adds nothing
      const int c_off = u.c_off;
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      const int r0 = mb * TILE_M + static_cast<int>(rank) * kBM + quarter * 32;
      const int row = r0 + lane;
      const bool row_ok = row < p.M;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      // Operands of the epilogue that come from global memory (residual rows, the RoPE table row of
      // this lane's position) are read into `pre` before the accumulator is ready, so that their
      // latency overlaps this tile's main loop instead of following each TMEM read.
      uint32_t pre[64];
      if constexpr (CF32) {
        // f32 units are 32 columns; the warp's i-th unit (c = half + 2i) uses pre[32 (i & 1) ...],
        // refilled with unit i + 2 once unit i has consumed it.
        constexpr int kUnits = BN / 64;
        auto load_res = [&](int c, int slot) {
          const int col0 = nb * BN + c * 32;
          if (!residual || !row_ok || col0 >= p.N) return;
          const float* res = static_cast<const float*>(p.aux) + static_cast<size_t>(row) * p.ld_aux + col0;
          if (col0 + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 q = reinterpret_cast<const uint4*>(res)[j];
              pre[32 * slot + 4 * j] = q.x;
              pre[32 * slot + 4 * j + 1] = q.y;
              pre[32 * slot + 4 * j + 2] = q.z;
              pre[32 * slot + 4 * j + 3] = q.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) pre[32 * slot + j] = col0 + j < p.N ? __float_as_uint(res[j]) : 0u;
          }
        };
        load_res(half, 0);
        if (kUnits > 1) load_res(half + 2, 1);
        if (!mbar_wait(&acc_full[buf], use & 1u, abort_flag, SJ_DEV_GEMM_EPILOGUE_WAIT)) break;
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < kUnits; ++i) {
          const int c = half + 2 * i;
          const int col0 = nb * BN + c * 32;
          if (col0 < p.N) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * p.alpha);
            if (bias != nullptr) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float x = __uint_as_float(r[j]) + (col0 + j < p.N ? bias[col0 + j] : 0.f);
                if (gelu) x = gelu_erf(x);
                r[j] = __float_as_uint(x);
              }
            }
            if (residual && row_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(pre[32 * (i & 1) + j]));
            }
            if (i + 2 < kUnits) load_res(c + 4, i & 1);
            uint8_t* sbuf = my_c;
            if (lane == 0) bulk_wait_read0();  // this warp's previous slab has been read out
            __syncwarp();
            stage_row128(sbuf, lane, r);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (r0 < p.M && !empty_unit) {  // boxes are clipped at M and N; a slab wholly past M is not issued
                if (p.epilogue == SJ_EPI_ACCUM)
                  tma_reduce_add_2d(&map_c, sbuf, col0, r0 + c_off);
                else
                  tma_store_2d(&map_c, sbuf, col0, r0 + c_off);
              }
              bulk_commit();
            }
          }
        }
      } else {
        // bf16 units are 64 columns (one RoPE head); a warp has at most two per tile (c = half,
        // half + 2).  Residual: unit i in pre[32 i ...] (64 bf16).  RoPE: the (cos, sin) pairs of this
        // row's position, pre[0..63], shared by every head of the tile.
        constexpr int kUnits = (BN / 64 + 1) / 2;
        const bool rope_tab = rope && row_ok && nb * BN < p.rope_cols;
        if (rope_tab && !p.aux) {  // no table given: (cos, sin) of pos * theta^(-2i/64), i = 0..31
          const float fpos = static_cast<float>(row % p.rope_t);
#pragma unroll
          for (int j = 0; j < 64; j += 2) {
            float sn, cs;
            sincosf(fpos * expf((-2.0f * static_cast<float>(j >> 1) / 64.0f) * p.rope_log_theta), &sn, &cs);
            pre[j] = __float_as_uint(cs);
            pre[j + 1] = __float_as_uint(sn);
          }
        } else if (rope_tab) {
          const uint4* tab = reinterpret_cast<const uint4*>(static_cast<const float*>(p.aux) +
                                                            static_cast<size_t>(row % p.rope_t) * 64);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint4 q = tab[j];
            pre[4 * j] = q.x;
            pre[4 * j + 1] = q.y;
            pre[4 * j + 2] = q.z;
            pre[4 * j + 3] = q.w;
          }
        } else if (residual && row_ok) {
#pragma unroll
          for (int i = 0; i < kUnits; ++i) {
            const int col0 = nb * BN + (half + 2 * i) * 64;
            if (half + 2 * i < BN / 64 && col0 < p.N) {
              const __nv_bfloat16* res =
                  static_cast<const __nv_bfloat16*>(p.aux) + static_cast<size_t>(row) * p.ld_aux + col0;
              if (col0 + 64 <= p.N) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const uint4 q = reinterpret_cast<const uint4*>(res)[j];
                  pre[32 * i + 4 * j] = q.x;
                  pre[32 * i + 4 * j + 1] = q.y;
                  pre[32 * i + 4 * j + 2] = q.z;
                  pre[32 * i + 4 * j + 3] = q.w;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  const float lo = col0 + 2 * j < p.N ? bf2f(res[2 * j]) : 0.f;
                  const float hi = col0 + 2 * j + 1 < p.N ? bf2f(res[2 * j + 1]) : 0.f;
                  pre[32 * i + j] = pack_bf16x2(lo, hi);
                }
              }
            }
          }
        }
        if (!mbar_wait(&acc_full[buf], use & 1u, abort_flag, SJ_DEV_GEMM_EPILOGUE_WAIT)) break;
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < kUnits; ++i) {
          const int c = half + 2 * i;
          const int col0 = nb * BN + c * 64;
          if (c < BN / 64 && col0 < p.N) {
            uint8_t* sbuf = my_c;
            uint8_t* hbuf = my_h;
            if (lane == 0) bulk_wait_read0();  // this warp's previous slabs have been read out
            __syncwarp();
            // two halves of 32 columns: (RoPE pairs, SwiGLU gate|up blocks and residual all stay
            // within a half)
            uint32_t rr[2][32];
            if constexpr (!OPS) {  // both halves requested; the second completes during the first's arithmetic
              tmem_ld_32x32b_x32(taddr + c * 64, rr[0]);
              tmem_wait_ld();
              tmem_ld_32x32b_x32(taddr + c * 64 + 32, rr[1]);
            }
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
              uint32_t r[32];
              if constexpr (OPS) {
                tmem_ld_32x32b_x32(taddr + c * 64 + 32 * hb, r);
                tmem_wait_ld();
              } else {
                if (hb == 1) tmem_wait_ld_dep(rr[1]);
#pragma unroll
                for (int j = 0; j < 32; ++j) r[j] = rr[hb][j];
              }
              float v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
              if (bias != nullptr) {
                const int cb = col0 + 32 * hb;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  v[j] += cb + j < p.N ? bias[cb + j] : 0.f;
                  if (gelu) v[j] = gelu_erf(v[j]);
                }
              }
              uint32_t w[16];
              if constexpr (swiglu) {
                // columns come as blocks of 16 gate then the same 16 up features; g and u are
                // rounded to bf16 before h = silu(g) * u (projection.py:464-470)
                uint32_t hw[8];
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                  float hv[2];
#pragma unroll
                  for (int e = 0; e < 2; ++e) {
                    const float g = round_bf16(v[j + e]);
                    const float u = round_bf16(v[16 + j + e]);
                    // silu(g) = g sigmoid(g) = g (1/2 + tanh(g/2) / 2): one special-function op
                    hv[e] = g * fmaf(0.5f, tanh_approx(0.5f * g), 0.5f) * u;
                  }
                  hw[j >> 1] = pack_bf16x2(hv[0], hv[1]);
                }
                stage_chunk64(hbuf, lane, 2 * hb, hw[0], hw[1], hw[2], hw[3]);
                stage_chunk64(hbuf, lane, 2 * hb + 1, hw[4], hw[5], hw[6], hw[7]);
              } else if constexpr (rope) {
                if (col0 < p.rope_cols && row_ok) {
#pragma unroll
                  for (int j = 0; j < 32; j += 2) {  // pair (32 hb + j) / 2 of the row's (cos, sin)
                    const float cs = __uint_as_float(pre[32 * hb + j]);
                    const float sn = __uint_as_float(pre[32 * hb + j + 1]);
                    const float a = v[j], b = v[j + 1];
                    v[j] = a * cs - b * sn;
                    v[j + 1] = a * sn + b * cs;
                  }
                }
              } else if constexpr (residual) {
                if (row_ok) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    const float2 a = unpack_bf16x2(pre[32 * i + 16 * hb + j]);
                    v[2 * j] += a.x;
                    v[2 * j + 1] += a.y;
                  }
                }
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
              stage_half128(sbuf, lane, hb, w);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (r0 < p.M) {
                tma_store_2d(&map_c, sbuf, col0, r0);
                if (swiglu) tma_store_2d(&map_h, hbuf, col0 / 2, r0);
              }
              bulk_commit();
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(acc_empty_bar0 + 8u * static_cast<uint32_t>(buf));
        else
          mbar_arrive(&acc_empty[buf]);
      }
    }
    if (lane == 0) bulk_wait_all();  // staged slabs must be read out before the CTA exits
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the even CTA's products into this CTA's TMEM have retired
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
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

// 2-D tensor map: `inner` contiguous elements per row, `outer` rows, row stride `ld` elements.
static int make_map(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int esize, uint64_t inner,
                    uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SJ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(esize)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SJ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SJ_OK;
}

int tensor_map(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SJ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (rank < 1 || rank > 5) return fail(SJ_ERR_ARGUMENT, "tensor map rank %d", rank);
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, rank, const_cast<void*>(ptr), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SJ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SJ_OK;
}

int bf16_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
             uint32_t box_outer) {
  return make_map(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, outer, ld, box_inner, box_outer,
                  CU_TENSOR_MAP_SWIZZLE_128B);
}

// `kernel` over clusters of two CTAs (programmatic serialization as in launch()).
template <typename... KArgs, typename... Args>
static void launch_pairs(void (*kernel)(KArgs...), int grid, int smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  [&](KArgs... coerced) {
    void* pargs[] = {const_cast<void*>(static_cast<const void*>(&coerced))...};
    cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), pargs);
  }(std::forward<Args>(args)...);
}

// Clusters of two CTAs (at the GEMM's thread count and the largest shared-memory size) that can be
// resident at once on the current device: the pair kernel's persistent grid.  Asked once per device.
static int max_pair_clusters() {
  static std::atomic<int> cache[KernelAttrOnce::kMaxDevices];
  static KernelAttrOnce attr_once;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const bool tracked = dev >= 0 && dev < KernelAttrOnce::kMaxDevices;
  if (tracked) {
    const int v = cache[dev].load(std::memory_order_acquire);
    if (v > 0) return v;
  }
  auto kernel = gemm_tcgen05_kernel<256, false, false, kEkPlain, false, true>;
  if (ensure_max_smem(attr_once, reinterpret_cast<const void*>(kernel), kSmemLimit, "gemm shared-memory attribute") !=
      SJ_OK)
    return 0;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * sm_count());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemLimit;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kernel), &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (tracked && n > 0) cache[dev].store(n, std::memory_order_release);
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EK, bool CF32, bool PAIR>
static int launch_gemm(const CUtensorMap* maps, const GemmParams& p, int grid, int smem, cudaStream_t stream) {
  auto kernel = gemm_tcgen05_kernel<BN, A_MN, B_MN, EK, CF32, PAIR>;
  static KernelAttrOnce attr_once;  // one per template instance
  const int attr_rc = ensure_max_smem(attr_once, reinterpret_cast<const void*>(kernel), kSmemLimit,
                                      "gemm shared-memory attribute");
  if (attr_rc != SJ_OK) return attr_rc;
  if constexpr (PAIR)
    launch_pairs(kernel, grid, smem, stream, maps[0], maps[1], maps[2], maps[3], p);
  else
    launch(kernel, grid, kThreads, smem, stream, maps[0], maps[1], maps[2], maps[3], p);
  SJ_LAUNCH_CHECK("gemm launch");
  return SJ_OK;
}

// Instances: the plain epilogue for every operand major and C type; the others (forward products,
// A K-major) for the C types they take -- SwiGLU and RoPE write bf16, residual and bias either.
template <int BN, bool A_MN, bool B_MN, bool PAIR>
static int dispatch_epilogue(const CUtensorMap* maps, const GemmParams& p, int grid, int smem, cudaStream_t s) {
  const int ek = epilogue_kind(p.epilogue);
  if constexpr (PAIR) {  // pair instances: K-major A, BN = 256, plain and SwiGLU epilogues
    static_assert(BN == 256 && !A_MN, "CTA pairs are instantiated at BN = 256 with a K-major A");
    if (ek == kEkPlain)
      return p.c_f32 ? launch_gemm<BN, false, B_MN, kEkPlain, true, true>(maps, p, grid, smem, s)
                     : launch_gemm<BN, false, B_MN, kEkPlain, false, true>(maps, p, grid, smem, s);
    if (ek == kEkSwiglu && !p.c_f32)
      return launch_gemm<BN, false, B_MN, kEkSwiglu, false, true>(maps, p, grid, smem, s);
    return fail(SJ_ERR_UNSUPPORTED, "sj_gemm: no CTA-pair kernel for epilogue %d", p.epilogue);
  } else {
    if (ek == kEkPlain)
      return p.c_f32 ? launch_gemm<BN, A_MN, B_MN, kEkPlain, true, false>(maps, p, grid, smem, s)
                     : launch_gemm<BN, A_MN, B_MN, kEkPlain, false, false>(maps, p, grid, smem, s);
    if constexpr (!A_MN) {
      if (ek == kEkSwiglu && !p.c_f32)
        return launch_gemm<BN, false, B_MN, kEkSwiglu, false, false>(maps, p, grid, smem, s);
      if (ek == kEkRope && !p.c_f32) return launch_gemm<BN, false, B_MN, kEkRope, false, false>(maps, p, grid, smem, s);
      if (ek == kEkResidual)
        return p.c_f32 ? launch_gemm<BN, false, B_MN, kEkResidual, true, false>(maps, p, grid, smem, s)
                       : launch_gemm<BN, false, B_MN, kEkResidual, false, false>(maps, p, grid, smem, s);
      if (ek == kEkBias)
        return p.c_f32 ? launch_gemm<BN, false, B_MN, kEkBias, true, false>(maps, p, grid, smem, s)
                       : launch_gemm<BN, false, B_MN, kEkBias, false, false>(maps, p, grid, smem, s);
    }
    return fail(SJ_ERR_UNSUPPORTED, "sj_gemm: epilogue %d with an M-major A or this C type", p.epilogue);
  }
}

template <int BN>
static int dispatch_majors(bool a_mn, bool b_mn, bool pair, const CUtensorMap* maps, const GemmParams& p, int grid,
                           int smem, cudaStream_t s) {
  if (pair) {
    if constexpr (BN == 256) {
      if (!a_mn)
        return b_mn ? dispatch_epilogue<BN, false, true, true>(maps, p, grid, smem, s)
                    : dispatch_epilogue<BN, false, false, true>(maps, p, grid, smem, s);
    }
    return fail(SJ_ERR_UNSUPPORTED, "sj_gemm: no CTA-pair kernel for this tile or operand layout");
  }
  if (!a_mn && b_mn) return dispatch_epilogue<BN, false, true, false>(maps, p, grid, smem, s);
  if (!a_mn && !b_mn) return dispatch_epilogue<BN, false, false, false>(maps, p, grid, smem, s);
  if (a_mn && b_mn) return dispatch_epilogue<BN, true, true, false>(maps, p, grid, smem, s);
  return dispatch_epilogue<BN, true, false, false>(maps, p, grid, smem, s);
}

}  // namespace sj

namespace sj {

struct Grouping {
  const int* rows = nullptr;  // device [groups + 1]
  int groups = 0, mode = 0, b_rows = 0, c_rows = 0;
};

static int gemm_impl(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c, int ldc,
                     int c_dtype, int m, int n, int k, int epilogue, float alpha, void* aux, int ld_aux,
                     int rope_cols, int rope_t, float rope_theta, int split_k, const float* bias, void* stream,
                     const Grouping& grouping = Grouping(), int* plan = nullptr) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(SJ_ERR_SHAPE, "sj_gemm: empty problem %dx%dx%d", m, n, k);
  if (!a || !b || !c) return fail(SJ_ERR_ARGUMENT, "sj_gemm: null operand");
  if (!aligned16(a) || !aligned16(b) || !aligned16(c))
    return fail(SJ_ERR_ARGUMENT, "sj_gemm: A, B and C must be 16-byte aligned");
  if ((lda % 8) || (ldb % 8)) return fail(SJ_ERR_ARGUMENT, "sj_gemm: lda/ldb must be multiples of 8 elements");
  const int a_rows_min = a_trans ? m : k, b_rows_min = b_trans ? k : n;
  if (lda < a_rows_min || ldb < b_rows_min || ldc < n)
    return fail(SJ_ERR_SHAPE, "sj_gemm: leading dimension smaller than the matrix width");
  if (c_dtype != SJ_BF16 && c_dtype != SJ_F32) return fail(SJ_ERR_ARGUMENT, "sj_gemm: C must be bf16 or f32");
  if ((c_dtype == SJ_BF16 && ldc % 8) || (c_dtype == SJ_F32 && ldc % 4))
    return fail(SJ_ERR_ARGUMENT, "sj_gemm: C rows must be 16-byte multiples");
  switch (epilogue) {
    case SJ_EPI_STORE:
      break;
    case SJ_EPI_ACCUM:
      if (c_dtype != SJ_F32) return fail(SJ_ERR_ARGUMENT, "sj_gemm: ACCUM needs an f32 C");
      break;
    case SJ_EPI_RESIDUAL:
      if (!aux || !aligned16(aux) || (ld_aux % 8))
        return fail(SJ_ERR_ARGUMENT, "sj_gemm: RESIDUAL needs a 16-byte aligned aux (same dtype as C)");
      break;
    case SJ_EPI_SWIGLU:
      if (c_dtype != SJ_BF16 || !aux || !aligned16(aux) || (n % 64) || (ld_aux % 8))
        return fail(SJ_ERR_ARGUMENT, "sj_gemm: SWIGLU needs bf16 C, an aligned aux and N %% 64 == 0");
      break;
    case SJ_EPI_ROPE:
      if (c_dtype != SJ_BF16 || rope_t <= 0 || (rope_cols % 64) || (rope_theta <= 0.f && !aux) ||
          (aux && !aligned16(aux)))
        return fail(SJ_ERR_ARGUMENT,
                    "sj_gemm: ROPE needs bf16 C, rope_t > 0, rope_cols %% 64 == 0 and a table or theta");
      break;
    case SJ_EPI_BIAS:
    case SJ_EPI_BIAS_GELU:
      if (!bias || !aligned16(bias)) return fail(SJ_ERR_ARGUMENT, "sj_gemm_bias: a 16-byte aligned bias is required");
      break;
    case SJ_EPI_BIAS_RESIDUAL:
      if (!bias || !aligned16(bias) || !aux || !aligned16(aux) || (ld_aux % 8))
        return fail(SJ_ERR_ARGUMENT, "sj_gemm_bias: BIAS_RESIDUAL needs an aligned bias and aux (same dtype as C)");
      break;
    default:
      return fail(SJ_ERR_ARGUMENT, "sj_gemm: unknown epilogue %d", epilogue);
  }
  if (split_k > 1 && epilogue != SJ_EPI_ACCUM) return fail(SJ_ERR_ARGUMENT, "sj_gemm: split_k needs ACCUM");

  const int sms = sm_count();
  const int m_tiles = (m + kBM - 1) / kBM;
  const int kb_total = (k + kBK - 1) / kBK;
  // Tile width and split count from cost models fitted to B200 measurements of the step's shapes.
  // Per FLOP a 128 x 256 tile is the most efficient (cost x1.0 per k-block), 128 x 192 costs 0.83
  // of its k-block time for 0.75 of its work, 128 x 128 about 0.8-0.88 for half of it.
  int bn = 128, splits = 1;
  bool pair = false;
  const int candidates[3] = {128, 192, 256};
  if (epilogue == SJ_EPI_ACCUM) {
    // Weight gradients: time ~ waves x (k-blocks per unit + epilogue) x (k-block cost); split-K
    // shortens units at the price of a reduce-add epilogue each.  N <= 128: one 128-wide tile.
    const double weight[3] = {0.88, 0.83, 1.0};
    const double epi_blocks = 3.0;
    double best = 1e30;
    for (int ci = 0; ci < 3; ++ci) {
      const int cbn = candidates[ci];
      if ((n > 128) != (cbn > 128)) continue;
      const int tiles = m_tiles * ((n + cbn - 1) / cbn);
      int sp_lo = 1, sp_hi = 1;
      if (split_k > 0)
        sp_lo = sp_hi = std::min(split_k, kb_total);
      else
        sp_hi = std::max(1, std::min(kb_total / 4, 4 * sms / std::max(tiles, 1) + 1));
      for (int sp = sp_lo; sp <= sp_hi; ++sp) {
        const int kb_unit = (kb_total + sp - 1) / sp;
        const int waves = (tiles * sp + sms - 1) / sms;
        const double cost = waves * (kb_unit + epi_blocks) * weight[ci];
        if (cost < best - 1e-9) {
          best = cost;
          bn = cbn;
          splits = sp;
        }
      }
    }
  } else {
    // A CTA overlaps the epilogue of one tile with the main loop of the next, so a CTA with t tiles
    // takes about t x max(ML, EP) + min(ML, EP): ML = k-blocks x k-block cost of the width, EP = the
    // epilogue's traffic in the same unit, (BN / 256) per byte that one output column moves per row
    // (C, plus the residual read or the SwiGLU h), and for RoPE a table row per tile shared by
    // its BN / 64 heads.
    const double weight[3] = {0.8, 0.83, 1.0};
    const int c_bytes = c_dtype == SJ_F32 ? 4 : 2;
    const double col_bytes = (epilogue == SJ_EPI_RESIDUAL || epilogue == SJ_EPI_BIAS_RESIDUAL) ? 2.0 * c_bytes
                             : epilogue == SJ_EPI_SWIGLU ? 3.0
                                                         : static_cast<double>(c_bytes);
    double best = 1e30;
    for (int ci = 0; ci < 3; ++ci) {
      const int cbn = candidates[ci];
      if (n <= 128 && cbn > 128) continue;
      const int tiles = m_tiles * ((n + cbn - 1) / cbn);
      const int per_cta = (tiles + sms - 1) / sms;
      const double ml = kb_total * weight[ci];
      const double ep = (cbn / 256.0) * col_bytes + (epilogue == SJ_EPI_ROPE ? 2.0 * 256.0 / cbn : 0.0);
      const double cost = per_cta * std::max(ml, ep) + std::min(ml, ep);
      if (cost < best - 1e-9) {
        best = cost;
        bn = cbn;
      }
    }
    // CTA pairs: a 256 x 256 pair tile moves a third less operand data per CTA and k-block than
    // a 128 x 256 tile (A: 128 rows, B: 128 rows), which shortens the k-block from about 920 to
    // 780 cycles at K = 768 on B200.  That pays only where the main loop dominates: the gate/up
    // product of the global stage (4096 x 4096 x 768: 33.1 -> 31.7 us).  Where the epilogue or
    // the tile count bounds the time (K = 256 products, N = 768 / 1280 outputs) the pair is
    // slower, since a pair's accumulator is free only when both CTAs' epilogues are done.
    pair = !a_trans && grouping.mode == 0 && bn == 256 && m >= 8 * kBM && n >= 2048 && kb_total >= 12 &&
           (epilogue == SJ_EPI_STORE || epilogue == SJ_EPI_SWIGLU) && max_pair_clusters() > 0;
  }
  if (grouping.mode != 0) splits = 1;
  const int n_tiles = (n + bn - 1) / bn;
  const int kb_per_split = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per_split - 1) / kb_per_split;  // no empty split

  if (plan != nullptr) {  // the tile plan only (sj_gemm_plan)
    plan[0] = bn;
    plan[1] = splits;
    plan[2] = pair ? 1 : 0;
    return SJ_OK;
  }
  const int stage_bytes = (kBM + (pair ? bn / 2 : bn)) * kBK * 2;
  const int staging = kStagingC + (epilogue == SJ_EPI_SWIGLU ? kStagingH : 0);
  // four stages for single CTAs: more never helped on B200 and cost up to 20% on large problems
  const int stages = std::min(pair ? kPairStages : 4, (kSmemLimit - 1024 - kBarrierBytes - staging) / stage_bytes);
  if (stages < 2) return fail(SJ_ERR_CAPACITY, "sj_gemm: shared memory too small for the pipeline");
  const int smem = 1024 + stages * stage_bytes + staging + kBarrierBytes;

  CUtensorMap maps[4];
  int rc;
  if (!a_trans)
    rc = bf16_map(&maps[0], a, static_cast<uint64_t>(k), static_cast<uint64_t>(m), lda, 64, 128);
  else
    rc = bf16_map(&maps[0], a, static_cast<uint64_t>(m), static_cast<uint64_t>(k), lda, 64, 64);
  if (rc) return rc;
  if (b_trans)
    rc = bf16_map(&maps[1], b, static_cast<uint64_t>(k),
                  static_cast<uint64_t>(grouping.mode == 1 ? grouping.groups * grouping.b_rows : n), ldb, 64,
                  static_cast<uint32_t>(pair ? bn / 2 : bn));
  else
    rc = bf16_map(&maps[1], b, static_cast<uint64_t>(n),
                  static_cast<uint64_t>(grouping.mode == 1 ? grouping.groups * grouping.b_rows : k), ldb, 64, 64);
  if (rc) return rc;
  if (c_dtype == SJ_F32)
    rc = make_map(&maps[2], c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, static_cast<uint64_t>(n),
                  static_cast<uint64_t>(grouping.mode == 2 ? grouping.groups * grouping.c_rows : m),
                  ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = make_map(&maps[2], c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<uint64_t>(n), static_cast<uint64_t>(m),
                  ldc, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (epilogue == SJ_EPI_SWIGLU)
    rc = make_map(&maps[3], aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<uint64_t>(n / 2),
                  static_cast<uint64_t>(m), ld_aux, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  else
    maps[3] = maps[2];
  if (rc) return rc;

  GemmParams p;
  p.M = m;
  p.N = n;
  p.K = k;
  p.m_tiles = pair ? (m + 2 * kBM - 1) / (2 * kBM) : m_tiles;
  p.n_tiles = n_tiles;
  p.splits = splits;
  p.kb_per_split = kb_per_split;
  p.kb_total = kb_total;
  p.stages = stages;
  p.c_f32 = c_dtype == SJ_F32;
  p.epilogue = epilogue;
  p.alpha = alpha;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.rope_cols = rope_cols;
  p.rope_t = rope_t > 0 ? rope_t : 1;
  p.rope_log_theta = rope_theta > 0.f ? logf(rope_theta) : 0.f;
  p.bias = bias;
  p.group_rows = grouping.rows;
  p.groups = grouping.groups;
  p.group_mode = grouping.mode;
  p.b_group_rows = grouping.b_rows;
  p.c_group_rows = grouping.c_rows;
  const int total = p.m_tiles * n_tiles * splits * (grouping.mode == 2 ? grouping.groups : 1);
  const int grid = pair ? 2 * std::min(total, max_pair_clusters()) : std::min(total, sms);
  const bool a_mn = a_trans != 0;   // A stored [K, M]
  const bool b_mn = b_trans == 0;   // B stored [K, N]
  if (bn == 256) return dispatch_majors<256>(a_mn, b_mn, pair, maps, p, grid, smem, as_stream(stream));
  if (bn == 192) return dispatch_majors<192>(a_mn, b_mn, pair, maps, p, grid, smem, as_stream(stream));
  return dispatch_majors<128>(a_mn, b_mn, pair, maps, p, grid, smem, as_stream(stream));
}

}  // namespace sj

extern "C" int sj_gemm_plan(int m, int n, int k, int a_trans, int b_trans, int c_dtype, int epilogue, int split_k,
                            int* plan) {
  if (!plan) return sj::fail(SJ_ERR_ARGUMENT, "sj_gemm_plan: null plan");
  // operands are never read: aligned stand-in addresses pass the argument checks
  void* dummy = reinterpret_cast<void*>(static_cast<uintptr_t>(256));
  const int lda = a_trans ? m : k, ldb = b_trans ? k : n;
  return sj::gemm_impl(dummy, (lda + 7) / 8 * 8, a_trans, dummy, (ldb + 7) / 8 * 8, b_trans, dummy, (n + 7) / 8 * 8,
                       c_dtype, m, n, k, epilogue, 1.0f, dummy, (n + 7) / 8 * 8, 64, 1, 1.0f, split_k,
                       static_cast<const float*>(dummy), nullptr, sj::Grouping(), plan);
}

extern "C" int sj_gemm(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c, int ldc,
                       int c_dtype, int m, int n, int k, int epilogue, float alpha, void* aux, int ld_aux,
                       int rope_cols, int rope_t, float rope_theta, int split_k, void* stream) {
  if (epilogue >= SJ_EPI_BIAS && epilogue <= SJ_EPI_BIAS_RESIDUAL)
    return sj::fail(SJ_ERR_ARGUMENT, "sj_gemm: bias epilogues go through sj_gemm_bias");
  return sj::gemm_impl(a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epilogue, alpha, aux, ld_aux,
                       rope_cols, rope_t, rope_theta, split_k, nullptr, stream);
}

extern "C" int sj_gemm_grouped(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c,
                               int ldc, int c_dtype, int m, int n, int k, int epilogue, void* aux, int ld_aux,
                               int groups, const int32_t* group_rows, int group_mode, int b_group_rows,
                               int c_group_rows, void* stream) {
  using namespace sj;
  if (groups <= 0 || groups > kMaxGroups || !group_rows)
    return fail(SJ_ERR_ARGUMENT, "sj_gemm_grouped: 1..%d groups and their device row offsets required", kMaxGroups);
  Grouping gp;
  gp.rows = group_rows;
  gp.groups = groups;
  gp.mode = group_mode;
  gp.b_rows = b_group_rows;
  gp.c_rows = c_group_rows;
  if (group_mode == 1) {
    if (epilogue != SJ_EPI_STORE && epilogue != SJ_EPI_SWIGLU)
      return fail(SJ_ERR_ARGUMENT, "sj_gemm_grouped: grouped rows take STORE or SWIGLU");
    if (m % kBM) return fail(SJ_ERR_SHAPE, "sj_gemm_grouped: row capacity %d must be a multiple of 128", m);
    if (b_group_rows != (b_trans ? n : k))
      return fail(SJ_ERR_SHAPE, "sj_gemm_grouped: b_group_rows must be the stored rows of one group's B");
  } else if (group_mode == 2) {
    if (epilogue != SJ_EPI_ACCUM || c_dtype != SJ_F32 || !a_trans || b_trans)
      return fail(SJ_ERR_ARGUMENT, "sj_gemm_grouped: grouped reduction is C_g += A_g^T B_g (f32 ACCUM)");
    if (k % kBM) return fail(SJ_ERR_SHAPE, "sj_gemm_grouped: reduction capacity %d must be a multiple of 128", k);
    if (c_group_rows < m) return fail(SJ_ERR_SHAPE, "sj_gemm_grouped: c_group_rows below the rows of one group's C");
  } else {
    return fail(SJ_ERR_ARGUMENT, "sj_gemm_grouped: group_mode must be 1 (rows) or 2 (reduction)");
  }
  return gemm_impl(a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epilogue, 1.0f, aux, ld_aux, 0, 0, 0.f,
                   1, nullptr, stream, gp);
}

extern "C" int sj_gemm_bias(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c,
                            int ldc, int c_dtype, int m, int n, int k, int epilogue, float alpha, const float* bias,
                            void* aux, int ld_aux, void* stream) {
  if (epilogue < SJ_EPI_BIAS || epilogue > SJ_EPI_BIAS_RESIDUAL)
    return sj::fail(SJ_ERR_ARGUMENT, "sj_gemm_bias: epilogue %d is not a bias epilogue", epilogue);
  return sj::gemm_impl(a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epilogue, alpha, aux, ld_aux, 0,
                       0, 0.f, 0, bias, stream);
}
