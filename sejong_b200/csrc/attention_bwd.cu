// Causal grouped-query attention backward on the 5th-generation tensor cores, head dim 64, optional
// sliding window.
//
// Restates python/sejong_kernels/ops/hierarchy.py:42-104 (the dQ and dK/dV programs): with
// P = exp(S scale - LSE) and dS = P (dP - Delta) scale, dV = P^T dO, dK = dS^T Q, dQ = dS K; the
// inverse RoPE rotation of the tape's backward (crates/sejong-gpu/src/graph.rs:879-882) is applied
// to dQ and dK on the way out.
//
// Persistent: one CTA per SM walks work items (batch, kv head, 128-key tile).  An item visits every
// query head of its group and every query tile its keys are visible to, so dK and dV of the kv head
// accumulate in TMEM across the whole group and are written once (no partials).  18 warps:
//   warp 0      TMA: the item's K and V tiles (double-buffered by item), and per step the Q and dO
//               tiles and the step's 128 LSE and Delta values (2-deep ring; the delta kernel lays
//               both out per head, contiguous over the sequence).
//   warp 1      TMEM owner and MMA issuer, per step g:
//                 S^T_g = K Q_g^T and dP^T_g = V dO_g^T (M128 N128 K64) into TMEM,
//                 then, once P^T_g and dS^T_g are in shared memory,
//                 dV += P^T_g dO_g, dK += dS^T_g Q_g (M128 N64 K128, accumulated in TMEM) and
//                 dQ_g = dS_g K (the dS^T buffer read as an MN-major operand) into one of two TMEM
//                 buffers.
//               S^T_{g+1} / dP^T_{g+1} are issued before waiting for P^T_g, so the two overlap.
//   warps 2-17  elementwise: thread <-> key row (TMEM lane), four threads per row, 32 query columns
//               each, in two chunks of 16: P^T and dS^T computed from TMEM (the first chunk while the
//               previous step's MMAs still read the shared-memory buffers), then stored in bf16 into
//               K-major 128-byte-swizzled shared memory; after handing them over, the previous
//               step's dQ goes through the warp's 2 KB slab into an f32 accumulator [rows, hq*64] by
//               a TMA reduce-add (attn_dq_finish_kernel applies the inverse RoPE and writes bf16)
//               and, at the end of an item, dK and dV likewise into f32 partial sums (items split by
//               head) or, rotated back, to global bf16.
// Every wait is bounded (SJ_DEV_ATTN_WAIT in the device error word).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {

constexpr int kBT = 128;                          // keys per item, queries per step
constexpr int kBD = 64;                           // head dim
constexpr int kEwWarps = 16;                     // 4 per TMEM lane quarter
constexpr int kEwCols = kBT / (kEwWarps / 4);    // 32 query columns of P^T / dS^T per thread
constexpr int kEwHead = kBD / (kEwWarps / 4);    // 16 head columns of dQ / dK / dV per thread
static_assert(kEwCols == 32 && kEwHead == 16, "elementwise mapping");
constexpr int kBwdThreads = 32 * (2 + kEwWarps);
constexpr int kTile = kBT * kBD * 2;              // 16 KB: 128 rows x 128 B
// shared memory: K | V | Q ring | dO ring | P^T | dS^T | LSE/Delta ring | staging slabs | barriers
// K, V tiles per item: two, because the MMA thread issues an item's last dV / dK / dQ after the
// next item's first S^T / dP^T, which need that item's K and V already loaded.
constexpr int kKvStages = 2;
constexpr int kQdStages = 2;                     // Q, dO tiles (and LSE, Delta) per step
constexpr int kOffKb = 0;
constexpr int kOffVb = kOffKb + kKvStages * kTile;
constexpr int kOffQb = kOffVb + kKvStages * kTile;
constexpr int kOffDOb = kOffQb + kQdStages * kTile;
constexpr int kOffPt = kOffDOb + kQdStages * kTile;  // 32 KB: two 64-query halves
constexpr int kOffDSt = kOffPt + 2 * kTile;          // 32 KB
constexpr int kOffLd = kOffDSt + 2 * kTile;          // [kQdStages][LSE*log2e 128 | Delta 128] f32
static_assert(kKvStages == 2 && kQdStages <= 4, "K/V double buffer; barrier slots");
constexpr uint32_t kTmemColsB = 512;
constexpr uint32_t kColSt = 0, kColDPt = 128, kColDV = 256, kColDK = 320, kColDQ = 384;  // dQ: 2 x 64
constexpr float kLog2eB = 1.4426950408889634f;

struct BwdParams {
  int t, hq, hk, window, batch, nkt, items;
  float scale, scale_log2;
  const float* lse_t;    // [hq][batch][tpad]: LSE * log2(e), per head contiguous over the sequence
  const float* delta_t;  // [hq][batch][tpad]: Delta
  int tpad;              // t rounded up to 128
  float* dq_acc;         // [rows, hq * 64] f32, zeroed
  __nv_bfloat16 *dk, *dv;
  int lddk, lddv;
  const float2* rope_tab;  // [t][32] (cos, sin) or null
  float rope_log_theta;    // > 0 when no table: angles evaluated inline
  int hsplit;              // head slices per (batch, kv head, key tile): 1, or the group size
  float* dkv_acc;          // hsplit > 1: [rows, hk, dK 64 | dV 64] f32, zeroed; null otherwise
};

SJ_DEVICE float ex2b(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Item -> (batch, kv head, key tile, head slice) and its query range per head: heaviest first (the
// first key tiles see the most causal query tiles).  An item visits the query heads
// [h0, h0 + gh) of its GQA group: all of them (hsplit 1) or one (hsplit = group).
struct BItem {
  int b, kvh, kt, k0, qt_lo, nq, h0, gh;
};
SJ_DEVICE BItem decode_bitem(const BwdParams& p, int item) {
  BItem it;
  const int bk = p.batch * p.hk * p.hsplit;
  const int rest = item % bk;
  it.kt = item / bk;
  it.b = rest / (p.hk * p.hsplit);
  it.kvh = (rest / p.hsplit) % p.hk;
  it.gh = p.hq / p.hk / p.hsplit;
  it.h0 = (rest % p.hsplit) * it.gh;
  it.k0 = it.kt * kBT;
  const int nqt = (p.t + kBT - 1) / kBT;
  it.qt_lo = it.kt;
  const int qt_hi = p.window > 0 ? min(nqt - 1, (it.k0 + kBT - 1 + p.window - 1) / kBT) : nqt - 1;
  it.nq = qt_hi - it.qt_lo + 1;
  return it;
}

// (cos, sin) of the RoPE angle of position pos, pair i (head dim 64).
SJ_DEVICE float2 rope_cs(const float2* tab, float log_theta, int pos, int i) {
  if (tab != nullptr) return tab[static_cast<size_t>(pos) * 32 + i];
  float s, c;
  sincosf(static_cast<float>(pos) * expf((-2.0f * static_cast<float>(i) / 64.0f) * log_theta), &s, &c);
  return make_float2(c, s);
}

// 1-D bulk copy global -> shared completing on an mbarrier (16-byte aligned, size a multiple of 16).
SJ_DEVICE void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

SJ_DEVICE void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
SJ_DEVICE void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
SJ_DEVICE void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
SJ_DEVICE void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
SJ_DEVICE void bulk_wait_all_groups() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
SJ_DEVICE void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// Row `lane` (16 f32, 64 bytes) of a 32 x 64-byte SWIZZLE_64B slab.
SJ_DEVICE void stage_f32x16(uint8_t* slab, int lane, const uint32_t (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(slab + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// General kernel's staging: a 2 KB slab per elementwise warp (32 rows x 16 f32) from which TMA
// reduce-adds dQ (and, with the items split by head, the dK / dV partials) into their f32
// accumulators -- thread-per-row vector reductions touched 32 cache lines per instruction.
constexpr int kGSlab = 2048;
constexpr int kGOffStage = kOffLd + kQdStages * 2 * kBT * 4;
constexpr int kGOffBar = kGOffStage + kEwWarps * kGSlab;
constexpr int kGLayout = kGOffBar + 256;
constexpr int kSmemGen = 232448;  // the per-block maximum; what the layout leaves is alignment slack
static_assert(kGOffStage % 1024 == 0 && kGLayout <= kSmemGen, "general attention backward shared memory");

}  // namespace

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_do,
                       const __grid_constant__ CUtensorMap map_dq, const __grid_constant__ CUtensorMap map_dkv,
                       const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad + kGLayout > kSmemGen) {  // uniform over the CTA, before any barrier or TMEM use
    if (threadIdx.x == 0) record_error(SJ_DEV_SMEM_ALIGN);
    pdl_wait();
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGOffBar);
  uint64_t* kv_full = bars;          // kKvStages (<= 2)
  uint64_t* kv_empty = bars + 2;     // kKvStages
  uint64_t* qd_full = bars + 4;      // kQdStages (<= 4)
  uint64_t* qd_empty = bars + 8;     // kQdStages
  uint64_t* sp_full = bars + 12;     // 1: S^T, dP^T in TMEM
  uint64_t* sp_empty = bars + 13;    // 1: elementwise warps have them in registers
  uint64_t* ps_full = bars + 14;     // 1: P^T, dS^T in shared memory
  uint64_t* ps_empty = bars + 15;    // 1: their MMAs are done
  uint64_t* dq_empty = bars + 16;    // 2: dQ_g (TMEM buffer g & 1) read out
  uint64_t* acc_empty = bars + 18;   // 1: an item's dK / dV read out
  uint64_t* drain = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* ldbuf = reinterpret_cast<float*>(smem + kOffLd);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = p.hq / p.hk;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < kQdStages; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(sp_empty, kEwWarps);
    mbar_init(ps_full, kEwWarps);
    mbar_init(ps_empty, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&dq_empty[i], kEwWarps);
    mbar_init(acc_empty, kEwWarps);  // the elementwise warps read dK / dV out
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_q);
    tma_prefetch_map(&map_k);
    tma_prefetch_map(&map_v);
    tma_prefetch_map(&map_do);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemColsB);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // operands may come from the previous kernel
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (whole warp)
    int n = 0, g = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++n) {
      const BItem it = decode_bitem(p, item);
      const int row_base = it.b * p.t;
      const int ks = n % kKvStages;
      if (lane == 0) {
        ok = mbar_wait_sleep(&kv_empty[ks], ((n / kKvStages) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT);
        if (ok) {
          mbar_arrive_expect_tx(&kv_full[ks], 2 * kTile);
          tma_load_2d(smem + kOffKb + ks * kTile, &map_k, &kv_full[ks], it.kvh * kBD, row_base + it.k0);
          tma_load_2d(smem + kOffVb + ks * kTile, &map_v, &kv_full[ks], it.kvh * kBD, row_base + it.k0);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int hh = 0; hh < it.gh && ok; ++hh) {
        const int h = it.kvh * group + it.h0 + hh;
        for (int j = 0; j < it.nq && ok; ++j, ++g) {
          const int st = g % kQdStages;
          const int q0 = (it.qt_lo + j) * kBT;
          if (lane == 0) ok = mbar_wait_sleep(&qd_empty[st], ((g / kQdStages) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            ++g;
            break;
          }
          if (lane == 0) {
            // Q, dO tiles and the step's 128 LSE*log2(e) and Delta values (one contiguous run each)
            float* lsl = ldbuf + st * 2 * kBT;
            const size_t run = (static_cast<size_t>(h) * p.batch + it.b) * p.tpad + q0;
            mbar_arrive_expect_tx(&qd_full[st], 2 * kTile + 2 * kBT * 4);
            tma_load_2d(smem + kOffQb + st * kTile, &map_q, &qd_full[st], h * kBD, row_base + q0);
            tma_load_2d(smem + kOffDOb + st * kTile, &map_do, &qd_full[st], h * kBD, row_base + q0);
            bulk_load(lsl, p.lse_t + run, kBT * 4, &qd_full[st]);
            bulk_load(lsl + kBT, p.delta_t + run, kBT * 4, &qd_full[st]);
          }
        }
      }
    }
    if (lane == 0) {
      for (int i = max(0, n - kKvStages); i < n; ++i)
        mbar_wait_sleep(&kv_full[i % kKvStages], (i / kKvStages) & 1, nullptr, SJ_DEV_ATTN_WAIT);
      for (int i = max(0, g - kQdStages); i < g; ++i)
        mbar_wait_sleep(&qd_full[i % kQdStages], (i / kQdStages) & 1, nullptr, SJ_DEV_ATTN_WAIT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t kIdS = umma_idesc_bf16(kBT, kBT, 0, 0);   // K-major A, K-major B
      constexpr uint32_t kIdAcc = umma_idesc_bf16(kBT, kBD, 0, 1);  // K-major A, MN-major B
      constexpr uint32_t kIdDq = umma_idesc_bf16(kBT, kBD, 1, 1);   // MN-major A, MN-major B
      // the second half of a step: dV, dK (accumulated) and dQ from P^T / dS^T of step i
      int pend_i = -1, pend_ks = 0, pend_first = 0, pend_last = 0, pend_n = 0;
      bool ok = true;
      auto issue_acc = [&]() -> bool {
        const int i = pend_i;
        const int st = i % kQdStages;
        if (!mbar_wait_sleep(ps_full, i & 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        const int qb = i & 1;  // dQ buffer
        if (!mbar_wait_sleep(&dq_empty[qb], ((i >> 1) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        if (pend_first && !mbar_wait_sleep(acc_empty, (pend_n & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        tc_fence_after();
        // descriptors of the k = 0 slices; a k step adds its byte offset / 16 to the start-address
        // field (all of shared memory is below 256 KB, so the 14-bit field does not carry)
        const uint64_t d_pt = umma_desc(smem_u32(smem + kOffPt), 16, 1024);
        const uint64_t d_dst = umma_desc(smem_u32(smem + kOffDSt), 16, 1024);
        const uint64_t d_dst_mn = umma_desc(smem_u32(smem + kOffDSt), kTile, 1024);
        const uint64_t d_q = umma_desc(smem_u32(smem + kOffQb + st * kTile), 8192, 1024);
        const uint64_t d_do = umma_desc(smem_u32(smem + kOffDOb + st * kTile), 8192, 1024);
        const uint64_t d_k = umma_desc(smem_u32(smem + kOffKb + pend_ks * kTile), 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < kBT / 16; ++kk) {
          const uint64_t kmaj = ((kk >> 2) * kTile + (kk & 3) * 32) >> 4;  // K-major step in a 128 x 128 tile
          const uint64_t mn = (kk * 2048) >> 4;                              // MN-major step
          const uint32_t acc = (pend_first && kk == 0) ? 0u : 1u;
          umma_f16(tmem + kColDV, d_pt + kmaj, d_do + mn, kIdAcc, acc);
          umma_f16(tmem + kColDK, d_dst + kmaj, d_q + mn, kIdAcc, acc);
          umma_f16(tmem + kColDQ + qb * kBD, d_dst_mn + mn, d_k + mn, kIdDq, kk > 0 ? 1u : 0u);
        }
        umma_commit(ps_empty);  // also: dQ_i, and at an item's last step dK / dV, complete in TMEM
        umma_commit(&qd_empty[st]);
        if (pend_last) umma_commit(&kv_empty[pend_ks]);
        pend_i = -1;
        return true;
      };
      int n = 0, g = 0;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++n) {
        const BItem it = decode_bitem(p, item);
        const int ks = n % kKvStages;
        if (!mbar_wait_sleep(&kv_full[ks], (n / kKvStages) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) break;
        const uint32_t ka = smem_u32(smem + kOffKb + ks * kTile), va = smem_u32(smem + kOffVb + ks * kTile);
        const int steps = it.gh * it.nq;
        for (int s = 0; s < steps && ok; ++s, ++g) {
          const int st = g % kQdStages;
          if (!mbar_wait_sleep(&qd_full[st], (g / kQdStages) & 1, abort_flag, SJ_DEV_ATTN_WAIT) ||
              !mbar_wait_sleep(sp_empty, (g & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t d_k = umma_desc(ka, 16, 1024), d_v = umma_desc(va, 16, 1024);
          const uint64_t d_q = umma_desc(smem_u32(smem + kOffQb + st * kTile), 16, 1024);
          const uint64_t d_do = umma_desc(smem_u32(smem + kOffDOb + st * kTile), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kBD / 16; ++kk) {
            const uint64_t step = (kk * 32) >> 4;
            umma_f16(tmem + kColSt, d_k + step, d_q + step, kIdS, kk > 0 ? 1u : 0u);
            umma_f16(tmem + kColDPt, d_v + step, d_do + step, kIdS, kk > 0 ? 1u : 0u);
          }
          umma_commit(sp_full);
          if (pend_i >= 0 && !issue_acc()) {
            ok = false;
            break;
          }
          pend_i = g;
          pend_ks = ks;
          pend_first = s == 0;
          pend_last = s == steps - 1;
          pend_n = n;
        }
      }
      if (ok && pend_i >= 0) issue_acc();
      umma_commit(drain);
      mbar_wait_sleep(drain, 0, nullptr, SJ_DEV_ATTN_WAIT);
    }
  } else {
    // ---------------------------------------------------------------- elementwise warps
    // thread <-> TMEM lane r: a key row for P^T / dS^T and dK / dV, a query row for dQ; part selects
    // 32 of the 128 query columns (P^T, dS^T) and 16 of the 64 head columns (dQ, dK, dV)
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    // step whose dQ (and, at an item's end, dK / dV) is still to be read out of TMEM
    int pend_g = -1, pend_h = 0, pend_last = 0;
    BItem pend_it{};
    uint8_t* slab = smem + kGOffStage + (warp - 2) * kGSlab;
    int pend_q0 = 0;
    // dQ_g: staged in the warp's slab and reduce-added into the f32 accumulator by TMA
    // (attn_dq_finish_kernel writes bf16); at the item's last step also its dK and dV: reduce-added
    // into the f32 partial sums when the items are split by head, else rotated back and written
    // in bf16; then the TMEM is released
    auto read_out = [&]() {
      const int qb = pend_g & 1;
      const int c0 = part * kEwHead;
      {
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem + lane_off + kColDQ + qb * kBD + c0, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&dq_empty[qb]);
          bulk_wait_read_all();  // the slab's previous reduce has read it
        }
        __syncwarp();
        stage_f32x16(slab, lane, v);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&map_dq, slab, pend_h * kBD + c0, pend_q0 + quarter * 32, pend_it.b);
          bulk_commit_group();
        }
      }
      if (!pend_last) return;
      const int kpos = pend_it.k0 + r;
      const size_t row = static_cast<size_t>(pend_it.b) * p.t + min(kpos, p.t - 1);
      uint32_t vk[16], vv[16];
      tmem_ld_32x32b_x16(tmem + lane_off + kColDK + c0, vk);
      tmem_ld_32x32b_x16(tmem + lane_off + kColDV + c0, vv);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (p.dkv_acc != nullptr) {
        // one slice of the group's heads: f32 partial sums (the finish kernel rotates dK and
        // writes bf16 once every slice has added its part); the 3-D map clips rows past the end
        const int y = pend_it.k0 + quarter * 32;
#pragma unroll
        for (int part_kv = 0; part_kv < 2; ++part_kv) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          stage_f32x16(slab, lane, part_kv == 0 ? vk : vv);
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_3d(&map_dkv, slab, pend_it.kvh * 2 * kBD + part_kv * kBD + c0, y, pend_it.b);
            bulk_commit_group();
          }
        }
      } else if (kpos < p.t) {
        const bool rope = p.rope_tab != nullptr || p.rope_log_theta > 0.f;
        uint32_t w[8];
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          float a = __uint_as_float(vk[c]), b = __uint_as_float(vk[c + 1]);
          if (rope) {
            const float2 cs = rope_cs(p.rope_tab, p.rope_log_theta, kpos, (c0 + c) >> 1);
            const float na = a * cs.x + b * cs.y, nb = -a * cs.y + b * cs.x;  // inverse rotation
            a = na;
            b = nb;
          }
          w[c >> 1] = pack_bf16x2(a, b);
        }
        uint4* out = reinterpret_cast<uint4*>(p.dk + row * p.lddk + pend_it.kvh * kBD + c0);
        out[0] = make_uint4(w[0], w[1], w[2], w[3]);
        out[1] = make_uint4(w[4], w[5], w[6], w[7]);
#pragma unroll
        for (int c = 0; c < 16; c += 2) w[c >> 1] = pack_bf16x2(__uint_as_float(vv[c]), __uint_as_float(vv[c + 1]));
        out = reinterpret_cast<uint4*>(p.dv + row * p.lddv + pend_it.kvh * kBD + c0);
        out[0] = make_uint4(w[0], w[1], w[2], w[3]);
        out[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    };
    int n = 0, g = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < p.items && alive; item += gridDim.x, ++n) {
      const BItem it = decode_bitem(p, item);
      const int kpos = it.k0 + r;
      const int steps = it.gh * it.nq;
      for (int s = 0; s < steps && alive; ++s, ++g) {
        const int st = g % kQdStages;
        const int q0 = (it.qt_lo + s % it.nq) * kBT;
        if (!mbar_wait_sleep(&qd_full[st], (g / kQdStages) & 1, abort_flag, SJ_DEV_ATTN_WAIT) ||
            !mbar_wait_sleep(sp_full, g & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const float* lsl = ldbuf + st * 2 * kBT + part * kEwCols;
        const float* dls = lsl + kBT;
        // visible queries of this key row in this part's columns: [lo, hi]
        const int cbase = q0 + part * kEwCols;
        const bool full_tile =
            q0 >= it.k0 + kBT - 1 && q0 + kBT <= p.t && it.k0 + kBT <= p.t &&
            (p.window <= 0 || q0 + kBT - 1 - it.k0 < p.window);
        int lo = 0, hi = kEwCols - 1;
        if (!full_tile) {
          lo = kpos - cbase;
          hi = min(p.window > 0 ? kpos + p.window - 1 : p.t - 1, p.t - 1) - cbase;
          if (kpos >= p.t) hi = -1;
        }
        // this thread's 32 query columns of S^T and dP^T, in two chunks of 16: P^T and dS^T are computed
        // and packed to bf16 (the first chunk while the previous step's MMAs may still read the
        // buffers) and stored as two 16-byte pieces each: 64-query half part / 2, chunks 4 (part & 1) ..
        uint8_t* pt = smem + kOffPt + (part >> 1) * kTile;
        uint8_t* dst = smem + kOffDSt + (part >> 1) * kTile;
#pragma unroll
        for (int chunk = 0; chunk < 2; ++chunk) {
          uint32_t sv[16], dv[16];
          tmem_ld_32x32b_x16(tmem + lane_off + kColSt + part * kEwCols + chunk * 16, sv);
          tmem_ld_32x32b_x16(tmem + lane_off + kColDPt + part * kEwCols + chunk * 16, dv);
          tmem_wait_ld();
          if (chunk == 1) {  // S^T / dP^T are in registers: the next step's products may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sp_empty);
          }
          uint32_t pw[8], dw[8];
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const int cc = chunk * 16 + c;
            const float4 l4 = *reinterpret_cast<const float4*>(lsl + cc);
            const float4 d4 = *reinterpret_cast<const float4*>(dls + cc);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dlv[4] = {d4.x, d4.y, d4.z, d4.w};
            float pr[4], ds[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const bool valid = cc + e >= lo && cc + e <= hi;  // (LSE / Delta past the sequence end are not data)
              pr[e] = valid ? ex2b(fmaf(__uint_as_float(sv[c + e]), p.scale_log2, -lv[e])) : 0.f;  // P^T
              ds[e] = valid ? pr[e] * (__uint_as_float(dv[c + e]) - dlv[e]) * p.scale : 0.f;       // dS^T
            }
            pw[c >> 1] = pack_bf16x2(pr[0], pr[1]);
            pw[(c >> 1) + 1] = pack_bf16x2(pr[2], pr[3]);
            dw[c >> 1] = pack_bf16x2(ds[0], ds[1]);
            dw[(c >> 1) + 1] = pack_bf16x2(ds[2], ds[3]);
          }
          if (chunk == 0) {
            // P^T and dS^T may overwrite the buffers once the previous step's MMAs have read them
            // (which also completes that step's dQ and, at an item's end, its dK / dV)
            if (!mbar_wait_sleep(ps_empty, (g & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
              alive = false;
              break;
            }
            tc_fence_after();
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int off = r * 128 + ((((part & 1) * 4 + chunk * 2 + j) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(pt + off) = make_uint4(pw[4 * j], pw[4 * j + 1], pw[4 * j + 2], pw[4 * j + 3]);
            *reinterpret_cast<uint4*>(dst + off) = make_uint4(dw[4 * j], dw[4 * j + 1], dw[4 * j + 2], dw[4 * j + 3]);
          }
        }
        if (!alive) break;
        fence_proxy_async_shared();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ps_full);
        if (pend_g >= 0) read_out();
        pend_g = g;
        pend_it = it;
        pend_h = it.kvh * group + it.h0 + s / it.nq;
        pend_q0 = q0;
        pend_last = s == steps - 1;
      }
    }
    // the last step's products
    if (alive && pend_g >= 0 && mbar_wait_sleep(ps_empty, pend_g & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
      tc_fence_after();
      read_out();
    }
    if (lane == 0) bulk_wait_all_groups();  // the reduces have read their slabs
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemColsB);
  }
}

// ---------------------------------------------------------------- banded backward
// A sliding window of at most 128 keys with one query head per kv head (the local stages of the
// hierarchical model): query tile q sees only key tiles q-1 and q, key tile k only query tiles k and
// k+1.  Each CTA takes a contiguous range of the key tiles of all (batch, head) pairs, flattened as
// u = (b * hk + h) * nkt + kt, and walks it with the steps
//   halo (kt-1, kt)  only at a range start inside a sequence: the part of dQ of query tile kt that
//                    the previous range's key tile contributes (recomputed here, nothing exchanged);
//   diag (kt, kt)    completes dQ of query tile kt;
//   off  (kt, kt+1)  completes dK / dV of key tile kt, and starts dQ of query tile kt+1 when that tile
//                    is in the range (else the next range's halo makes it).
// dQ accumulates in TMEM over two consecutive steps (two buffers by query-tile parity), dK / dV over
// two, and the CTA that completes a tile writes it once in bf16 (inverse RoPE on dQ and dK): no f32
// accumulator, no zero fill, no finish pass.  Each K / V and Q / dO tile is loaded once per range.
// Roles, shared-memory layout and TMEM columns are those of attn_bwd_tc_kernel.
enum : int {
  kStKv = 1, kStKvFirst = 2, kStKvLast = 4, kStDq = 8, kStDqFirst = 16, kStDqLast = 32,
  kStNewK = 64, kStLastK = 128, kStNewQ = 256, kStLastQ = 512
};
struct BandStep {
  int bh, kt, qt, flags;
};
struct BandCursor {
  int u, u0, u1, phase;  // phase 0: halo (when due), 1: diag, 2: off
};
// Advance to the next step of the range; false past its end.  Every role walks the same sequence.
SJ_DEVICE bool band_next(int nkt, BandCursor& c, BandStep& s) {
  while (c.u < c.u1) {
    const int kt = c.u % nkt, bh = c.u / nkt;
    if (c.phase == 0) {
      c.phase = 1;
      if (kt > 0 && c.u == c.u0) {
        s = {bh, kt - 1, kt, kStDq | kStDqFirst | kStNewK | kStLastK | kStNewQ};
        return true;
      }
    } else if (c.phase == 1) {
      const bool off = kt + 1 < nkt;
      c.phase = 2;
      s = {bh, kt, kt,
           kStKv | kStKvFirst | (off ? 0 : kStKvLast) | kStDq | (kt == 0 ? kStDqFirst : 0) | kStDqLast | kStNewK |
               (off ? 0 : kStLastK) | (kt == 0 ? kStNewQ : 0) | kStLastQ};
      return true;
    } else {
      c.phase = 0;
      ++c.u;
      if (kt + 1 < nkt) {
        const bool own = c.u < c.u1;  // the range goes on with key tile kt+1, so query tile kt+1 is its own
        s = {bh, kt, kt + 1, kStKv | kStKvLast | (own ? (kStDq | kStDqFirst) : kStLastQ) | kStLastK | kStNewQ};
        return true;
      }
    }
  }
  return false;
}

struct BandParams {
  int t, nkt, tiles, batch, hk, window;
  float scale, scale_log2;
  const float* lse_t;    // [hq][batch][tpad]: LSE * log2(e)
  const float* delta_t;  // [hq][batch][tpad]: Delta
  int tpad;
  int rope;              // dq, dk leave rotated back by the table (map_rope)
};

// Banded kernel layout.  Sixteen elementwise warps (four per TMEM lane quarter): a thread owns one key
// row of 32 query columns of S^T / dP^T, and 16 head columns of a dQ / dK / dV row.  Each of those
// warps has a 2 KB shared-memory slab that takes, in turn, the RoPE rows of a tile (32 positions x 16
// floats, by TMA) and the warp's bf16 output slabs (32 rows x 32 B each) that a TMA store writes out:
// a thread's row-wise loads and stores, 32 distinct lines per instruction, were most of the kernel's
// time.
constexpr int kBandEw = 16;
constexpr int kBandCols = kBT / (kBandEw / 4);   // query columns of S^T / dP^T per thread
constexpr int kBandHc = kBD / (kBandEw / 4);     // head columns of dQ / dK / dV per thread
constexpr int kBandThreads = 32 * (2 + kBandEw);
constexpr int kBandSlab = 32 * kBandHc * 4;      // the RoPE rows; also two output slabs of 32 x kBandHc bf16
constexpr int kBandOut = 32 * kBandHc * 2;
static_assert(kBandCols == 32 && kBandHc == 16, "banded elementwise mapping");
constexpr int kBOffStage = kOffLd + kQdStages * 2 * kBT * 4;  // 1024-aligned (194 KB)
constexpr int kBOffBar = kBOffStage + kBandEw * kBandSlab;
constexpr int kBandLayout = kBOffBar + 512;
constexpr int kSmemBand = 232448;  // the per-block maximum; what the layout leaves is alignment slack
static_assert(kBOffStage % 1024 == 0, "slabs hold 128-byte-swizzled TMA boxes");
static_assert(kBandLayout <= kSmemBand, "banded attention backward shared memory");


// 16 f32 values of a row -> 8 bf16 pairs, inverse-rotated by the row's (cos, sin) pairs when `rope`.
SJ_DEVICE void rotate_pack16(uint32_t (&w)[8], const uint32_t (&v)[16], bool rope, const float (&cs)[16]) {
#pragma unroll
  for (int c = 0; c < 16; c += 2) {
    float a = __uint_as_float(v[c]), b = __uint_as_float(v[c + 1]);
    if (rope) {
      const float co = cs[c], si = cs[c + 1];
      const float na = a * co + b * si, nb = -a * si + b * co;  // inverse rotation
      a = na;
      b = nb;
    }
    w[c >> 1] = pack_bf16x2(a, b);
  }
}
// Row `lane` (32 bytes) of a 32 x 32-byte SWIZZLE_32B slab: chunk j at lane*32 + ((j ^ ((lane >> 2) & 1)) * 16).
SJ_DEVICE void stage_row32b(uint8_t* slab, int lane, const uint32_t (&w)[8]) {
#pragma unroll
  for (int j = 0; j < 2; ++j)
    *reinterpret_cast<uint4*>(slab + lane * 32 + ((j ^ ((lane >> 2) & 1)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

__global__ void __launch_bounds__(kBandThreads, 1)
    attn_bwd_band_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_do,
                         const __grid_constant__ CUtensorMap map_dq, const __grid_constant__ CUtensorMap map_dk,
                         const __grid_constant__ CUtensorMap map_dv, const __grid_constant__ CUtensorMap map_rope,
                         const BandParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad + kBandLayout > kSmemBand) {  // uniform over the CTA, before any barrier or TMEM use
    if (threadIdx.x == 0) record_error(SJ_DEV_SMEM_ALIGN);
    pdl_wait();
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBOffBar);
  uint64_t* kv_full = bars;         // 2: K / V slots
  uint64_t* kv_empty = bars + 2;    // 2
  uint64_t* qd_full = bars + 4;     // 2: Q / dO (+ LSE, Delta) slots
  uint64_t* qd_empty = bars + 6;    // 2
  uint64_t* sp_full = bars + 8;     // S^T, dP^T in TMEM
  uint64_t* sp_empty = bars + 9;    // the elementwise warps have them in registers
  uint64_t* ps_full = bars + 10;    // P^T, dS^T in shared memory
  uint64_t* ps_empty = bars + 11;   // their MMAs are done
  uint64_t* dq_empty = bars + 12;   // 2: dQ buffer (query-tile parity) read out
  uint64_t* acc_empty = bars + 14;  // dK / dV read out
  uint64_t* drain = bars + 15;
  uint64_t* rope_full = bars + 16;  // kBandEw: a warp's RoPE rows in its slab
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16 + kBandEw);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* ldbuf = reinterpret_cast<float*>(smem + kOffLd);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = static_cast<int>(static_cast<long long>(blockIdx.x) * p.tiles / gridDim.x);
  const int u1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.tiles / gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&dq_empty[i], kBandEw);
    }
    mbar_init(sp_full, 1);
    mbar_init(sp_empty, kBandEw);
    mbar_init(ps_full, kBandEw);
    mbar_init(ps_empty, 1);
    mbar_init(acc_empty, kBandEw);
    mbar_init(drain, 1);
    for (int i = 0; i < kBandEw; ++i) mbar_init(&rope_full[i], 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_q);
    tma_prefetch_map(&map_k);
    tma_prefetch_map(&map_v);
    tma_prefetch_map(&map_do);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemColsB);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // operands may come from the previous kernel
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (one thread)
    if (lane == 0) {
      BandCursor c{u0, u0, u1, 0};
      BandStep s;
      int nk = 0, nq = 0;
      bool ok = true;
      while (ok && band_next(p.nkt, c, s)) {
        const int b = s.bh / p.hk, h = s.bh % p.hk;
        const int row_base = b * p.t;
        if (s.flags & kStNewK) {
          const int slot = nk & 1;
          ok = mbar_wait_sleep(&kv_empty[slot], ((nk >> 1) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT);
          if (!ok) break;
          mbar_arrive_expect_tx(&kv_full[slot], 2 * kTile);
          tma_load_2d(smem + kOffKb + slot * kTile, &map_k, &kv_full[slot], h * kBD, row_base + s.kt * kBT);
          tma_load_2d(smem + kOffVb + slot * kTile, &map_v, &kv_full[slot], h * kBD, row_base + s.kt * kBT);
          ++nk;
        }
        if (s.flags & kStNewQ) {
          const int slot = nq & 1;
          ok = mbar_wait_sleep(&qd_empty[slot], ((nq >> 1) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT);
          if (!ok) break;
          const int q0 = s.qt * kBT;
          float* lsl = ldbuf + slot * 2 * kBT;
          const size_t run = (static_cast<size_t>(h) * p.batch + b) * p.tpad + q0;
          mbar_arrive_expect_tx(&qd_full[slot], 2 * kTile + 2 * kBT * 4);
          tma_load_2d(smem + kOffQb + slot * kTile, &map_q, &qd_full[slot], h * kBD, row_base + q0);
          tma_load_2d(smem + kOffDOb + slot * kTile, &map_do, &qd_full[slot], h * kBD, row_base + q0);
          bulk_load(lsl, p.lse_t + run, kBT * 4, &qd_full[slot]);
          bulk_load(lsl + kBT, p.delta_t + run, kBT * 4, &qd_full[slot]);
          ++nq;
        }
      }
      // copies still in flight must land before the CTA exits
      for (int i = max(0, nk - 2); i < nk; ++i) mbar_wait_sleep(&kv_full[i & 1], (i >> 1) & 1, nullptr, SJ_DEV_ATTN_WAIT);
      for (int i = max(0, nq - 2); i < nq; ++i) mbar_wait_sleep(&qd_full[i & 1], (i >> 1) & 1, nullptr, SJ_DEV_ATTN_WAIT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t kIdS = umma_idesc_bf16(kBT, kBT, 0, 0);   // K-major A, K-major B
      constexpr uint32_t kIdAcc = umma_idesc_bf16(kBT, kBD, 0, 1);  // K-major A, MN-major B
      constexpr uint32_t kIdDq = umma_idesc_bf16(kBT, kBD, 1, 1);   // MN-major A, MN-major B
      BandStep pend{};
      int pend_g = -1, pend_ks = 0, pend_qs = 0;
      int nkv = 0, dq_uses[2] = {0, 0};
      bool ok = true;
      // the second half of a step: dV, dK (accumulated over the key tile's steps) and dQ (over the
      // query tile's) from its P^T / dS^T
      auto issue_acc = [&]() -> bool {
        const int f = pend.flags;
        if (!mbar_wait(ps_full, pend_g & 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        if ((f & kStKvFirst) && !mbar_wait(acc_empty, (nkv & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        if (f & kStKvFirst) ++nkv;
        const int qb = pend.qt & 1;
        if ((f & kStDqFirst) && !mbar_wait(&dq_empty[qb], (dq_uses[qb] & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT))
          return false;
        if (f & kStDqFirst) ++dq_uses[qb];
        tc_fence_after();
        const uint64_t d_pt = umma_desc(smem_u32(smem + kOffPt), 16, 1024);
        const uint64_t d_dst = umma_desc(smem_u32(smem + kOffDSt), 16, 1024);
        const uint64_t d_dst_mn = umma_desc(smem_u32(smem + kOffDSt), kTile, 1024);
        const uint64_t d_q = umma_desc(smem_u32(smem + kOffQb + pend_qs * kTile), 8192, 1024);
        const uint64_t d_do = umma_desc(smem_u32(smem + kOffDOb + pend_qs * kTile), 8192, 1024);
        const uint64_t d_k = umma_desc(smem_u32(smem + kOffKb + pend_ks * kTile), 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < kBT / 16; ++kk) {
          const uint64_t kmaj = ((kk >> 2) * kTile + (kk & 3) * 32) >> 4;  // K-major step in a 128 x 128 tile
          const uint64_t mn = (kk * 2048) >> 4;                              // MN-major step
          if (f & kStKv) {
            const uint32_t acc = ((f & kStKvFirst) && kk == 0) ? 0u : 1u;
            umma_f16(tmem + kColDV, d_pt + kmaj, d_do + mn, kIdAcc, acc);
            umma_f16(tmem + kColDK, d_dst + kmaj, d_q + mn, kIdAcc, acc);
          }
          if (f & kStDq)
            umma_f16(tmem + kColDQ + qb * kBD, d_dst_mn + mn, d_k + mn, kIdDq, ((f & kStDqFirst) && kk == 0) ? 0u : 1u);
        }
        umma_commit(ps_empty);  // also: the step's dQ / dK / dV contributions are in TMEM
        if (f & kStLastQ) umma_commit(&qd_empty[pend_qs]);
        if (f & kStLastK) umma_commit(&kv_empty[pend_ks]);
        pend_g = -1;
        return true;
      };
      BandCursor c{u0, u0, u1, 0};
      BandStep s;
      int g = 0, nk = 0, nq = 0, ks = 0, qs = 0;
      while (ok && band_next(p.nkt, c, s)) {
        if (s.flags & kStNewK) {
          ks = nk & 1;
          if (!mbar_wait(&kv_full[ks], (nk >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) break;
          ++nk;
        }
        if (s.flags & kStNewQ) {
          qs = nq & 1;
          if (!mbar_wait(&qd_full[qs], (nq >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) break;
          ++nq;
        }
        if (!mbar_wait(sp_empty, (g & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) break;
        tc_fence_after();
        const uint64_t d_k = umma_desc(smem_u32(smem + kOffKb + ks * kTile), 16, 1024);
        const uint64_t d_v = umma_desc(smem_u32(smem + kOffVb + ks * kTile), 16, 1024);
        const uint64_t d_q = umma_desc(smem_u32(smem + kOffQb + qs * kTile), 16, 1024);
        const uint64_t d_do = umma_desc(smem_u32(smem + kOffDOb + qs * kTile), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kBD / 16; ++kk) {
          const uint64_t step = (kk * 32) >> 4;
          umma_f16(tmem + kColSt, d_k + step, d_q + step, kIdS, kk > 0 ? 1u : 0u);
          umma_f16(tmem + kColDPt, d_v + step, d_do + step, kIdS, kk > 0 ? 1u : 0u);
        }
        umma_commit(sp_full);
        if (pend_g >= 0 && !issue_acc()) {
          ok = false;
          break;
        }
        pend = s;
        pend_g = g;
        pend_ks = ks;
        pend_qs = qs;
        ++g;
      }
      if (ok && pend_g >= 0) issue_acc();
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, SJ_DEV_ATTN_WAIT);
    }
  } else {
    // ---------------------------------------------------------------- elementwise warps
    // thread <-> TMEM lane r: a key row for P^T / dS^T (query columns [32 part, 32 part + 32)) and for
    // dK / dV, a query row for dQ (head columns [16 part, 16 part + 16) of those three)
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int part = ew >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int hc = part * kBandHc;  // head columns of dQ / dK / dV
    uint8_t* slab = smem + kBOffStage + ew * kBandSlab;
    BandStep pend{};
    int pend_g = -1;
    int rope_loads = 0;          // loads issued into the slab (their barrier's phase count)
    bool rope_pending = false;   // a load issued and not yet read
    // the rows a read-out of step `st` rotates with: its query tile (dQ) or key tile (dK)
    auto rope_tile_of = [&](const BandStep& st) { return (st.flags & kStDqLast) ? st.qt : st.kt; };
    // request the RoPE rows of the pending step's read-out (this warp's 32 positions, its 8 (cos, sin)
    // pairs), once the slab's previous stores have read it; they land while the step computes
    auto request_rope = [&]() {
      if (!p.rope || pend_g < 0 || !(pend.flags & (kStDqLast | kStKvLast))) return;
      if (lane == 0) {
        bulk_wait_read_all();
        mbar_arrive_expect_tx(&rope_full[ew], kBandSlab);
        tma_load_2d(slab, &map_rope, &rope_full[ew], hc, rope_tile_of(pend) * kBT + quarter * 32);
      }
      __syncwarp();
      ++rope_loads;
      rope_pending = true;
    };
    // a completed step's finished tiles: dQ of its query tile and / or dK, dV of its key tile, staged
    // in the slab and written by TMA (the 3-D maps clip rows past the sequence end)
    auto read_out = [&]() -> bool {
      const int b = pend.bh / p.hk, h = pend.bh % p.hk;
      const bool dq_last = pend.flags & kStDqLast, kv_last = pend.flags & kStKvLast;
      if (!dq_last && !kv_last) return true;
      float cs[16];
      if (rope_pending) {
        if (!mbar_wait(&rope_full[ew], (rope_loads - 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // 64-byte swizzled row `lane`
          const float4 v = *reinterpret_cast<const float4*>(slab + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4));
          cs[4 * j] = v.x;
          cs[4 * j + 1] = v.y;
          cs[4 * j + 2] = v.z;
          cs[4 * j + 3] = v.w;
        }
        rope_pending = false;
      } else if (lane == 0) {
        bulk_wait_read_all();  // the slab's previous stores have read it
      }
      __syncwarp();
      const int y = rope_tile_of(pend) * kBT + quarter * 32;
      uint32_t w[8];
      int used = 0;  // output slabs holding staged rows
      if (dq_last) {
        const int qb = pend.qt & 1;
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem + lane_off + kColDQ + qb * kBD + hc, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_empty[qb]);
        rotate_pack16(w, v, p.rope != 0, cs);
        stage_row32b(slab, lane, w);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) tma_store_3d(&map_dq, slab, h * kBD + hc, y, b);
        used = 1;
      }
      if (kv_last) {
        uint32_t vk[16], vv[16];
        tmem_ld_32x32b_x16(tmem + lane_off + kColDK + hc, vk);
        tmem_ld_32x32b_x16(tmem + lane_off + kColDV + hc, vv);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
        rotate_pack16(w, vk, p.rope != 0, cs);
        stage_row32b(slab + used * kBandOut, lane, w);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) tma_store_3d(&map_dk, slab + used * kBandOut, h * kBD + hc, y, b);
        if (used) {  // dQ and dK fill the slab: dV follows once both have been read
          if (lane == 0) {
            bulk_commit_group();
            bulk_wait_read_all();
          }
          __syncwarp();
          used = 0;
        } else {
          used = 1;
        }
        rotate_pack16(w, vv, false, cs);
        stage_row32b(slab + used * kBandOut, lane, w);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) tma_store_3d(&map_dv, slab + used * kBandOut, h * kBD + hc, y, b);
      }
      if (lane == 0) bulk_commit_group();
      __syncwarp();
      return true;
    };
    BandCursor c{u0, u0, u1, 0};
    BandStep s;
    int g = 0, nq = 0, qs = 0;
    uint32_t qpar = 0;
    bool alive = true;
    while (alive && band_next(p.nkt, c, s)) {
      if (s.flags & kStNewQ) {
        qs = nq & 1;
        qpar = (nq >> 1) & 1;
        ++nq;
      }
      request_rope();  // lands while this step computes; read out at its end
      // LSE / Delta of the step's query tile (their bulk copies complete on qd_full), then S^T, dP^T
      if (!mbar_wait(&qd_full[qs], qpar, abort_flag, SJ_DEV_ATTN_WAIT) ||
          !mbar_wait(sp_full, g & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const float* lsl = ldbuf + qs * 2 * kBT + part * kBandCols;
      const float* dls = lsl + kBT;
      // visible queries of this key row among this thread's 32 columns: [lo, hi]
      const int kpos = s.kt * kBT + r;
      const int cbase = s.qt * kBT + part * kBandCols;
      const int lo = kpos - cbase;
      const int hi = kpos < p.t ? min(kpos + p.window - 1, p.t - 1) - cbase : -1;
      // columns [32 part, 32 part + 32): 64-query half part / 2 of P^T / dS^T, 16-byte chunks 4 (part & 1) ..
      uint8_t* pt = smem + kOffPt + (part >> 1) * kTile;
      uint8_t* dst = smem + kOffDSt + (part >> 1) * kTile;
      // two chunks of 16 columns, each read from TMEM, turned into P^T / dS^T and stored (the first once
      // the previous step's MMAs are done with the buffers)
#pragma unroll
      for (int chunk = 0; chunk < 2; ++chunk) {
        uint32_t sv[16], dv[16];
        tmem_ld_32x32b_x16(tmem + lane_off + kColSt + part * kBandCols + chunk * 16, sv);
        tmem_ld_32x32b_x16(tmem + lane_off + kColDPt + part * kBandCols + chunk * 16, dv);
        tmem_wait_ld();
        if (chunk == 1) {  // S^T / dP^T are in registers: the next step's products may start
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(sp_empty);
        }
        uint32_t pw[8], dw[8];
#pragma unroll
        for (int c4 = 0; c4 < 16; c4 += 4) {
          const int cc = chunk * 16 + c4;
          const float4 l4 = *reinterpret_cast<const float4*>(lsl + cc);
          const float4 d4 = *reinterpret_cast<const float4*>(dls + cc);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dlv[4] = {d4.x, d4.y, d4.z, d4.w};
          float pr[4], ds[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const bool valid = cc + e >= lo && cc + e <= hi;
            pr[e] = ex2b(valid ? fmaf(__uint_as_float(sv[c4 + e]), p.scale_log2, -lv[e]) : -INFINITY);  // P^T
            ds[e] = pr[e] * fmaf(__uint_as_float(dv[c4 + e]), p.scale, -dlv[e]);  // dS^T (Delta pre-scaled)
          }
          pw[c4 >> 1] = pack_bf16x2(pr[0], pr[1]);
          pw[(c4 >> 1) + 1] = pack_bf16x2(pr[2], pr[3]);
          dw[c4 >> 1] = pack_bf16x2(ds[0], ds[1]);
          dw[(c4 >> 1) + 1] = pack_bf16x2(ds[2], ds[3]);
        }
        if (chunk == 0) {  // P^T and dS^T overwrite the buffers once the previous step's MMAs have read them
          if (!mbar_wait(ps_empty, (g & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
            alive = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int off = r * 128 + ((((part & 1) * 4 + chunk * 2 + j) ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(pt + off) = make_uint4(pw[4 * j], pw[4 * j + 1], pw[4 * j + 2], pw[4 * j + 3]);
          *reinterpret_cast<uint4*>(dst + off) = make_uint4(dw[4 * j], dw[4 * j + 1], dw[4 * j + 2], dw[4 * j + 3]);
        }
      }
      if (!alive) break;
      fence_proxy_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ps_full);
      if (pend_g >= 0 && !read_out()) {
        alive = false;
        break;
      }
      pend = s;
      pend_g = g;
      ++g;
    }
    if (alive && pend_g >= 0 && mbar_wait(ps_empty, pend_g & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
      tc_fence_after();
      request_rope();
      read_out();
    }
    // a RoPE load still in flight (an abandoned read-out) lands before the slab goes away; the
    // stores finish reading their slabs
    if (rope_pending) mbar_wait(&rope_full[ew], (rope_loads - 1) & 1, nullptr, SJ_DEV_ATTN_WAIT);
    if (lane == 0) bulk_wait_all_groups();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemColsB);
  }
}

// Delta = sum_d dO * O per (row, head) (hierarchy.py:53-57), times `delta_scale` (the banded kernel
// takes Delta pre-multiplied by the softmax scale), and the LSE times log2(e), both written transposed
// to [head][batch][tpad] so that a step's 128 values are one contiguous run; the same threads zero the
// (row, head) slice of the f32 dQ accumulator (when there is one: the banded kernel has none) and, for
// head < hk when the items are split by head, the (row, kv head) slice of the f32 dK / dV accumulator.
// Eight lanes per (row, head), each with 8 of its 64 columns: a warp reads four rows' 128-byte head
// slices of O and dO and writes their accumulator slices as whole lines; heads outermost, rows next
// (measured faster than rows outermost, and than four slices per thread).
__global__ void attn_delta_kernel(const __nv_bfloat16* o, int ldo, const __nv_bfloat16* dout, int lddo,
                                  const float* lse, float* delta_t, float* lse_t, float* dq_acc, float* dkv_acc,
                                  int rows, int t, int tpad, int hq, int hk, float delta_scale) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t slices = static_cast<size_t>(rows) * hq;
  const bool live = i < slices * 8;
  const size_t rh = live ? i >> 3 : 0;
  const int j = static_cast<int>(i & 7);
  const int h = static_cast<int>(rh / rows), row = static_cast<int>(rh % rows);
  float acc = 0.f;
  if (live) {
    const uint4 x = *reinterpret_cast<const uint4*>(dout + static_cast<size_t>(row) * lddo + h * kBD + 8 * j);
    const uint4 y = *reinterpret_cast<const uint4*>(o + static_cast<size_t>(row) * ldo + h * kBD + 8 * j);
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 u = unpack_bf16x2(xs[e]), v = unpack_bf16x2(ys[e]);
      acc = fmaf(u.x, v.x, fmaf(u.y, v.y, acc));
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (!live) return;
  if (j == 0) {
    const int b = row / t, pos = row % t;
    const size_t dst = (static_cast<size_t>(h) * (rows / t) + b) * tpad + pos;
    delta_t[dst] = acc * delta_scale;
    lse_t[dst] = lse[static_cast<size_t>(row) * hq + h] * kLog2eB;
  }
  if (dq_acc == nullptr) return;
  float4* z = reinterpret_cast<float4*>(dq_acc + (static_cast<size_t>(row) * hq + h) * kBD + 8 * j);
  z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (dkv_acc != nullptr && h < hk) {
    z = reinterpret_cast<float4*>(dkv_acc + (static_cast<size_t>(row) * hk + h) * (2 * kBD) + 16 * j);
#pragma unroll
    for (int e = 0; e < 4; ++e) z[e] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// 8 f32 values (4 column pairs from pair q4 on) -> bf16 at dst, inverse-rotated when `rotate`.
SJ_DEVICE void finish_quad(const float* src, __nv_bfloat16* dst, bool rotate, const float2* tab, float log_theta,
                           int pos, int q4) {
  const float4 v0 = reinterpret_cast<const float4*>(src)[0], v1 = reinterpret_cast<const float4*>(src)[1];
  float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  if (rotate) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 cs = rope_cs(tab, log_theta, pos, 4 * q4 + e);
      const float a = x[2 * e], b = x[2 * e + 1];
      x[2 * e] = a * cs.x + b * cs.y;
      x[2 * e + 1] = -a * cs.y + b * cs.x;
    }
  }
  *reinterpret_cast<uint4*>(dst) =
      make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
}

// dq = bf16(inverse RoPE(dq_acc)), one thread per (row, head, 4 column pairs); when the items were
// split by head, further threads per (row, kv head, 4 column pairs) write dk = bf16(inverse
// RoPE(dK partial sum)) and dv = bf16(dV partial sum).
__global__ void attn_dq_finish_kernel(const float* acc, __nv_bfloat16* dq, int lddq, const float* dkv_acc,
                                      __nv_bfloat16* dk, int lddk, __nv_bfloat16* dv, int lddv, int rows, int t,
                                      int hq, int hk, const float2* tab, float log_theta) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  constexpr int kQuads = kBD / 8;
  const bool rotate = tab != nullptr || log_theta > 0.f;
  const size_t nq = static_cast<size_t>(rows) * hq * kQuads;
  if (i < nq) {
    const int row = static_cast<int>(i / (hq * kQuads));
    const int rem = static_cast<int>(i % (hq * kQuads));
    const int h = rem / kQuads, q4 = rem % kQuads;
    finish_quad(acc + i * 8, dq + static_cast<size_t>(row) * lddq + h * kBD + 8 * q4, rotate, tab, log_theta,
                row % t, q4);
    return;
  }
  if (dkv_acc == nullptr) return;
  const size_t j = i - nq;
  if (j >= static_cast<size_t>(rows) * hk * kQuads) return;
  const int row = static_cast<int>(j / (hk * kQuads));
  const int rem = static_cast<int>(j % (hk * kQuads));
  const int h = rem / kQuads, q4 = rem % kQuads;
  const float* src = dkv_acc + (static_cast<size_t>(row) * hk + h) * (2 * kBD) + 8 * q4;
  finish_quad(src, dk + static_cast<size_t>(row) * lddk + h * kBD + 8 * q4, rotate, tab, log_theta, row % t, q4);
  finish_quad(src + kBD, dv + static_cast<size_t>(row) * lddv + h * kBD + 8 * q4, false, tab, log_theta, row % t,
              q4);
}

}  // namespace sj

using namespace sj;

// Head slices per (batch, kv head, key tile) item: when those items are fewer than B200's 148 SMs,
// each item takes one query head of its GQA group (the heaviest items, the first key tiles of a
// causal sequence, would otherwise set the launch's length with SMs idle); a function of the
// shape alone, so that the workspace size is too.
static int bwd_head_slices(int batch, int t, int hq, int hk) {
  constexpr int kB200Sms = 148;
  const long items = static_cast<long>(batch) * hk * ((t + kBT - 1) / kBT);
  return (hq > hk && items < kB200Sms) ? hq / hk : 1;
}

// The banded kernel (attn_bwd_band_kernel) serves a window of at most one key tile with one query
// head per kv head; everything else takes the general kernel.
// (with a RoPE table, or no rotation: the banded kernel reads the table's rows by TMA).
static bool bwd_banded(int window, int hq, int hk, float rope_theta, const float* rope_table) {
  return window > 0 && window <= kBT && hq == hk && (rope_table != nullptr || rope_theta <= 0.f);
}

// 3-D bf16 map [batch][t][cols] (row stride ld elements) with boxes of 32 rows x the banded kernel's
// head columns per thread and the 32-byte swizzle: a store of a box never crosses into the next
// sequence's rows.
static int bf16_map_bt(CUtensorMap* map, const void* ptr, int cols, int t, int batch, int ld) {
  const uint64_t dims[3] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(t), static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(ld) * 2 * t};
  const uint32_t box[3] = {kBandHc, 32, 1};
  static_assert(kBandHc * 2 == 32, "32-byte rows: the 32-byte swizzle");
  return tensor_map(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_32B);
}

extern "C" size_t sj_attn_workspace(int batch, int t, int hq, int hk) {
  if (batch <= 0 || t <= 0 || hq <= 0 || hk <= 0 || hq % hk) return 0;
  const size_t rows = static_cast<size_t>(batch) * t;
  const size_t tpad = static_cast<size_t>((t + kBT - 1) / kBT) * kBT;
  // the f32 dQ accumulator [rows, hq*64], then Delta and LSE*log2(e) transposed, [hq][batch][tpad]
  // each, then (items split by head) the f32 dK / dV accumulator [rows, hk, 128]
  const size_t dkv = bwd_head_slices(batch, t, hq, hk) > 1 ? rows * hk * 2 * kBD : 0;
  return rows * hq * kBD + 2 * static_cast<size_t>(hq) * batch * tpad + dkv;
}

extern "C" int sj_attn_gqa_bwd(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv, const void* o,
                               int ldo, const float* lse, const void* dout, int lddo, void* dq, int lddq, void* dk,
                               int lddk, void* dv, int lddv, float* workspace, int batch, int t, int hq, int hk,
                               int head_dim, int window, float rope_theta, const float* rope_table, void* stream) {
  if (head_dim != kBD) return fail(SJ_ERR_UNSUPPORTED, "attention: head_dim %d (this build: 64)", head_dim);
  if (batch <= 0 || t <= 0 || hq <= 0 || hk <= 0 || hq % hk || window < 0)
    return fail(SJ_ERR_SHAPE, "attention: bad shape batch=%d t=%d hq=%d hk=%d window=%d", batch, t, hq, hk, window);
  if ((ldq | ldk | ldv | ldo | lddo | lddq | lddk | lddv) % 8)
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: strides must be multiples of 8");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dout) || !aligned16(dq) ||
      !aligned16(dk) || !aligned16(dv))
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: 16-byte aligned operands required");
  if (!workspace || !aligned16(workspace)) return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: workspace must be aligned");
  if (rope_table && (reinterpret_cast<uintptr_t>(rope_table) & 7))
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: rope table must be 8-byte aligned");
  const bool band = bwd_banded(window, hq, hk, rope_theta, rope_table);
  if (band && rope_table && (reinterpret_cast<uintptr_t>(rope_table) & 15))
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_bwd: rope table must be 16-byte aligned for a window <= 128");
  static KernelAttrOnce attr_once, band_attr_once;
  const int attr_rc =
      band ? ensure_max_smem(band_attr_once, reinterpret_cast<const void*>(attn_bwd_band_kernel), kSmemBand,
                             "banded attention backward shared-memory attribute")
           : ensure_max_smem(attr_once, reinterpret_cast<const void*>(attn_bwd_tc_kernel), kSmemGen,
                             "attention backward shared-memory attribute");
  if (attr_rc != SJ_OK) return attr_rc;
  cudaStream_t s = as_stream(stream);
  const size_t rows = static_cast<size_t>(batch) * t;
  const int tpad = ((t + kBT - 1) / kBT) * kBT;
  float* dq_acc = workspace;
  float* delta_t = dq_acc + rows * hq * kBD;
  float* lse_t = delta_t + static_cast<size_t>(hq) * batch * tpad;
  const int hsplit = bwd_head_slices(batch, t, hq, hk);
  float* dkv_acc = !band && hsplit > 1 ? lse_t + static_cast<size_t>(hq) * batch * tpad : nullptr;
  const size_t row_heads = rows * hq;
  const size_t delta_threads = row_heads * 8;
  launch(attn_delta_kernel, static_cast<unsigned>((delta_threads + 255) / 256), 256, 0, s,
         static_cast<const __nv_bfloat16*>(o), ldo, static_cast<const __nv_bfloat16*>(dout), lddo, lse, delta_t, lse_t,
         band ? nullptr : dq_acc, dkv_acc, static_cast<int>(rows), t, tpad, hq, hk, band ? 0.125f : 1.0f);
  SJ_LAUNCH_CHECK("attn_delta");
  CUtensorMap maps[4];
  int rc = bf16_map(&maps[0], q, static_cast<uint64_t>(hq) * kBD, rows, ldq, kBD, kBT);
  if (!rc) rc = bf16_map(&maps[1], k, static_cast<uint64_t>(hk) * kBD, rows, ldk, kBD, kBT);
  if (!rc) rc = bf16_map(&maps[2], v, static_cast<uint64_t>(hk) * kBD, rows, ldv, kBD, kBT);
  if (!rc) rc = bf16_map(&maps[3], dout, static_cast<uint64_t>(hq) * kBD, rows, lddo, kBD, kBT);
  if (rc) return rc;
  const float2* rope_tab = reinterpret_cast<const float2*>(rope_table);
  const float rope_log_theta = rope_table ? 0.f : (rope_theta > 0.f ? logf(rope_theta) : 0.f);
  if (band) {
    CUtensorMap out[4];
    rc = bf16_map_bt(&out[0], dq, hq * kBD, t, batch, lddq);
    if (!rc) rc = bf16_map_bt(&out[1], dk, hk * kBD, t, batch, lddk);
    if (!rc) rc = bf16_map_bt(&out[2], dv, hk * kBD, t, batch, lddv);
    if (!rc) {  // [t][64] f32 (cos, sin) pairs, boxes of 32 positions x 16 floats (64-byte rows)
                // (with no table, an unused map of the workspace)
      const uint64_t dims[2] = {64, static_cast<uint64_t>(t)}, strides[1] = {256};
      const uint32_t box[2] = {kBandHc, 32};
      rc = tensor_map(&out[3], rope_table ? static_cast<const void*>(rope_table) : static_cast<const void*>(lse_t),
                      CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
    }
    if (rc) return rc;
    BandParams bp;
    bp.t = t;
    bp.nkt = (t + kBT - 1) / kBT;
    bp.tiles = batch * hk * bp.nkt;
    bp.batch = batch;
    bp.hk = hk;
    bp.window = window;
    bp.scale = 0.125f;
    bp.scale_log2 = 0.125f * kLog2eB;
    bp.lse_t = lse_t;
    bp.delta_t = delta_t;
    bp.tpad = tpad;
    bp.rope = rope_table != nullptr;
    launch(attn_bwd_band_kernel, std::min(bp.tiles, sm_count()), kBandThreads, kSmemBand, s, maps[0], maps[1],
           maps[2], maps[3], out[0], out[1], out[2], out[3], bp);
    SJ_LAUNCH_CHECK("attn_bwd_band");
    return SJ_OK;
  }
  BwdParams p;
  p.t = t;
  p.hq = hq;
  p.hk = hk;
  p.window = window;
  p.batch = batch;
  p.nkt = (t + kBT - 1) / kBT;
  p.hsplit = hsplit;
  p.dkv_acc = dkv_acc;
  p.items = batch * hk * hsplit * p.nkt;
  p.scale = 0.125f;
  p.scale_log2 = 0.125f * kLog2eB;
  p.lse_t = lse_t;
  p.delta_t = delta_t;
  p.tpad = tpad;
  p.dq_acc = dq_acc;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.lddk = lddk;
  p.lddv = lddv;
  p.rope_tab = rope_tab;
  p.rope_log_theta = rope_log_theta;
  const int grid = std::min(p.items, sm_count());
  // f32 accumulators as [batch][t][cols] with 32-row x 16-column boxes (64-byte rows, 64-byte swizzle)
  CUtensorMap acc_maps[2];
  {
    const uint64_t dq_dims[3] = {static_cast<uint64_t>(hq) * kBD, static_cast<uint64_t>(t), static_cast<uint64_t>(batch)};
    const uint64_t dq_str[2] = {static_cast<uint64_t>(hq) * kBD * 4, static_cast<uint64_t>(hq) * kBD * 4 * t};
    const uint32_t box[3] = {16, 32, 1};
    rc = tensor_map(&acc_maps[0], dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq_dims, dq_str, box,
                    CU_TENSOR_MAP_SWIZZLE_64B);
    if (!rc && dkv_acc != nullptr) {
      const uint64_t kv_dims[3] = {static_cast<uint64_t>(hk) * 2 * kBD, static_cast<uint64_t>(t),
                                   static_cast<uint64_t>(batch)};
      const uint64_t kv_str[2] = {static_cast<uint64_t>(hk) * 2 * kBD * 4, static_cast<uint64_t>(hk) * 2 * kBD * 4 * t};
      rc = tensor_map(&acc_maps[1], dkv_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, kv_dims, kv_str, box,
                      CU_TENSOR_MAP_SWIZZLE_64B);
    } else {
      acc_maps[1] = acc_maps[0];  // unused: no split items
    }
    if (rc) return rc;
  }
  launch(attn_bwd_tc_kernel, grid, kBwdThreads, kSmemGen, s, maps[0], maps[1], maps[2], maps[3], acc_maps[0],
         acc_maps[1], p);
  SJ_LAUNCH_CHECK("attn_bwd_tc");
  const size_t quads = rows * (hq + (dkv_acc ? hk : 0)) * (kBD / 8);
  launch(attn_dq_finish_kernel, static_cast<unsigned>((quads + 255) / 256), 256, 0, s, dq_acc,
         static_cast<__nv_bfloat16*>(dq), lddq, static_cast<const float*>(dkv_acc), p.dk, lddk, p.dv, lddv,
         static_cast<int>(rows), t, hq, hk, p.rope_tab, p.rope_log_theta);
  SJ_LAUNCH_CHECK("attn_dq_finish");
  return SJ_OK;
}
