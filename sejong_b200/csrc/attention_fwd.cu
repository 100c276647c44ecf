// Causal grouped-query attention forward on the 5th-generation tensor cores (tcgen05 / TMEM / TMA),
// head dim 64, optional sliding window.
//
// Restates python/sejong_kernels/ops/hierarchy.py:7-39 (hierarchy_attention): query (b, t, h) attends
// keys s of kv head h / (HQ/HK) with max(0, t+1-W) <= s <= t, scale 64^-1/2; O and the natural-log
// LSE per (row, head).
//
// Persistent: one CTA per SM walks 128-query tiles of (batch, head), 14 warps:
//   warp 0      TMA: each item's Q tile into one of two Q buffers, then its 128-key K and V tiles
//               into 3-deep rings (K released once S_j is done, V once O_j is), running ahead into
//               the next item.
//   warp 1      TMEM owner and MMA issuer: S_j = Q K_j^T (M128 N128 K64) into one of two TMEM
//               S buffers, then O_j = P_j V_j (M128 N64 K128, P from shared memory) into one of two
//               TMEM O buffers.  S_{j+1} is issued before waiting for P_j, so QK^T of the next tile
//               overlaps the softmax of this one.
//   warps 2-9   softmax: a row of the tile (TMEM lane) is shared by two threads that each take 64
//               of its keys, so row maxima need one exchange per tile and no shuffles.  P_j goes
//               to shared memory in bf16, in the K-major 128-byte-swizzled layout the MMA reads.
//   warps 10-13 correction: fold each O_j (read from TMEM) into the f32 output rows with the
//               online-softmax rescale and write finished rows, off the softmax critical path.
// Every wait is bounded (SJ_DEV_ATTN_WAIT in the device error word), after which each role drains
// and exits.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {

constexpr int kT = 128;           // queries per CTA and keys per tile
constexpr int kD = 64;            // head dim
constexpr int kSoftmaxWarps = 8;
constexpr int kCorrectionWarps = 4;
constexpr int kThreadsTc = 32 * (2 + kSoftmaxWarps + kCorrectionWarps);  // TMA, MMA, softmax, correction
constexpr int kRecSlots = 4;                               // per-tile records in flight
constexpr int kTileBytes = kT * kD * 2;          // 16 KB: 128 rows x 128 B
constexpr int kPBytes = 2 * kTileBytes;          // P: 128 rows x 128 keys bf16, two 64-key halves
constexpr int kKvStages = 3;                     // K and V rings (separately released)
// shared memory: Q0 Q1 | K0..K2 | V0..V2 | P0 P1 | barriers
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kTileBytes;
constexpr int kOffV = kOffK + kKvStages * kTileBytes;
constexpr int kOffP = kOffV + kKvStages * kTileBytes;
// per-tile exchange and records: xmax [2 slots][2 halves][128], xsum [4][2][128], rbase / rmax /
// rrow [4][128], rhead [4]
constexpr int kOffX = kOffP + 2 * kPBytes;
constexpr int kXBytes = (2 * 2 * 128 + 4 * 2 * 128 + 3 * 4 * 128 + 4) * 4;
constexpr int kOffBar = kOffX + ((kXBytes + 127) & ~127);
constexpr int kSmemFwd = kOffBar + 512 + 1024;    // + barriers + alignment slack
constexpr uint32_t kTmemCols = 512;               // S0 S1 (128 each), O0 O1 (64 each)
constexpr uint32_t kColS = 0, kColO = 256;
constexpr float kLog2eTc = 1.4426950408889634f;
constexpr float kLn2Tc = 0.6931471805599453f;

struct FwdParams {
  int t, hq, hk, window, batch, nqt, items;
  float scale_log2;
  __nv_bfloat16* out;
  int ldo;
  float* lse;
};

// 2^x on the special-function unit (PTX ex2.approx, flush-to-zero): the softmax exponent.
SJ_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Work item -> (batch, head, query tile).  Items run heaviest first: all last query tiles (the
// longest causal rows), then the ones before, so a static round-robin over CTAs balances.
struct Item {
  int b, h, qt, q0, kb_lo, nk;
};
SJ_DEVICE Item decode_item(const FwdParams& p, int item) {
  Item it;
  const int bh = p.batch * p.hq;
  const int rest = item % bh;
  it.qt = p.nqt - 1 - item / bh;
  it.b = rest / p.hq;
  it.h = rest % p.hq;
  it.q0 = it.qt * kT;
  it.kb_lo = p.window > 0 ? max(0, it.q0 - p.window + 1) / kT : 0;
  it.nk = min(it.q0 + kT - 1, p.t - 1) / kT - it.kb_lo + 1;
  return it;
}

}  // namespace

// Persistent: one CTA per SM walks the work items blockIdx.x, +gridDim.x, ...  Barrier phases run
// on per-CTA counters: n (items: Q double buffer) and g (key tiles: K/V ring, S, P and O buffers).
__global__ void __launch_bounds__(kThreadsTc, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;           // 2
  uint64_t* q_empty = bars + 2;      // 2
  uint64_t* k_full = bars + 4;       // 3
  uint64_t* k_empty = bars + 7;      // 3
  uint64_t* v_full = bars + 10;      // 3
  uint64_t* v_empty = bars + 13;     // 3
  uint64_t* s_full = bars + 16;      // 2
  uint64_t* p_full = bars + 18;      // 2
  uint64_t* o_full = bars + 20;      // 2
  uint64_t* o_empty = bars + 22;     // 2
  uint64_t* drain = bars + 24;       // 1
  uint64_t* xchg = bars + 25;        // 2: softmax half-row exchange
  uint64_t* rec_full = bars + 27;    // 4: tile records for the correction warps (softmax runs ahead
                                     //    of them by up to three tiles, so two phases would alias)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 31);
  float* xmax = reinterpret_cast<float*>(smem + kOffX);
  float* xsum = xmax + 2 * 2 * kT;
  float* rbase = xsum + kRecSlots * 2 * kT;
  float* rmax = rbase + kRecSlots * kT;
  int* rrow = reinterpret_cast<int*>(rmax + kRecSlots * kT);
  int* rhead = rrow + kRecSlots * kT;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = p.hq / p.hk;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftmaxWarps);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], kCorrectionWarps);
      mbar_init(&xchg[i], kSoftmaxWarps);
    }
    for (int i = 0; i < kRecSlots; ++i) mbar_init(&rec_full[i], kSoftmaxWarps);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_q);
    tma_prefetch_map(&map_k);
    tma_prefetch_map(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // operands may come from the previous kernel
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int n = 0, g = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++n) {
        const Item it = decode_item(p, item);
        const int row_base = it.b * p.t;
        const int qs = n & 1;
        if (!mbar_wait(&q_empty[qs], ((n >> 1) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) break;
        mbar_arrive_expect_tx(&q_full[qs], kTileBytes);
        tma_load_2d(smem + kOffQ + qs * kTileBytes, &map_q, &q_full[qs], it.h * kD, row_base + it.q0);
        const int kvh = it.h / group;
        for (int j = 0; j < it.nk; ++j, ++g) {
          const int st = g % kKvStages;
          const uint32_t ph = static_cast<uint32_t>(g / kKvStages) & 1u;
          const int k0 = (it.kb_lo + j) * kT;
          if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, SJ_DEV_ATTN_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], kTileBytes);
          tma_load_2d(smem + kOffK + st * kTileBytes, &map_k, &k_full[st], kvh * kD, row_base + k0);
          if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, SJ_DEV_ATTN_WAIT)) {
            ok = false;
            ++g;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], kTileBytes);
          tma_load_2d(smem + kOffV + st * kTileBytes, &map_v, &v_full[st], kvh * kD, row_base + k0);
        }
      }
      // drain: copies still in flight into the Q buffers and the K/V rings must land before exit
      for (int i = max(0, n - 2); i < n; ++i) mbar_wait(&q_full[i & 1], (i >> 1) & 1, nullptr, SJ_DEV_ATTN_WAIT);
      for (int i = max(0, g - kKvStages); i < g; ++i) {
        mbar_wait(&k_full[i % kKvStages], (i / kKvStages) & 1, nullptr, SJ_DEV_ATTN_WAIT);
        mbar_wait(&v_full[i % kKvStages], (i / kKvStages) & 1, nullptr, SJ_DEV_ATTN_WAIT);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdescS = umma_idesc_bf16(kT, kT, 0, 0);
      constexpr uint32_t kIdescO = umma_idesc_bf16(kT, kD, 0, 1);
      // O_i = P_i V_i into O buffer i&1 once P_i is written and O_{i-2} has been consumed
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1;
        const int vs = i % kKvStages;
        if (!mbar_wait(&p_full[st], (i >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        if (!mbar_wait(&o_empty[st], ((i >> 1) & 1) ^ 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        if (!mbar_wait(&v_full[vs], (i / kKvStages) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + kOffP + st * kPBytes);
        const uint32_t v_addr = smem_u32(smem + kOffV + vs * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk) {
          const uint64_t da = umma_desc(p_addr + (kk >> 2) * kTileBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t db = umma_desc(v_addr + kk * 2048, 8192, 1024);
          umma_f16(tmem + kColO + st * kD, da, db, kIdescO, kk > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[st]);
        umma_commit(&v_empty[vs]);
        return true;
      };
      int n = 0, g = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++n) {
        const Item it = decode_item(p, item);
        const int qs = n & 1;
        if (!mbar_wait(&q_full[qs], (n >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) break;
        const uint32_t q_addr = smem_u32(smem + kOffQ + qs * kTileBytes);
        for (int j = 0; j < it.nk; ++j, ++g) {
          const int st = g & 1;
          const int ks = g % kKvStages;
          if (!mbar_wait(&k_full[ks], (g / kKvStages) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + kOffK + ks * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t da = umma_desc(q_addr + kk * 32, 16, 1024);
            const uint64_t db = umma_desc(k_addr + kk * 32, 16, 1024);
            umma_f16(tmem + kColS + st * kT, da, db, kIdescS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
          umma_commit(&k_empty[ks]);                       // K_g is read by S_g only
          if (j == it.nk - 1) umma_commit(&q_empty[qs]);  // the item's Q is read by its S products only
          if (g > 0 && !issue_pv(g - 1)) {
            ok = false;
            ++g;
            break;
          }
        }
      }
      if (ok && g > 0) issue_pv(g - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, SJ_DEV_ATTN_WAIT);
    }
  } else if (warp < 2 + kSoftmaxWarps) {
    // softmax warps 2-9: TMEM lane quarter warp % 4 (thread <-> query row r of the item's tile);
    // warps 2-5 take key columns 0-63, warps 6-9 columns 64-127.  The two halves of a row exchange
    // their partial maxima once per tile through shared memory (bounded mbarrier); their partial
    // sums go to the correction warps with the rest of the tile's record.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f, base_prev = 0.f;
    bool alive = true;
    int g = 0;
    for (int item = blockIdx.x; item < p.items && alive; item += gridDim.x) {
      const Item it = decode_item(p, item);
      const int qpos = it.q0 + r;
      for (int j = 0; j < it.nk; ++j, ++g) {
        const int st = g & 1;
        const int rec = g & (kRecSlots - 1);
        const int k0 = (it.kb_lo + j) * kT;
        if (!mbar_wait(&s_full[st], (g >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
          alive = false;
          break;
        }
        tc_fence_after();
        if (j == 0) {
          m = -INFINITY;
          l = 0.f;
          base_prev = 0.f;
        }
        uint32_t sr[64];
        tmem_ld_32x32b_x32(tmem + lane_off + kColS + st * kT + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld_32x32b_x32(tmem + lane_off + kColS + st * kT + half * 64 + 32,
                           *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tmem_wait_ld();
        float* s = reinterpret_cast<float*>(sr);
        // masks only where the tile crosses the causal diagonal, the window edge or the sequence
        // end (uniform over the CTA); valid keys of this row in tile columns: [lo, hi]
        const bool full_tile =
            k0 + kT - 1 <= it.q0 && k0 + kT <= p.t && (p.window <= 0 || it.q0 + kT - 1 - k0 < p.window);
        if (!full_tile) {
          const int hi = min(qpos, p.t - 1) - k0 - half * 64;
          const int lo = p.window > 0 ? qpos - p.window + 1 - k0 - half * 64 : -1;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c < lo || c > hi) s[c] = -INFINITY;
        }
        float pm[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = s[u];
#pragma unroll
        for (int c = 8; c < 64; ++c) pm[c & 7] = fmaxf(pm[c & 7], s[c]);
        const float my_max =
            fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        xmax[(st * 2 + half) * kT + r] = my_max;
        __syncwarp();
        if (lane == 0) mbar_arrive(&xchg[st]);
        if (!mbar_wait(&xchg[st], (g >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
          alive = false;
          break;
        }
        const float other = xmax[(st * 2 + (half ^ 1)) * kT + r];
        const float mx = fmaxf(m, fmaxf(my_max, other) * p.scale_log2);  // running max in log2 units
        const float base = mx == -INFINITY ? 0.f : mx;
        l *= ex2(base_prev - base);
        float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          s[c] = ex2(fmaf(s[c], p.scale_log2, -base));
          ps[c & 7] += s[c];
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        m = mx;
        base_prev = base;
        // the tile's record for the correction warps (4-slot ring, written before P is released)
        const bool last = j == it.nk - 1;
        xsum[(rec * 2 + half) * kT + r] = l;
        if (half == 0) {
          rbase[rec * kT + r] = base;
          rmax[rec * kT + r] = m;
          rrow[rec * kT + r] = (last ? 2 : 0) | (j == 0 ? 1 : 0) | ((qpos < p.t ? it.b * p.t + qpos + 1 : 0) << 2);
          if (r == 0) rhead[rec] = it.h;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rec_full[rec]);
        // P_g overwrites P_{g-2}: its PV product must have finished reading
        if (g >= 2 && !mbar_wait(&o_full[st], ((g - 2) >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
          alive = false;
          break;
        }
        // P in bf16, K-major 128-byte swizzle: this half's 64 keys fill one 16 KB half of P
        uint8_t* pbuf = smem + kOffP + st * kPBytes + half * kTileBytes;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const uint4 w =
              make_uint4(pack_bf16x2(s[8 * c8], s[8 * c8 + 1]), pack_bf16x2(s[8 * c8 + 2], s[8 * c8 + 3]),
                         pack_bf16x2(s[8 * c8 + 4], s[8 * c8 + 5]), pack_bf16x2(s[8 * c8 + 6], s[8 * c8 + 7]));
          *reinterpret_cast<uint4*>(pbuf + r * 128 + ((c8 ^ (r & 7)) << 4)) = w;
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[st]);
      }
    }
  } else {
    // correction warps 10-13: fold each O_g into the f32 output row (thread <-> row, 64 columns)
    // with the online-softmax rescale, and write the row when its item's last tile is in
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float o[kD];
#pragma unroll
    for (int c = 0; c < kD; ++c) o[c] = 0.f;
    float o_base = 0.f;
    int g = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < p.items && alive; item += gridDim.x) {
      const Item it = decode_item(p, item);
      for (int j = 0; j < it.nk; ++j, ++g) {
        const int st = g & 1;
        const int rec = g & (kRecSlots - 1);
        // the tile's record, then O_g
        if (!mbar_wait(&rec_full[rec], (g / kRecSlots) & 1, abort_flag, SJ_DEV_ATTN_WAIT) ||
            !mbar_wait(&o_full[st], (g >> 1) & 1, abort_flag, SJ_DEV_ATTN_WAIT)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const float bi = rbase[rec * kT + r];
        const int info = rrow[rec * kT + r];
        const float scale = (info & 1) ? 0.f : ex2(o_base - bi);
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + lane_off + kColO + st * kD + hc * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[hc * 32 + c] = fmaf(o[hc * 32 + c], scale, __uint_as_float(v[c]));
        }
        o_base = bi;
        // everything read from the record before the O buffer (and with it the slot) is released
        const float lsum = xsum[(rec * 2 + 0) * kT + r] + xsum[(rec * 2 + 1) * kT + r];
        const float mfin = rmax[rec * kT + r];
        const int hh = rhead[rec];
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[st]);
        if ((info & 2) && (info >> 2) > 0) {
          const int row = (info >> 2) - 1;
          const float inv = 1.f / lsum;
          __nv_bfloat16* dst = p.out + static_cast<size_t>(row) * p.ldo + hh * kD;
#pragma unroll
          for (int c8 = 0; c8 < kD / 8; ++c8) {
            const uint4 w = make_uint4(pack_bf16x2(o[8 * c8] * inv, o[8 * c8 + 1] * inv),
                                       pack_bf16x2(o[8 * c8 + 2] * inv, o[8 * c8 + 3] * inv),
                                       pack_bf16x2(o[8 * c8 + 4] * inv, o[8 * c8 + 5] * inv),
                                       pack_bf16x2(o[8 * c8 + 6] * inv, o[8 * c8 + 7] * inv));
            reinterpret_cast<uint4*>(dst)[c8] = w;
          }
          p.lse[static_cast<size_t>(row) * p.hq + hh] = (mfin + log2f(lsum)) * kLn2Tc;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace sj

using namespace sj;

extern "C" int sj_attn_gqa_fwd(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv, void* o,
                               int ldo, float* lse, int batch, int t, int hq, int hk, int head_dim, int window,
                               void* stream) {
  if (head_dim != kD) return fail(SJ_ERR_UNSUPPORTED, "attention: head_dim %d (this build: 64)", head_dim);
  if (batch <= 0 || t <= 0 || hq <= 0 || hk <= 0 || hq % hk || window < 0)
    return fail(SJ_ERR_SHAPE, "attention: bad shape batch=%d t=%d hq=%d hk=%d window=%d", batch, t, hq, hk, window);
  if ((ldq | ldk | ldv | ldo) % 8 || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !lse)
    return fail(SJ_ERR_ARGUMENT, "sj_attn_gqa_fwd: 16-byte aligned rows required");
  static KernelAttrOnce attr_once;
  const int attr_rc = ensure_max_smem(attr_once, reinterpret_cast<const void*>(attn_fwd_tc_kernel), kSmemFwd,
                                      "attention forward shared-memory attribute");
  if (attr_rc != SJ_OK) return attr_rc;
  const uint64_t rows = static_cast<uint64_t>(batch) * t;
  CUtensorMap maps[3];
  int rc = bf16_map(&maps[0], q, static_cast<uint64_t>(hq) * kD, rows, ldq, kD, kT);
  if (!rc) rc = bf16_map(&maps[1], k, static_cast<uint64_t>(hk) * kD, rows, ldk, kD, kT);
  if (!rc) rc = bf16_map(&maps[2], v, static_cast<uint64_t>(hk) * kD, rows, ldv, kD, kT);
  if (rc) return rc;
  FwdParams p;
  p.t = t;
  p.hq = hq;
  p.hk = hk;
  p.window = window;
  p.batch = batch;
  p.nqt = (t + kT - 1) / kT;
  p.items = batch * hq * p.nqt;
  p.scale_log2 = 0.125f * kLog2eTc;
  p.out = static_cast<__nv_bfloat16*>(o);
  p.ldo = ldo;
  p.lse = lse;
  const int grid = std::min(p.items, sm_count());
  launch(attn_fwd_tc_kernel, grid, kThreadsTc, kSmemFwd, as_stream(stream), maps[0], maps[1], maps[2], p);
  SJ_LAUNCH_CHECK("attn_fwd_tc");
  return SJ_OK;
}
