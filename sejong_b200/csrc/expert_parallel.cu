// Expert parallelism for the MoE blocks: the experts of a layer are sharded over the ranks of the
// data-parallel group (experts / world per rank) and the routed rows travel over NVLink as plain
// peer loads and stores into a symmetric heap -- one device allocation of the same size on every
// rank, mapped into every peer with CUDA IPC, so a buffer has the same offset everywhere.
//
// The reference runs every expert on one device (crates/sejong-gpu/src/hierarchy_ops.rs:280-454);
// sharding is this build's addition, designed so that a step over world ranks computes what one
// device computes on the ranks' batches concatenated in rank order:
//   * every rank routes its own rows (sj_route_topk) and publishes its per-expert counts into row
//     `rank` of every rank's count matrix; from the full matrix each rank derives the packed layout
//     of every owner: expert e's segment (padded to 128 rows) holds the rows of rank 0, then rank
//     1, ..., each in slot order -- the order of the single-device pack on the concatenated batch;
//   * dispatch pushes each routed row into its owner's packed A; the owner zeroes its padding rows;
//   * the owner runs the grouped expert GEMMs on its own segments only;
//   * combine pulls the expert outputs back (one writer per output element, deterministic);
//   * backward: the source pushes gate * dy into the owner's d_out and pulls <out, dy> for the gate
//     gradient; the owner runs the backward GEMMs; the source pulls dA and sums its k rows.
// Ordering between ranks is a flag barrier: each rank stores an epoch into its slot of every
// peer's flag array (release, system scope) and waits (acquire) until every slot of its own array
// has reached that epoch.  Epochs come from a per-rank device counter that every barrier advances,
// so a captured graph replays correctly.  Every wait is bounded; on expiry it records
// SJ_DEV_EP_WAIT and the kernel returns.
#include <cstring>
#include <initializer_list>

#include "common.cuh"
#include "internal.h"

namespace sj {

namespace {
constexpr int kMaxRanks = 8;
constexpr int kMaxExperts = 32;
constexpr int kSegment = 128;
constexpr int kPackThreads = 1024;

// Heap base address of every rank (index = rank), passed by value.
struct Peers {
  uint64_t base[kMaxRanks];
};

template <typename T>
SJ_DEVICE T* at(const Peers& p, int r, size_t off) {
  return reinterpret_cast<T*>(p.base[r] + off);
}

SJ_DEVICE void flag_release(uint32_t* flag, uint32_t v) {
  asm volatile("st.release.sys.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}
SJ_DEVICE uint32_t flag_acquire(const uint32_t* flag) {
  uint32_t v;
  asm volatile("ld.acquire.sys.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
  return v;
}
// Bounded wait until *flag has reached `epoch` (wrap-safe comparison).
SJ_DEVICE bool flag_wait(const uint32_t* flag, uint32_t epoch, uint64_t limit_ns) {
  if (static_cast<int32_t>(flag_acquire(flag) - epoch) >= 0) return true;
  const uint64_t start = globaltimer();
  while (static_cast<int32_t>(flag_acquire(flag) - epoch) < 0) {
    if (globaltimer() - start > limit_ns) {
      record_error(SJ_DEV_EP_WAIT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Signal every rank, then wait for every rank (threads 0 .. world-1 of the calling CTA).  Returns
// false in the thread whose wait expired (SJ_DEV_EP_WAIT is then in the device error word).
SJ_DEVICE bool exchange_epoch(const Peers& peers, int rank, int world, size_t flags_off, uint32_t epoch,
                              uint64_t limit_ns) {
  const int t = threadIdx.x;
  if (t < world) flag_release(at<uint32_t>(peers, t, flags_off) + rank, epoch);
  if (t < world) return flag_wait(at<uint32_t>(peers, rank, flags_off) + t, epoch, limit_ns);
  return true;
}

SJ_DEVICE void load8_bf16(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
}  // namespace

// A barrier over the ranks: every earlier write of this GPU (its earlier kernels included) is
// visible to every rank before any rank leaves.  One CTA of 32 threads.
__global__ void ep_barrier_kernel(Peers peers, int rank, int world, size_t flags_off, uint32_t* epoch_ctr,
                                  uint64_t limit_ns) {
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(epoch_ctr) + 1u;
  __threadfence_system();
  exchange_epoch(peers, rank, world, flags_off, epoch, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) *epoch_ctr = epoch;
}

// Count exchange and layout.  One CTA: histogram of this rank's routed slots, counts published to
// every rank, barrier, then from the full [world][experts] matrix: this rank's segments
// (group_rows[0..local] = segment starts and end, group_rows[local+1+g] = end of the valid rows of
// segment g) and, for every slot of this rank, its row in the owner's packed buffer (pos).
__global__ void __launch_bounds__(kPackThreads) ep_route_pack_kernel(const int32_t* ids, int slots, int experts,
                                                                     int rank, int world, Peers peers,
                                                                     size_t counts_off, size_t flags_off,
                                                                     uint32_t* epoch_ctr, uint64_t limit_ns,
                                                                     int32_t* group_rows, int32_t* pos, int cap) {
  pdl_wait();
  __shared__ int count[kMaxExperts], base[kMaxExperts];
  __shared__ int warp_count[kPackThreads / 32][kMaxExperts];
  __shared__ int overflow;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int local = experts / world;
  if (t < kMaxExperts) count[t] = 0;
  if (t == 0) overflow = 0;
  __syncthreads();
  for (int i = t; i < slots; i += kPackThreads) {
    const int e = ids[i];
    if (e >= 0 && e < experts) atomicAdd(&count[e], 1);
  }
  __syncthreads();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(epoch_ctr) + 1u;
  for (int i = t; i < world * experts; i += kPackThreads) {
    const int r = i / experts, e = i % experts;
    reinterpret_cast<volatile int*>(at<int>(peers, r, counts_off))[rank * experts + e] = count[e];
  }
  __threadfence_system();
  __syncthreads();
  // A peer that never arrived leaves the count matrix stale: route nothing on it (the same exit as
  // an overflow) and leave the epoch counter where it was.  After SJ_DEV_EP_WAIT the ranks' epoch
  // counters disagree, so the expert-parallel context must be rebuilt before another step.
  if (!exchange_epoch(peers, rank, world, flags_off, epoch, limit_ns)) overflow = 2;
  __syncthreads();
  if (t == 0 && !overflow) {
    *epoch_ctr = epoch;
    __threadfence_system();
    const volatile int* m = at<int>(peers, rank, counts_off);
    int off = 0;
    for (int e = 0; e < experts; ++e) {
      const int g = e % local;
      if (g == 0) off = 0;
      int total = 0, before = 0;
      for (int s = 0; s < world; ++s) {
        const int c = m[s * experts + e];
        total += c;
        if (s < rank) before += c;
      }
      base[e] = off + before;
      if (e / local == rank) {
        group_rows[g] = off;
        group_rows[local + 1 + g] = off + total;
      }
      off += (total + kSegment - 1) / kSegment * kSegment;
      if (g == local - 1) {
        if (e / local == rank) group_rows[local] = off;
        if (off > cap) overflow = 1;
      }
    }
  }
  __syncthreads();
  if (overflow) {  // a receive buffer would overflow (the host sizes cap so this cannot happen), or the
                   // count exchange timed out: route nothing
    if (t == 0 && overflow == 1) record_error(SJ_DEV_EP_CAPACITY);
    for (int i = t; i < slots; i += kPackThreads) pos[i] = -1;
    for (int i = t; i <= 2 * local; i += kPackThreads) group_rows[i] = 0;
    return;
  }
  for (int c0 = 0; c0 < slots; c0 += kPackThreads) {
    const int i = c0 + t;
    const int e = i < slots ? ids[i] : -1;
    const unsigned lt = (1u << lane) - 1u;
    int r = 0;
    for (int x = 0; x < experts; ++x) {
      const unsigned msk = __ballot_sync(0xffffffffu, e == x);
      if (lane == 0) warp_count[warp][x] = __popc(msk);
      if (e == x) r = __popc(msk & lt);
    }
    __syncthreads();
    if (e >= 0 && e < experts) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += warp_count[w][e];
      pos[i] = base[e] + before + r;
    } else if (i < slots) {
      pos[i] = -1;
    }
    __syncthreads();
    if (t < experts) {
      int total = 0;
      for (int w = 0; w < kPackThreads / 32; ++w) total += warp_count[w][t];
      base[t] += total;
    }
    __syncthreads();
  }
}

// Zero the padding rows [fill_g, start_{g+1}) of this rank's segments in the packed buffer `dst`
// (thread index i over local * 128 rows * d/8 vectors).
SJ_DEVICE void zero_padding(__nv_bfloat16* dst, const int32_t* group_rows, int local, int d, size_t i) {
  const int vpr = d / 8;
  const int g = static_cast<int>(i / (static_cast<size_t>(kSegment) * vpr));
  if (g >= local) return;
  const int r = group_rows[local + 1 + g] + static_cast<int>((i / vpr) % kSegment);
  const int c = static_cast<int>(i % vpr) * 8;
  if (r < group_rows[g + 1]) *reinterpret_cast<uint4*>(dst + static_cast<size_t>(r) * d + c) = make_uint4(0u, 0u, 0u, 0u);
}

// Push every routed row z[slot / k] into A at its owner (thread per 8 columns), then the padding.
__global__ void ep_dispatch_kernel(const __nv_bfloat16* z, int ldz, const int32_t* ids, const int32_t* pos, int slots,
                                   int k, int d, int local, Peers peers, int rank, size_t a_off,
                                   const int32_t* group_rows) {
  pdl_wait();
  const int vpr = d / 8;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t push = static_cast<size_t>(slots) * vpr;
  if (i < push) {
    const int s = static_cast<int>(i / vpr), c = static_cast<int>(i % vpr) * 8;
    const int e = ids[s], p = pos[s];
    if (p < 0 || e < 0) return;
    const uint4 v = *reinterpret_cast<const uint4*>(z + static_cast<size_t>(s / k) * ldz + c);
    *reinterpret_cast<uint4*>(at<__nv_bfloat16>(peers, e / local, a_off) + static_cast<size_t>(p) * d + c) = v;
    return;
  }
  zero_padding(at<__nv_bfloat16>(peers, rank, a_off), group_rows, local, d, i - push);
}

// y[t] = x[t] + sum_j gate[t, j] out_owner(j)[pos[t, j]], pulled from the owners; thread per 8 columns.
__global__ void ep_combine_kernel(Peers peers, size_t out_off, const int32_t* ids, const int32_t* pos,
                                  const float* gates, const float* x, float* y, int rows, int k, int d, int local) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int vpr = d / 8;
  if (i >= static_cast<size_t>(rows) * vpr) return;
  const int t = static_cast<int>(i / vpr), c = static_cast<int>(i % vpr) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const size_t s = static_cast<size_t>(t) * k + j;
    const int p = pos[s], e = ids[s];
    if (p < 0 || e < 0) continue;
    const float g = gates[s];
    float v[8];
    load8_bf16(at<__nv_bfloat16>(peers, e / local, out_off) + static_cast<size_t>(p) * d + c, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = fmaf(g, v[q], acc[q]);
  }
  const float4* xs = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * d + c);
  const float4 a = xs[0], b = xs[1];
  float4* ys = reinterpret_cast<float4*>(y + static_cast<size_t>(t) * d + c);
  ys[0] = make_float4(a.x + acc[0], a.y + acc[1], a.z + acc[2], a.w + acc[3]);
  ys[1] = make_float4(b.x + acc[4], b.y + acc[5], b.z + acc[6], b.w + acc[7]);
}

// Warp per slot: d_out_owner[pos] = gate * dy[t] (pushed, bf16), d_gates[slot] = <out_owner[pos], dy[t]>
// (pulled); the warps past the slots zero the padding rows of this rank's d_out.
__global__ void ep_combine_bwd_kernel(Peers peers, size_t out_off, size_t d_out_off, const int32_t* ids,
                                      const int32_t* pos, const float* gates, const float* dy, float* d_gates,
                                      const int32_t* group_rows, int slots, int k, int d, int local, int rank) {
  pdl_wait();
  const size_t w = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<size_t>(slots)) {
    const size_t rows_done = w - slots;  // a warp zeroes one padding row candidate: 32 lanes x d/32 columns
    const int vpr = d / 8;
    for (int c = lane; c < vpr; c += 32)
      zero_padding(at<__nv_bfloat16>(peers, rank, d_out_off), group_rows, local, d, rows_done * vpr + c);
    return;
  }
  const int s = static_cast<int>(w);
  const int e = ids[s], p = pos[s];
  if (p < 0 || e < 0) {
    if (lane == 0) d_gates[s] = 0.f;
    return;
  }
  const int o = e / local;
  const __nv_bfloat16* src = at<__nv_bfloat16>(peers, o, out_off) + static_cast<size_t>(p) * d;
  __nv_bfloat16* dst = at<__nv_bfloat16>(peers, o, d_out_off) + static_cast<size_t>(p) * d;
  const int t = s / k;
  const float g = gates[s];
  float dot = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    float v[8];
    load8_bf16(src + c, v);
    const float4* ds = reinterpret_cast<const float4*>(dy + static_cast<size_t>(t) * d + c);
    const float4 a = ds[0], b = ds[1];
    const float q[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint4 u;
    u.x = pack_bf16x2(g * q[0], g * q[1]);
    u.y = pack_bf16x2(g * q[2], g * q[3]);
    u.z = pack_bf16x2(g * q[4], g * q[5]);
    u.w = pack_bf16x2(g * q[6], g * q[7]);
    *reinterpret_cast<uint4*>(dst + c) = u;
#pragma unroll
    for (int q2 = 0; q2 < 8; ++q2) dot = fmaf(v[q2], q[q2], dot);
  }
  dot = warp_sum(dot);
  if (lane == 0) d_gates[s] = dot;
}

// dz[t] = sum_j dA_owner(j)[pos[t, j]] (f32 rows pulled from the owners); thread per 8 columns.
__global__ void ep_dispatch_bwd_kernel(Peers peers, size_t da_off, const int32_t* ids, const int32_t* pos, float* dz,
                                       int ldz, int rows, int k, int d, int local) {
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int vpr = d / 8;
  if (i >= static_cast<size_t>(rows) * vpr) return;
  const int t = static_cast<int>(i / vpr), c = static_cast<int>(i % vpr) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const size_t s = static_cast<size_t>(t) * k + j;
    const int p = pos[s], e = ids[s];
    if (p < 0 || e < 0) continue;
    const float4* src = reinterpret_cast<const float4*>(at<float>(peers, e / local, da_off) + static_cast<size_t>(p) * d + c);
    const float4 a = src[0], b = src[1];
    acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
    acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
  }
  float4* o = reinterpret_cast<float4*>(dz + static_cast<size_t>(t) * ldz + c);
  o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

}  // namespace sj

using namespace sj;

namespace {
int make_peers(const void* const* peers, int rank, int world, Peers* out, const char* what) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(SJ_ERR_SHAPE, "%s: rank %d of world %d (1 <= world <= %d)", what, rank, world, kMaxRanks);
  if (!peers) return fail(SJ_ERR_ARGUMENT, "%s: null peer table", what);
  *out = Peers{};
  for (int r = 0; r < world; ++r) {
    if (!peers[r] || !aligned16(peers[r])) return fail(SJ_ERR_ARGUMENT, "%s: heap base of rank %d", what, r);
    out->base[r] = reinterpret_cast<uint64_t>(peers[r]);
  }
  return SJ_OK;
}
bool offsets_aligned(std::initializer_list<size_t> offs) {
  for (size_t o : offs)
    if (o % 16) return false;
  return true;
}
uint64_t limit_ns(int timeout_ms) { return static_cast<uint64_t>(timeout_ms > 0 ? timeout_ms : 1) * 1000000ull; }
}  // namespace

extern "C" int sj_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(SJ_ERR_ARGUMENT, "sj_ipc_alloc: bytes=%zu", bytes);
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    return fail(SJ_ERR_CAPACITY, "sj_ipc_alloc: %zu bytes required, %zu available", bytes, free_b);
  }
  int rc = zero_async(p, bytes, nullptr);
  if (rc == SJ_OK) rc = cuda_check(cudaStreamSynchronize(nullptr), "sj_ipc_alloc: zero fill");
  if (rc != SJ_OK) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return SJ_OK;
}

extern "C" int sj_ipc_free(void* ptr) { return ptr ? cuda_check(cudaFree(ptr), "sj_ipc_free") : SJ_OK; }

extern "C" int sj_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return fail(SJ_ERR_ARGUMENT, "sj_ipc_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == SJ_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  const int rc = cuda_check(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "sj_ipc_handle");
  if (rc == SJ_OK) memcpy(handle, &h, sizeof(h));
  return rc;
}

extern "C" int sj_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(SJ_ERR_ARGUMENT, "sj_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cuda_check(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "sj_ipc_open");
}

extern "C" int sj_ipc_close(void* ptr) { return ptr ? cuda_check(cudaIpcCloseMemHandle(ptr), "sj_ipc_close") : SJ_OK; }

extern "C" int sj_ep_receive_capacity(int rows, int k, int experts, int world) {
  if (rows <= 0 || k <= 0 || experts <= 0 || world <= 0 || experts % world) return 0;
  const int local = experts / world;
  const long long need = static_cast<long long>(rows) * world * k + static_cast<long long>(local) * (kSegment - 1);
  if (need > (1ll << 30)) return 0;
  return static_cast<int>((need + kSegment - 1) / kSegment * kSegment);
}

extern "C" int sj_ep_barrier(int rank, int world, const void* const* peers, size_t flags_off, uint32_t* epoch,
                             int timeout_ms, void* stream) {
  Peers p;
  int rc = make_peers(peers, rank, world, &p, "sj_ep_barrier");
  if (rc != SJ_OK) return rc;
  if (!epoch || flags_off % 4) return fail(SJ_ERR_ARGUMENT, "sj_ep_barrier: epoch counter / flag offset");
  launch(ep_barrier_kernel, 1, 32, 0, as_stream(stream), p, rank, world, flags_off, epoch, limit_ns(timeout_ms));
  SJ_LAUNCH_CHECK("ep_barrier");
  return SJ_OK;
}

extern "C" int sj_ep_route_pack(const int32_t* ids, int rows, int experts, int k, int rank, int world,
                                const void* const* peers, size_t counts_off, size_t flags_off, uint32_t* epoch,
                                int32_t* group_rows, int32_t* pos, int cap, int timeout_ms, void* stream) {
  Peers p;
  int rc = make_peers(peers, rank, world, &p, "sj_ep_route_pack");
  if (rc != SJ_OK) return rc;
  if (rows <= 0 || k <= 0 || experts <= 0 || experts > kMaxExperts || experts % world)
    return fail(SJ_ERR_SHAPE, "sj_ep_route_pack: rows=%d k=%d experts=%d (<= %d, a multiple of world %d)", rows, k,
                experts, kMaxExperts, world);
  if (cap < sj_ep_receive_capacity(rows, k, experts, world))
    return fail(SJ_ERR_CAPACITY, "sj_ep_route_pack: capacity %d below sj_ep_receive_capacity %d", cap,
                sj_ep_receive_capacity(rows, k, experts, world));
  if (!ids || !group_rows || !pos || !epoch || counts_off % 4 || flags_off % 4)
    return fail(SJ_ERR_ARGUMENT, "sj_ep_route_pack: null pointer or unaligned offset");
  launch(ep_route_pack_kernel, 1, kPackThreads, 0, as_stream(stream), ids, rows * k, experts, rank, world, p,
         counts_off, flags_off, epoch, limit_ns(timeout_ms), group_rows, pos, cap);
  SJ_LAUNCH_CHECK("ep_route_pack");
  return SJ_OK;
}

extern "C" int sj_ep_dispatch(const void* z, int ldz, const int32_t* ids, const int32_t* pos, int rows, int k, int d,
                              int experts, int rank, int world, const void* const* peers, size_t a_off,
                              const int32_t* group_rows, void* stream) {
  Peers p;
  int rc = make_peers(peers, rank, world, &p, "sj_ep_dispatch");
  if (rc != SJ_OK) return rc;
  if (rows <= 0 || k <= 0 || d <= 0 || d % 8 || ldz % 8 || experts <= 0 || experts % world)
    return fail(SJ_ERR_SHAPE, "sj_ep_dispatch: bad shape");
  if (!aligned16(z) || !ids || !pos || !group_rows || !offsets_aligned({a_off}))
    return fail(SJ_ERR_ARGUMENT, "sj_ep_dispatch: aligned operands");
  const int local = experts / world;
  const size_t n = (static_cast<size_t>(rows) * k + static_cast<size_t>(local) * kSegment) * (d / 8);
  launch(ep_dispatch_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream),
         static_cast<const __nv_bfloat16*>(z), ldz, ids, pos, rows * k, k, d, local, p, rank, a_off, group_rows);
  SJ_LAUNCH_CHECK("ep_dispatch");
  return SJ_OK;
}

extern "C" int sj_ep_combine(const void* const* peers, int world, size_t out_off, const int32_t* ids,
                             const int32_t* pos, const float* gates, const float* x, float* y, int rows, int k, int d,
                             int experts, void* stream) {
  Peers p;
  int rc = make_peers(peers, 0, world, &p, "sj_ep_combine");
  if (rc != SJ_OK) return rc;
  if (rows <= 0 || k <= 0 || d <= 0 || d % 8 || experts <= 0 || experts % world)
    return fail(SJ_ERR_SHAPE, "sj_ep_combine: bad shape");
  if (!aligned16(x) || !aligned16(y) || !ids || !pos || !gates || !offsets_aligned({out_off}))
    return fail(SJ_ERR_ARGUMENT, "sj_ep_combine: aligned operands");
  const size_t n = static_cast<size_t>(rows) * (d / 8);
  launch(ep_combine_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream), p, out_off, ids, pos,
         gates, x, y, rows, k, d, experts / world);
  SJ_LAUNCH_CHECK("ep_combine");
  return SJ_OK;
}

extern "C" int sj_ep_combine_bwd(const void* const* peers, int rank, int world, size_t out_off, size_t d_out_off,
                                 const int32_t* ids, const int32_t* pos, const float* gates, const float* dy,
                                 float* d_gates, const int32_t* group_rows, int rows, int k, int d, int experts,
                                 void* stream) {
  Peers p;
  int rc = make_peers(peers, rank, world, &p, "sj_ep_combine_bwd");
  if (rc != SJ_OK) return rc;
  if (rows <= 0 || k <= 0 || d <= 0 || d % 8 || experts <= 0 || experts % world)
    return fail(SJ_ERR_SHAPE, "sj_ep_combine_bwd: bad shape");
  if (!aligned16(dy) || !ids || !pos || !gates || !d_gates || !group_rows || !offsets_aligned({out_off, d_out_off}))
    return fail(SJ_ERR_ARGUMENT, "sj_ep_combine_bwd: aligned operands");
  const int local = experts / world;
  const size_t warps = static_cast<size_t>(rows) * k + static_cast<size_t>(local) * kSegment;
  launch(ep_combine_bwd_kernel, static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, as_stream(stream), p, out_off,
         d_out_off, ids, pos, gates, dy, d_gates, group_rows, rows * k, k, d, local, rank);
  SJ_LAUNCH_CHECK("ep_combine_bwd");
  return SJ_OK;
}

extern "C" int sj_ep_dispatch_bwd(const void* const* peers, int world, size_t da_off, const int32_t* ids,
                                  const int32_t* pos, float* dz, int ldz, int rows, int k, int d, int experts,
                                  void* stream) {
  Peers p;
  int rc = make_peers(peers, 0, world, &p, "sj_ep_dispatch_bwd");
  if (rc != SJ_OK) return rc;
  if (rows <= 0 || k <= 0 || d <= 0 || d % 8 || ldz % 4 || experts <= 0 || experts % world)
    return fail(SJ_ERR_SHAPE, "sj_ep_dispatch_bwd: bad shape");
  if (!aligned16(dz) || !ids || !pos || !offsets_aligned({da_off}))
    return fail(SJ_ERR_ARGUMENT, "sj_ep_dispatch_bwd: aligned operands");
  const size_t n = static_cast<size_t>(rows) * (d / 8);
  launch(ep_dispatch_bwd_kernel, static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream), p, da_off, ids,
         pos, dz, ldz, rows, k, d, experts / world);
  SJ_LAUNCH_CHECK("ep_dispatch_bwd");
  return SJ_OK;
}
