/*
 * sejong.h — C ABI of libsejong_b200.so, the sm_100a (B200) replacement for the
 * GPU operations of Sejong's byte / NativeValue Transformer training step.
 *
 * The reference reaches its kernels through Rust `Engine` methods that all end
 * in `Engine::launch(name, args, constants, grid)` (crates/sejong-gpu/src/lib.rs:
 * 366-487).  Each function below is the C-ABI form of one of those methods (or of a
 * fused group of them); the comment on each names the reference method and
 * kernel it replaces (file:line, paths relative to the reference project).
 *
 * Conventions
 *  - Plain device pointers, element counts and leading dimensions (in elements);
 *    matrices are row-major.  The caller owns every buffer; the library never
 *    allocates or frees caller memory.  Scratch ("workspace") is passed in.
 *  - Every call takes the `cudaStream_t` to launch on as `void* stream` and does
 *    not synchronise.
 *  - Return value: SJ_OK (0) or one of the SJ_ERR_* codes; `sj_last_error()`
 *    returns a thread-local message for the last failing call on this thread
 *    (mirrors sejong_core::Error, crates/sejong-core/src/lib.rs:8-25).
 *  - Device-side failures (a bounded wait that expired) never trap: the kernel
 *    writes a code into a device error word and returns; `sj_device_error()`
 *    reads (and optionally clears) it.
 */
#ifndef SEJONG_B200_H
#define SEJONG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum {
  SJ_OK = 0,
  SJ_ERR_SHAPE = 1,       /* shape / dimension mismatch (reference: Error::Message from ensure) */
  SJ_ERR_CAPACITY = 2,    /* not enough device memory / workspace (Error::Capacity) */
  SJ_ERR_CUDA = 3,        /* a CUDA runtime or driver call failed */
  SJ_ERR_NCCL = 4,        /* a collective failed */
  SJ_ERR_TIMEOUT = 5,     /* a bounded device-side wait expired */
  SJ_ERR_ARGUMENT = 6,    /* bad pointer alignment, dtype or flag */
  SJ_ERR_UNSUPPORTED = 7  /* valid request this build does not implement */
};

/* dtype codes: the reference's DType discriminants (crates/sejong-core/src/lib.rs:34-41) plus bf16 */
enum { SJ_F32 = 0, SJ_F64 = 1, SJ_F16 = 2, SJ_I32 = 3, SJ_BF16 = 4 };

/* device error codes written by kernels */
enum {
  SJ_DEV_GEMM_PRODUCER_WAIT = 101,
  SJ_DEV_GEMM_MMA_WAIT = 102,
  SJ_DEV_GEMM_EPILOGUE_WAIT = 103,
  SJ_DEV_GEMM_DRAIN_WAIT = 104,
  SJ_DEV_ATTN_WAIT = 105,
  SJ_DEV_SMEM_ALIGN = 106,  /* a kernel's dynamic shared memory lacked the alignment its layout needs */
  SJ_DEV_BAD_INDEX = 110,
  SJ_DEV_EP_WAIT = 111,     /* an expert-parallel barrier gave up waiting for a peer */
  SJ_DEV_EP_CAPACITY = 112  /* an expert-parallel receive buffer would overflow */
};

int sj_version(void);
const char* sj_last_error(void);
/* Initialise `device` (make current, resolve cuTensorMapEncodeTiled, set kernel
 * shared-memory limits).  Replaces Engine::new's device setup
 * (crates/sejong-gpu/src/lib.rs:197-233, hip.rs:126-178). */
int sj_device_init(int device);
/* Free / total device memory: the budget source of the reference allocator and
 * batch planner (crates/sejong-gpu/src/hip.rs:154-160,182-194). */
int sj_mem_info(size_t* free_bytes, size_t* total_bytes);
/* Read the device error word; clear it when `clear` != 0.  Synchronises `stream`. */
int sj_device_error(int* code, int clear, void* stream);
/* Zero `bytes` bytes at `ptr` on `stream` (Engine::full(.., 0), crates/sejong-gpu/src/lib.rs:544-553). */
int sj_zero(void* ptr, size_t bytes, void* stream);

/* ------------------------------------------------------------------ host: RNG and bytes (bit-exact) */
/* Rng::next_u64 (crates/sejong-core/src/lib.rs:599-605). */
uint64_t sj_rng_next_u64(uint64_t* state);
/* Rng::index (lib.rs:609-618). */
uint64_t sj_rng_index(uint64_t* state, uint64_t size);
/* n draws of Rng::normal (lib.rs:619-621) times `scale`, f32 arithmetic. */
int sj_rng_normal_fill(uint64_t* state, float* out, size_t n, float scale);
/* Synthetic document: n bytes i.i.d. Zipf(s) over 0..255 by inverse CDF of Rng::uniform. */
int sj_zipf_bytes(uint64_t seed, double s, uint8_t* out, size_t n);
/* Corpus::batch (crates/sejong-train/src/lib.rs:72-88) over the token stream
 * `tokens` (EOS + bytes + ... + EOS, lib.rs:24-71). */
int sj_corpus_batch(const int32_t* tokens, size_t n_tokens, uint64_t* rng_state, int batch, int sequence,
                    int32_t* inputs, int32_t* targets);
/* BLAKE3 (32-byte plain hash) of the concatenation of `count` parts, streamed (host code).  Used for
 * Corpus::open's fingerprint (crates/sejong-train/src/lib.rs:24-51: the blake3 crate over a domain
 * string and, per document, its u64 little-endian length and bytes), which checkpoints carry and a
 * resume compares. */
int sj_blake3(const void* const* parts, const uint64_t* lengths, int count, uint8_t* out);

/* ------------------------------------------------------------------ GEMM (tcgen05 / TMEM / TMA) */
/* Epilogues of sj_gemm. */
enum {
  SJ_EPI_STORE = 0,    /* C = alpha*acc                         (C bf16 or f32) */
  SJ_EPI_ACCUM = 1,    /* C += alpha*acc                        (C f32; split-K allowed) */
  SJ_EPI_RESIDUAL = 2, /* C = aux + alpha*acc                   (C, aux both bf16 or both f32; aux row
                          stride ld_aux) */
  SJ_EPI_SWIGLU = 3,   /* C = round(acc) (gate/up interleaved by 16 columns, bf16);
                          aux = silu(g)*u  [M, N/2] bf16 with row stride ld_aux */
  SJ_EPI_ROPE = 4,     /* C = RoPE(acc) on columns < rope_cols (head dim 64, pairs 2i,2i+1,
                          position = row mod rope_t), bf16; aux = the sj_rope_table of rope_t
                          positions (or null: angles evaluated inline from rope_theta) */
  /* sj_gemm_bias only (f32 bias [N]): */
  SJ_EPI_BIAS = 5,          /* C = alpha*acc + bias                        (C bf16 or f32) */
  SJ_EPI_BIAS_GELU = 6,     /* C = gelu(alpha*acc + bias), erf GELU         (C bf16 or f32) */
  SJ_EPI_BIAS_RESIDUAL = 7  /* C = aux + alpha*acc + bias (aux same dtype as C, row stride ld_aux) */
};
/* table[p*hd/2 + i] = (cos, sin) of (p + offset) * exp((-2 i / hd) * ln theta) for p < t, in f32 as
 * the reference's rope kernel evaluates it (python/sejong_kernels/ops/kernels.py:103-113).
 * `table` holds t*hd floats (t*hd/2 pairs). */
int sj_rope_table(float* table, int t, int head_dim, int offset, float theta, void* stream);
/* C[M,N] = op(A)[M,K] * op(B)[K,N], bf16 operands, f32 accumulation in TMEM.
 * a_trans: A stored [K,M] (lda >= M) instead of [M,K]; b_trans: B stored [N,K]
 * instead of [K,N] — the TA/TB flags of Engine::matmul (crates/sejong-gpu/src/
 * lib.rs:594-649, kernel python/sejong_kernels/ops/kernels.py:23-39) and of the
 * tape's backward rules dA = dY*B^T, dB = A^T*dY (crates/sejong-gpu/src/graph.rs:
 * 817-853).  Also covers Engine::project_qkv (projection_ops.rs:6-43, with
 * SJ_EPI_ROPE folding Engine::rope, lib.rs:734-758) and Engine::gate_up
 * (projection_ops.rs:45-79, SJ_EPI_SWIGLU).  `split_k` > 1 is valid with
 * SJ_EPI_ACCUM only.  Leading dimensions must be multiples of 8 elements and
 * A/B 16-byte aligned (TMA). */
int sj_gemm(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c, int ldc, int c_dtype,
            int m, int n, int k, int epilogue, float alpha, void* aux, int ld_aux, int rope_cols, int rope_t,
            float rope_theta, int split_k, void* stream);
/* sj_gemm with a bias epilogue: the reference's `linear` (x W^T then Engine::bias_add, crates/
 * sejong-model/src/native/bert.rs:335-347; common.py:27-30), optionally followed by Engine::gelu
 * (crates/sejong-gpu/src/lib.rs:985-994; kernels.py:227-232) or by the residual add of the post-LN
 * block (bert.rs:393-406).  epilogue: SJ_EPI_BIAS, SJ_EPI_BIAS_GELU or SJ_EPI_BIAS_RESIDUAL; bias
 * f32 [N], 16-byte aligned. */
int sj_gemm_bias(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c, int ldc,
                 int c_dtype, int m, int n, int k, int epilogue, float alpha, const float* bias, void* aux,
                 int ld_aux, void* stream);

/* The tile plan sj_gemm / sj_gemm_bias would launch for this shape on the current device:
 * plan[0] = tile width BN (128, 192 or 256), plan[1] = split-K count, plan[2] = 1 when the product
 * runs on CTA pairs (tcgen05 cta_group::2, 256-row tiles).  Nothing is launched.  Counterpart of
 * the reference's per-shape grid choice (crates/sejong-gpu/src/projection_ops.rs:6-79). */
int sj_gemm_plan(int m, int n, int k, int a_trans, int b_trans, int c_dtype, int epilogue, int split_k, int* plan);

/* ------------------------------------------------------------------ normalisation, embedding, elementwise */
/* Engine::norm / rmsnorm (crates/sejong-gpu/src/lib.rs:688-699; kernels.py:54-61).
 * x [rows,d] (x_dtype bf16 or f32), w f32 [d]; y bf16 [rows,d]; inv_rms f32 [rows] (optional).
 * x, y and w 16-byte aligned; d a multiple of 8 up to 1024. */
int sj_rmsnorm_fwd(const void* x, int x_dtype, const float* w, void* y, float* inv_rms, int rows, int d, float eps,
                   void* stream);
/* Engine::norm_backward (crates/sejong-gpu/src/norm_ops.rs:14-134; kernels.py:63-87) fused with the
 * residual gradient accumulation of the tape (graph.rs:503-513):
 *   dres[r,:] += rms_dx(x, w, dz) ;  dres_bf16 = bf16(dres) (optional) ;  dw += sum_r dz*x*inv.
 * x bf16 or f32 (x_dtype), dz f32, dres f32 (in/out), dw f32 accumulated.  `partials` is workspace
 * of at least sj_rmsnorm_workspace(rows, d) floats.  x, dz, dres, dres_bf16 and w 16-byte aligned. */
size_t sj_rmsnorm_workspace(int rows, int d);
int sj_rmsnorm_bwd(const void* x, int x_dtype, const float* w, const float* inv_rms, const float* dz, float* dres,
                   void* dres_bf16, float* dw, float* partials, int rows, int d, void* stream);
/* The same with accumulate = 0: dres = rms_dx(x, w, dz) (overwritten, not read), for the first
 * gradient into a residual stream, which saves zero-filling it. */
int sj_rmsnorm_bwd_ex(const void* x, int x_dtype, const float* w, const float* inv_rms, const float* dz, float* dres,
                      void* dres_bf16, float* dw, float* partials, int rows, int d, int accumulate, void* stream);
/* No counterpart in the reference: an addition for callers that cannot allocate device memory
 * (a plugin interface that passes only the op's tensors, or a process whose device memory is held
 * by another allocator).  Same arguments and results as sj_rmsnorm_bwd without `partials`: the
 * partials live in a fixed 4 MiB array inside the library's device image, so the call allocates
 * nothing.  Limit: sj_rmsnorm_workspace(rows, d) <= sj_rmsnorm_noalloc_limit() floats, else
 * SJ_ERR_CAPACITY.  Every call looks the array's device address up in the current context; the
 * first call in a context may load the library's device code there: make it before any stream
 * capture.  Calls that overlap in time on
 * one device share the array and race: serialise them. */
size_t sj_rmsnorm_noalloc_limit(void);
int sj_rmsnorm_bwd_noalloc(const void* x, int x_dtype, const float* w, const float* inv_rms, const float* dz,
                           float* dres, void* dres_bf16, float* dw, int rows, int d, void* stream);
/* Engine::embedding (lib.rs:650-665; kernels.py:41-45): y[i,:] = w[ids[i],:]; w bf16, y bf16 or f32
 * (y_dtype; f32 starts an f32 residual stream).  Ids outside [0, vocab) are an error recorded in the
 * device error word (row left zero). */
int sj_embedding_fwd(const void* w, const int32_t* ids, void* y, int y_dtype, int n, int d, int vocab, void* stream);
/* Engine::embedding_backward (lib.rs:666-687; kernels.py:47-52): dw[ids[i],:] += dy[i,:] (f32). */
int sj_embedding_bwd(const float* dy, const int32_t* ids, float* dw, int n, int d, int vocab, void* stream);
/* Engine::rope (lib.rs:734-758; kernels.py:103-113) standalone: x,y [rows, heads*hd] bf16. */
int sj_rope(const void* x, void* y, int rows, int heads, int head_dim, int t, int offset, float theta, int inverse,
            void* stream);
/* Engine::swiglu_backward (lib.rs:711-733; kernels.py:95-101): gu [rows,2f] bf16 interleaved by 16
 * columns (as written by SJ_EPI_SWIGLU), dh [rows,f] bf16 -> dgu [rows,2f] bf16 (same interleave). */
int sj_swiglu_bwd(const void* gu, const void* dh, void* dgu, int rows, int f, void* stream);
/* The same over the first *live_rows (device int32, at most rows) rows of a packed MoE buffer whose
 * used extent is known only on the device (group_rows[groups] of sj_ep_route_pack). */
int sj_swiglu_bwd_live(const void* gu, const void* dh, void* dgu, int rows, int f, const int32_t* live_rows,
                       void* stream);
/* Engine::patch_pool (crates/sejong-gpu/src/hierarchy_ops.rs:149-205; hierarchy.py:107-131). */
int sj_patch_pool_fwd(const void* x, void* y, int batch, int t, int d, int patch, void* stream);
/* dx[b,t,:] += dy[b, t/P, :] / count  (f32 accumulate) */
int sj_patch_pool_bwd(const float* dy, float* dx, int batch, int t, int d, int patch, void* stream);
/* Engine::patch_broadcast (hierarchy_ops.rs:207-278; hierarchy.py:134-172) fused with the tape add
 * (architecture.rs:386-387):  y[b,t,:] (+)= t/P >= 1 ? z[b, t/P - 1, :] : bos[:]  (z, bos bf16; y bf16 or
 * f32 per y_dtype; accumulate when add != 0). */
int sj_patch_broadcast_fwd(const void* z, const void* bos, void* y, int y_dtype, int add, int batch, int t, int d,
                           int patch, void* stream);
/* dz[b,p,:] = sum of dy over the bytes of patch p+1 ; dbos = sum of dy over the first patch of every row.
 * dy f32; dz [batch*patches, d] and dbos [d] bf16 (both feed the global_to_decoder backward GEMMs). */
int sj_patch_broadcast_bwd(const float* dy, void* dz, void* dbos, int batch, int t, int d, int patch, void* stream);
/* Engine::cross_entropy + cross_entropy_backward + loss_summary (lib.rs:881-912, 524-543;
 * kernels.py:176-191, 254-262), fused: loss[r] = lse(logits[r]) - logits[r,target];
 * dlogits[r,:] = (softmax - onehot) * seed (bf16, columns vocab..ld_d zeroed);
 * loss_sum[0] (f64) = sum_r loss[r] * weight. logits f32 [rows, ld] (first `vocab` columns used). */
int sj_cross_entropy(const float* logits, int ld, const int32_t* targets, int rows, int vocab, float seed,
                     float* loss_rows, void* dlogits, int ld_d, double* loss_sum, double weight, void* stream);
/* cast between f32 / bf16 / f64 (Engine::cast, lib.rs:554-571) */
int sj_cast(const void* x, int x_dtype, void* y, int y_dtype, size_t n, void* stream);
/* y = x + alpha*z (Engine::add / add_into, lib.rs:572-593; kernels.py:16-21), f32 or bf16 */
int sj_add(const void* x, const void* z, void* y, size_t n, float alpha, int dtype, void* stream);

/* ------------------------------------------------------------------ attention (GQA, causal, window) */
/* Engine::attention_grouped (crates/sejong-gpu/src/hierarchy_ops.rs:10-72; hierarchy.py:7-39).
 * q [batch*t, hq*64], k/v [batch*t, hk*64] (row strides ldq/ldk/ldv), bf16;  o bf16 (ldo);
 * lse f32 [batch*t*hq] natural log, index row*hq + head.  window 0 = full causal. */
int sj_attn_gqa_fwd(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv, void* o, int ldo,
                    float* lse, int batch, int t, int hq, int hk, int head_dim, int window, void* stream);
/* Engine::attention_grouped_backward (hierarchy_ops.rs:74-147; hierarchy.py:42-104).
 * do bf16 (lddo); dq/dk/dv bf16 with their own strides; when rope_table (an sj_rope_table of t
 * positions) is given, or else rope_theta > 0, the inverse rotation of Engine::rope(.., inverse=true)
 * (graph.rs:879-882) is applied to dq and dk before the store.  All operands 16-byte aligned, row
 * strides multiples of 8 elements.  `workspace` is 16-byte aligned f32 scratch of
 * sj_attn_workspace(batch, t, hq, hk) elements: the f32 dQ accumulator [batch*t, hq*64], then Delta
 * and LSE*log2(e) laid out [hq][batch][t rounded up to 128], then, when hq > hk and the
 * batch * hk * ceil(t/128) work items are fewer than 148 (each then split by query head), the f32
 * dK / dV accumulator [batch*t, hk, 128].  Returns 0 for a shape with hq not a multiple of hk. */
size_t sj_attn_workspace(int batch, int t, int hq, int hk);
int sj_attn_gqa_bwd(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv, const void* o, int ldo,
                    const float* lse, const void* dout, int lddo, void* dq, int lddq, void* dk, int lddk, void* dv,
                    int lddv, float* workspace, int batch, int t, int hq, int hk, int head_dim, int window,
                    float rope_theta, const float* rope_table, void* stream);

/* Grouped GEMM over device-side groups (the experts of an MoE layer in one launch, without reading
 * the expert counts back to the host as Engine::expert_routes does, hierarchy_ops.rs:332-378).
 * group_rows: device int32 [groups + 1] row offsets, each a multiple of 128 (sj_route_pack).
 *   group_mode 1 (grouped rows): A [m, k] and C [m, n] are packed by group, m the row capacity (a
 *     multiple of 128); rows [group_rows[g], group_rows[g+1]) use group g's B, stored as the g-th
 *     block of b_group_rows rows of B (b_group_rows = k for B [k, n], n for b_trans B [n, k]).
 *     Epilogue SJ_EPI_STORE or SJ_EPI_SWIGLU.
 *   group_mode 2 (grouped reduction): C_g [m, n] += A_g^T B_g over the packed rows [group_rows[g],
 *     group_rows[g+1]) of A (a_trans: stored [k, m]) and B ([k, n]); C_g is the g-th block of
 *     c_group_rows rows of C (f32).  Epilogue SJ_EPI_ACCUM.
 * groups <= 63. */
int sj_gemm_grouped(const void* a, int lda, int a_trans, const void* b, int ldb, int b_trans, void* c, int ldc,
                    int c_dtype, int m, int n, int k, int epilogue, void* aux, int ld_aux, int groups,
                    const int32_t* group_rows, int group_mode, int b_group_rows, int c_group_rows, void* stream);

/* ------------------------------------------------------------------ mixture of experts */
/* The MoE FFN of a block (crates/sejong-model/src/architecture.rs:229-241): router GEMM, then
 *   sj_route_topk      Engine::route_topk (hierarchy_ops.rs:280-295; hierarchy.py:174-190): softmax over
 *                      the experts; top-k by logit, lowest index on ties; gate = softmax probability.
 *                      logits f32 [rows, ld]; ids int32 [rows, k]; gates f32 [rows, k].  experts <= 32.
 *   sj_route_pack      Engine::expert_routes (hierarchy_ops.rs:332-378; hierarchy.py:211-225) on the
 *                      device: group_rows [experts + 1] (each expert's packed rows padded to 128),
 *                      pos [rows*k] (packed row of each routed slot row*k + j), row_slot [cap] (slot of
 *                      each packed row, -1 for padding); inside an expert, slots in increasing order.
 *                      cap >= sj_moe_capacity(rows, k, experts).
 *   sj_moe_dispatch    A[r] = z[row_slot[r] / k] (bf16, 0 for padding): the per-expert gather.
 *   sj_moe_combine     y = x + sum_j gates[:, j] out[pos[:, j]] (Engine::expert_combine,
 *                      hierarchy_ops.rs:380-419, and the block's residual add); out bf16 [cap, d], x, y f32.
 * and the backward: sj_moe_combine_bwd (Engine::expert_combine_backward, hierarchy_ops.rs:421-454:
 * d_out[r] = gate * dy[t], d_gates[slot] = <out[r], dy[t]>), sj_route_topk_bwd (route_topk_backward,
 * hierarchy_ops.rs:297-330: dlogits = p (dy_selected - sum gate dy), bf16 [rows, ldd]) and
 * sj_moe_dispatch_bwd (dz[t] = sum_j dA[pos[t, j]], f32). */
int sj_moe_capacity(int rows, int k, int experts);
int sj_route_topk(const float* logits, int ld, int rows, int experts, int k, int32_t* ids, float* gates, void* stream);
int sj_route_pack(const int32_t* ids, int rows, int experts, int k, int32_t* group_rows, int32_t* pos,
                  int32_t* row_slot, int cap, void* stream);
/* No counterpart in the reference (its experts take every routed row and it has no auxiliary loss);
 * opt-in additions for the MoE benchmark configuration (capacity factor 1.25, loss weight 0.01).
 * Expert capacity: each expert keeps at most `capacity` of the slots in
 * ids [rows, k] (every row's first choice before any second choice, rows in order within a choice);
 * dropped slots get id -1 in place, which the pack, combine and backwards skip.  Call between
 * sj_route_topk and sj_route_pack / sj_ep_route_pack. */
int sj_route_capacity(int32_t* ids, int rows, int k, int experts, int capacity, void* stream);
/* Load-balancing loss aux = weight * E * sum_e f_e P_e (f_e: share of the top-k choices, before any
 * capacity drop, that picked e; P_e: mean router probability of e), recomputed from the f32 router
 * logits (two kernels; no atomics): loss_sum[0] += loss_seed * aux, and dlogits (bf16 [rows, ldd], the router gradient that
 * sj_route_topk_bwd wrote) += grad_scale * d aux / d logits. */
int sj_moe_aux(const float* logits, int ld, int rows, int experts, int k, float weight, double loss_seed,
               double* loss_sum, void* dlogits, int ldd, float grad_scale, float* workspace, void* stream);
/* Floats of sj_moe_aux's workspace (per 256 rows, the choice counts and probability sums). */
size_t sj_moe_aux_workspace(int rows, int experts);
int sj_moe_dispatch(const void* z, int ldz, const int32_t* row_slot, int cap, int k, int d, void* a, void* stream);
int sj_moe_combine(const void* out, const int32_t* pos, const float* gates, const float* x, float* y, int rows, int k,
                   int d, void* stream);
int sj_moe_combine_bwd(const void* out, const int32_t* row_slot, const float* gates, const float* dy, void* d_out,
                       float* d_gates, int cap, int k, int d, void* stream);
int sj_route_topk_bwd(const float* logits, int ld, const int32_t* ids, const float* gates, const float* d_gates,
                      void* dlogits, int ldd, int rows, int experts, int k, void* stream);
int sj_moe_dispatch_bwd(const float* da, const int32_t* pos, float* dz, int ldz, int rows, int k, int d, void* stream);

/* ------------------------------------------------------------------ f32 step (BASELINE C1) */
/* The step in f32 arithmetic (the reference's DType::F32 precision): every operand, activation and
 * gradient f32, f32 FMA accumulation on the CUDA cores.
 *   sj_sgemm           C [m, n] = op(A) op(B) (f32) with the epilogues of sj_gemm: SJ_EPI_STORE, ACCUM
 *                      (C +=), RESIDUAL (C = AB + aux), ROPE (pairs of the first rope_cols columns rotated by
 *                      rope_table [rope_t, 64] at position row % rope_t), SWIGLU (C = the interleaved
 *                      gate|up blocks of 16, aux [m, n/2] = silu(g) u; no rounding of g, u).
 *   sj_rmsnorm_fwd_f32 sj_rmsnorm_fwd with an f32 x and y.  The backward is sj_rmsnorm_bwd (f32 x,
 *                      dres_bf16 = NULL).
 *   sj_cross_entropy_f32  sj_cross_entropy with f32 dlogits.
 *   sj_swiglu_bwd_f32  sj_swiglu_bwd on f32 gu, dh, dgu.
 *   sj_attn_f32_fwd / _bwd  sj_attn_gqa_fwd / _bwd on f32 q, k, v, o, dO, dq, dk, dv; the backward takes
 *                      sj_attn_f32_workspace(batch, t, hq) floats and the RoPE table (inverse rotation of
 *                      dq and dk). */
int sj_sgemm(const float* a, int lda, int a_trans, const float* b, int ldb, int b_trans, float* c, int ldc, int m,
             int n, int k, int epilogue, float* aux, int ld_aux, const float* rope_table, int rope_cols, int rope_t,
             void* stream);
int sj_rmsnorm_fwd_f32(const float* x, const float* w, float* y, float* inv_rms, int rows, int d, float eps,
                       void* stream);
/* sj_embedding_fwd with an f32 table and output (y[i] = w[ids[i]], row copies). */
int sj_embedding_fwd_f32(const float* w, const int32_t* ids, float* y, int n, int d, int vocab, void* stream);
int sj_cross_entropy_f32(const float* logits, int ld, const int32_t* targets, int rows, int vocab, float seed,
                         float* loss_rows, float* dlogits, int ld_d, double* loss_sum, double weight, void* stream);
int sj_swiglu_bwd_f32(const float* gu, const float* dh, float* dgu, int rows, int f, void* stream);
int sj_attn_f32_fwd(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* o, int ldo,
                    float* lse, int batch, int t, int hq, int hk, int head_dim, int window, void* stream);
size_t sj_attn_f32_workspace(int batch, int t, int hq);
int sj_attn_f32_bwd(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, const float* o, int ldo,
                    const float* lse, const float* dout, int lddo, float* dq, int lddq, float* dk, int lddk, float* dv,
                    int lddv, float* workspace, int batch, int t, int hq, int hk, int head_dim, int window,
                    const float* rope_table, void* stream);

/* ------------------------------------------------------------------ KV-cached inference */
/* cached_blocks (crates/sejong-model/src/architecture.rs:474-533).
 *   sj_attn_cached  Engine::attention_grouped with OFFSET: q bf16 [rows, ldq] holds the chunk's RoPE'd
 *                   queries at positions offset .. offset + rows - 1; k_cache / v_cache bf16 [offset +
 *                   rows, ld] hold every position up to the chunk's last (the chunk's own rows
 *                   appended first); causal with an optional window; o bf16 [rows, ldo].  Up to 16384
 *                   visible keys per row.
 *   sj_copy_rows    rows x row_bytes copy between strided buffers (the K/V append), 16-byte multiples. */
int sj_attn_cached(const void* q, int ldq, const void* k_cache, int ldk, const void* v_cache, int ldv, void* o,
                   int ldo, int rows, int offset, int hq, int hk, int head_dim, int window, void* stream);
int sj_copy_rows(const void* src, size_t ld_src_bytes, void* dst, size_t ld_dst_bytes, int rows, size_t row_bytes,
                 void* stream);
/* The patch state of hierarchical decoding (architecture.rs:749-770): acc f32 [d] = (reset ? 0 : acc) +
 * the sum of rows bf16 x [rows, ldx]; y bf16 [n] = x f32 * alpha. */
int sj_rows_sum_f32(const void* x, int ldx, int rows, int d, float* acc, int reset, void* stream);
int sj_scale_to_bf16(const float* x, int n, float alpha, void* y, void* stream);

/* ------------------------------------------------------------------ NativeValue head */
/* The categorical value head of NativeValue::forward_batch (crates/sejong-model/src/native/value.rs:
 * 111-160) with its loss (Engine::cross_entropy, lib.rs:524-543) and backward.  hidden bf16 [rows,
 * ldh] is the body's final-norm output; sel int32 [batch] the SEP row of each request; W f32 [d, nv]
 * (native_value), bias f32 [nv] (native_bias); labels int32 [batch].
 *   sj_value_head_fwd: logits f32 [batch, nv] = f32(hidden[sel]) W + bias; dlogits f32 [batch, nv] =
 *     (softmax - onehot(label)) * seed (optional); loss_sum += sum_b loss_b * weight (optional).
 *     A row or label out of range records SJ_DEV_BAD_INDEX and skips that request.  d <= 4096.
 *   sj_value_head_bwd: dW += f32(hidden[sel])^T dlogits, dbias += sum_b dlogits, dh[sel[b], :] =
 *     dlogits[b] W^T (f32 [rows, ldd]; only the selected rows are written). */
int sj_value_head_fwd(const void* hidden, int ldh, int rows, const int32_t* sel, int batch, int d, const float* w,
                      const float* bias, int nv, const int32_t* labels, float seed, float* logits, float* dlogits,
                      double* loss_sum, double weight, void* stream);
int sj_value_head_bwd(const void* hidden, int ldh, int rows, const int32_t* sel, int batch, int d, const float* w,
                      const float* dlogits, int nv, float* dw, float* dbias, float* dh, int ldd, void* stream);

/* ------------------------------------------------------------------ expert parallelism */
/* The MoE FFN with the experts sharded over the ranks of the data-parallel group (experts / world
 * experts per rank, rank r owning experts [r*local, (r+1)*local)).  No counterpart in the reference,
 * which runs every expert on one device (hierarchy_ops.rs:280-454); a step over `world` ranks
 * computes what sj_route_pack / sj_moe_* compute on one device for the ranks' rows concatenated in
 * rank order (same packed order inside each expert).
 *
 * Transport: a symmetric heap -- one device allocation of the same size on every rank, opened in
 * every peer with CUDA IPC (plain NVLink loads and stores, no multicast).  `peers` is a host array
 * of `world` heap base addresses as mapped in this process (peers[rank] = this rank's own heap);
 * buffers shared between ranks are given as byte offsets into the heap (16-byte aligned), the same
 * on every rank.  Cross-rank ordering uses a flag array (uint32 [world], heap offset flags_off) and
 * a per-rank device epoch counter (uint32, zero at start) that every barrier advances; every rank
 * must issue the same sequence of sj_ep_route_pack / sj_ep_barrier calls.  A wait that exceeds
 * timeout_ms records SJ_DEV_EP_WAIT in the device error word and returns.
 *
 *   sj_ipc_alloc / sj_ipc_free      a zero-filled device allocation for the heap.
 *   sj_ipc_handle / sj_ipc_open / sj_ipc_close   export a heap (SJ_IPC_HANDLE_BYTES bytes) and map a
 *                                   peer's heap into this process.
 *   sj_ep_receive_capacity          packed rows a rank must be able to receive (every routed slot of
 *                                   every rank on its experts, each segment padded to 128).
 *   sj_ep_route_pack   counts (int32 [world][experts] at counts_off, one matrix per MoE layer)
 *                      published to every rank, barrier, then group_rows [2*local + 1] (this rank's
 *                      segment starts and end, then the end of the valid rows of each segment) and
 *                      pos [rows*k] (the packed row, at the owner of ids[slot], of each of this rank's
 *                      slots).  One CTA.
 *   sj_ep_dispatch     A_owner[pos[s]] = z[s / k] pushed to the owners (A bf16 [cap, d] at a_off),
 *                      and this rank's padding rows of A zeroed.
 *   sj_ep_barrier      every earlier write of every rank visible to every rank.
 *   sj_ep_combine      y = x + sum_j gates[:, j] out_owner[pos[:, j]] (out bf16 [cap, d] at out_off),
 *                      pulled from the owners.
 *   sj_ep_combine_bwd  d_out_owner[pos[s]] = gate[s] dy[s / k] pushed (bf16, at d_out_off),
 *                      d_gates[s] = <out_owner[pos[s]], dy[s / k]> pulled, padding rows of this
 *                      rank's d_out zeroed.
 *   sj_ep_dispatch_bwd dz[t] = sum_j dA_owner[pos[t, j]] (dA f32 [cap, d] at da_off), pulled. */
#define SJ_IPC_HANDLE_BYTES 64
int sj_ipc_alloc(size_t bytes, void** ptr);
int sj_ipc_free(void* ptr);
int sj_ipc_handle(const void* ptr, void* handle);
int sj_ipc_open(const void* handle, void** ptr);
int sj_ipc_close(void* ptr);
int sj_ep_receive_capacity(int rows, int k, int experts, int world);
int sj_ep_route_pack(const int32_t* ids, int rows, int experts, int k, int rank, int world, const void* const* peers,
                     size_t counts_off, size_t flags_off, uint32_t* epoch, int32_t* group_rows, int32_t* pos, int cap,
                     int timeout_ms, void* stream);
int sj_ep_dispatch(const void* z, int ldz, const int32_t* ids, const int32_t* pos, int rows, int k, int d, int experts,
                   int rank, int world, const void* const* peers, size_t a_off, const int32_t* group_rows,
                   void* stream);
int sj_ep_barrier(int rank, int world, const void* const* peers, size_t flags_off, uint32_t* epoch, int timeout_ms,
                  void* stream);
int sj_ep_combine(const void* const* peers, int world, size_t out_off, const int32_t* ids, const int32_t* pos,
                  const float* gates, const float* x, float* y, int rows, int k, int d, int experts, void* stream);
int sj_ep_combine_bwd(const void* const* peers, int rank, int world, size_t out_off, size_t d_out_off,
                      const int32_t* ids, const int32_t* pos, const float* gates, const float* dy, float* d_gates,
                      const int32_t* group_rows, int rows, int k, int d, int experts, void* stream);
int sj_ep_dispatch_bwd(const void* const* peers, int world, size_t da_off, const int32_t* ids, const int32_t* pos,
                       float* dz, int ldz, int rows, int k, int d, int experts, void* stream);

/* ------------------------------------------------------------------ BERT encoder (MiniLM) forward */
/* BertEncoder::hidden (crates/sejong-model/src/native/bert.rs:360-411) on a batch of sequences packed
 * row after row: sequence s owns rows [cu_seqlens[s], cu_seqlens[s+1]), so nothing is padded and
 * each sequence attends to its own keys only, as the reference's one-sequence-at-a-time loop does.
 * Position of a row = its index inside its sequence; token types are 0. */
/* x = LayerNorm(word[id] + position[pos] + type0) (bert.rs:364-385, common.py:6-14).  Tables f32
 * row-major [vocab,d], [max_position,d], type0 [d]; x f32 [rows,d] and optional x_bf16 [rows,d].
 * d a multiple of 128 up to 1024.  An id or position out of range is read as row 0 and raises
 * SJ_DEV_BAD_INDEX in the device error word. */
int sj_bert_embed(const int32_t* ids, const int32_t* cu_seqlens, int batch, const float* word, int vocab,
                  const float* position, int max_position, const float* type0, const float* ln_w, const float* ln_b,
                  float eps, float* x, void* x_bf16, int rows, int d, void* stream);
/* Engine::layer_norm (crates/sejong-gpu/src/common_ops.rs:4-17; common.py:6-14): per row mean,
 * centred variance, y = (x - mean) / sqrt(var + eps) * w + b.  x, y f32 [rows,d]; y_bf16 optional. */
int sj_layernorm(const float* x, const float* w, const float* b, float eps, float* y, void* y_bf16, int rows, int d,
                 void* stream);
/* Engine::attention_mode(.., causal = false) (crates/sejong-gpu/src/lib.rs:771-815; kernels.py:115-136)
 * per packed sequence: qkv bf16 rows [q | k | v] (heads*head_dim columns each, row stride ldqkv),
 * out bf16 [rows, heads*head_dim] (ldo).  head_dim 32, sequences of at most 128 rows. */
int sj_bert_attention(const void* qkv, int ldqkv, const int32_t* cu_seqlens, int batch, int max_len, int heads,
                      int head_dim, void* out, int ldo, void* stream);

/* ------------------------------------------------------------------ optimizer */
/* FP64 sum of squares of a flat f32 buffer into `partials` (f64, sj_sumsq_partials(n) entries):
 * Engine::gradient_norm (crates/sejong-gpu/src/lib.rs:494-523; kernels.py:265-287). */
int sj_sumsq_partials(size_t n);
int sj_grad_sumsq(const float* g, size_t n, double* partials, void* stream);
/* Device-side step bookkeeping for Adam::update (crates/sejong-train/src/lib.rs:199-238) and
 * TrainConfig::lr (crates/sejong-core/src/lib.rs:422-433): reduces `partials` to the global norm,
 * derives clip scale = (clip_enabled && norm > clip ? clip/norm : 1)/loss_scale, increments the step
 * counter in state[0] and writes hyper = {lr(step-1), 1/(1-b1^step), 1/(1-b2^step), scale, norm}.
 * `state` (f64[2]: step, last norm) and `hyper` (f32[8]) are device buffers so the step needs no
 * host round trip and can be captured in a CUDA graph. */
int sj_optim_prepare(const double* partials, int n_partials, double* state, float* hyper, float learning_rate,
                     float min_learning_rate, int warmup_steps, int total_steps, float beta1, float beta2,
                     float clip_norm, int clip_enabled, float loss_scale, void* stream);
/* Multi-tensor AdamW over one flat parameter buffer (kernels.py:193-202 per element; the reference
 * launches it once per tensor, lib.rs:925-957).  Elements [0, n_decay) get decoupled weight decay
 * (rank>1 tensors), the rest none.  w/g/m/v f32; w_bf16 (optional) receives the bf16 copy used by the
 * next forward (Model::bind's per-step cast, crates/sejong-model/src/lib.rs:206-219). */
int sj_adamw(float* w, const float* g, float* m, float* v, void* w_bf16, size_t n, size_t n_decay,
             const float* hyper, float beta1, float beta2, float eps, float weight_decay, void* stream);
/* Plain SGD over a flat buffer (crates/sejong-train/src/control_variate.rs:775-799):
 * w = w*(1 - lr*decay) - lr*scale*g with decay on [0, n_decay). */
int sj_sgd(float* w, const float* g, void* w_bf16, size_t n, size_t n_decay, const float* hyper, float weight_decay,
           void* stream);

/* ------------------------------------------------------------------ parameter VJP (low-rank + selected rows) */
/* The index draw of the parameter_indices kernel (python/sejong_kernels/ops/parameter.py:25-62) as
 * launched by ParameterVjp::prepare (crates/sejong-gpu/src/parameter_vjp.rs:186-214): a SplitMix64
 * generator seeded with one next_u64 of `rng_state` (device memory, advanced in place) draws a
 * partial Fisher-Yates of r of the b donor columns, then of s of the nb feature blocks of `group`
 * rows.  columns [r]; rows [s*group] (feature index, -1 past a); row_map [a] (position in rows or -1).
 * The reference kernel's permutation scratch lives in shared memory (b + nb + s <= 12288).  Zero
 * sizes skip the corresponding draw, as the reference's do. */
int sj_param_indices(uint64_t* rng_state, int a, int b, int nb, int s, int r, int group, int32_t* columns,
                     int32_t* rows, int32_t* row_map, void* stream);
/* The same draw on the host from an explicit seed (the reference kernel's own inputs). */
int sj_param_indices_host(uint64_t seed, int a, int b, int nb, int s, int r, int group, int32_t* columns,
                          int32_t* rows, int32_t* row_map);
/* Orthonormal basis q [n, r] f32 of the selected donor columns Y[:, columns] with Y = x w (x bf16
 * [n, a], row stride ldx; w bf16 with row stride ldw, pointing at the donor's first column;
 * interleave > 0 selects the second half of a weight interleaved in blocks of `interleave`
 * columns): the CGS2 with small-norm cutoff `eps` of parameter.py:65-129 / parameter_vjp.rs:216-258.
 * workspace: sj_param_basis_workspace(n, a, r) bytes, 16-byte aligned.  r <= 32, a % 8 == 0. */
size_t sj_param_basis_workspace(int n, int a, int r);
int sj_param_basis(const void* x, int ldx, int n, int a, const void* w, int ldw, int interleave, const int32_t* columns,
                   int r, float eps, float* q, void* workspace, void* stream);
/* The prepare kernel (parameter.py:131-191, parameter_vjp.rs:260-290): left = x^T q [a, r] f32 and
 * E [(r + k), n] bf16 = [q^T ; (x - q left^T)[:, rows]^T * inverse] (zero rows where rows[i] < 0),
 * inverse = NB/S in f32.  E is the A operand of the coefficient GEMM (right; tail) = E dY. */
int sj_param_prepare(const void* x, int ldx, int n, int a, const float* q, int r, const int32_t* rows, int k,
                     float inverse, float* left, void* e, void* stream);
/* The factored gradient (parameter.py:204-244): g[i, j] (+)= sum_k left[i, k] coeff[k, j] +
 * coeff[r + row_map[i], j] (when row_map[i] >= 0), j < b; coeff rows [0, r) = right, [r, r+k) = tail. */
int sj_param_materialize(const float* left, const float* coeff, int ldc, const int32_t* row_map, int a, int b, int r,
                         float* g, int ldg, int accumulate, void* stream);

/* ---- control-variate SGD (crates/sejong-train/src/control_variate.rs:236-877) ---------------- */
/* SgdState::new / refresh_bases' Engine::orthonormalize_columns (hierarchy_ops.rs:592-615; kernel
 * hierarchy_orthogonal_column, hierarchy.py:346-397): q [rows, cols] f32 = the columns of x
 * orthonormalised in order by two passes of Gram-Schmidt each (a column left with a squared norm
 * below 1e-20 restarts from the unit vector at the row the earlier columns occupy least); gram (or
 * null) [cols, cols] = q^T q.  One CTA; x and q distinct; 0 < cols <= rows. */
int sj_cv_orthonormalize(const float* x, float* q, float* gram, int rows, int cols, void* stream);
/* Engine::transport_coefficients (hierarchy_ops.rs:512-553, hierarchy_coefficient_transport): for
 * each of `features` rows of h (row stride ld floats), the rank x rank coefficient at column col0 ->
 * y (same place) = left^T C right.  rank <= 55; h and y distinct. */
int sj_cv_transport(const float* h, int ld, int col0, const float* left, const float* right, float* y, int features,
                    int rank, void* stream);
/* augmented_feature (control_variate.rs:375-387): out [3 width + 1] = [row means of the encoded rows
 * (bf16 or f32, row stride ld), row means of the f32 embedding rows of `labels` (row stride emb_ld,
 * vocab rows), row means of their product, 1].  A label outside [0, vocab) records
 * SJ_DEV_BAD_INDEX and counts as a zero row. */
int sj_cv_feature(const void* encoded, int dtype, int ld, const float* embedding, int emb_ld, const int32_t* labels,
                  int rows, int width, int vocab, float* out, void* stream);
/* The gradient norm's correction terms (control_variate.rs:365-373,699-706), FP64 per block j:
 * out[j] = scale * (<X_j, GU_j X_j GV_j> + t_weight <T_j, X_j>), X, T, GU, GV [blocks][rank][rank]
 * f32 (t may be null).  Written into the optimizer's FP64 partials they enter the clipped norm. */
int sj_cv_block_terms(const float* gram_u, const float* gram_v, const float* x, const float* t, double* out,
                      int blocks, int rank, float t_weight, double scale, void* stream);
/* The deferred coefficient update (control_variate.rs:796-806): a = a (1 - lr wd) - lr clip delta
 * with lr = hyper[0] and clip = hyper[3] * loss_scale (the sj_optim_prepare output). */
int sj_cv_deferred_update(float* a, const float* delta, const float* hyper, float weight_decay, float loss_scale,
                          size_t n, void* stream);
/* The bound weight of a corrected matrix (Model::bind_with_corrections, crates/sejong-model/src/
 * lib.rs:206-250, with graph.rs:244-271's x W + ((x U) A) V^T folded into the weight):
 * wb (bf16) = master + correction, n elements. */
int sj_cv_bind(const float* master, const float* correction, void* wb, size_t n, void* stream);
/* out [out_rows, cols] = 0 except out[map[i], :] = v[i, :], i < rows (a member matrix's basis rows
 * placed at its columns of a fused weight); sj_cv_gather_rows the inverse, out[i, :] = alpha *
 * v[map[i], :].  An index outside the target records SJ_DEV_BAD_INDEX. */
int sj_cv_scatter_rows(const float* v, int rows, int cols, const int32_t* map, float* out, int out_rows,
                       void* stream);
int sj_cv_gather_rows(const float* v, int v_rows, int cols, const int32_t* map, float* out, int rows, float alpha,
                      void* stream);
/* The predictor gradient's outer product (control_variate.rs:718-725): out [f, n] += alpha x[i]
 * (p[j] - beta t[j]). */
int sj_cv_outer(const float* x, int f, const float* p, const float* t, float beta, int n, float alpha, float* out,
                void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SEJONG_B200_H */
