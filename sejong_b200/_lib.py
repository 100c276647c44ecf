"""ctypes binding of libsejong_b200.so (declarations in include/sejong.h).

The library is the only compute path: importing this module on a machine
without the built library raises, and there is no CPU fallback.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsejong_b200.so")

c_int, c_float, c_double, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_size_t, ctypes.c_void_p
c_u64, c_u64p = ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)

# name -> (restype, argtypes)
SIGNATURES = {
    "sj_version": (c_int, []),
    "sj_last_error": (ctypes.c_char_p, []),
    "sj_device_init": (c_int, [c_int]),
    "sj_mem_info": (c_int, [ctypes.POINTER(c_size_t), ctypes.POINTER(c_size_t)]),
    "sj_device_error": (c_int, [ctypes.POINTER(c_int), c_int, c_void_p]),
    "sj_zero": (c_int, [c_void_p, c_size_t, c_void_p]),
    "sj_rng_next_u64": (c_u64, [c_u64p]),
    "sj_rng_index": (c_u64, [c_u64p, c_u64]),
    "sj_rng_normal_fill": (c_int, [c_u64p, c_void_p, c_size_t, c_float]),
    "sj_zipf_bytes": (c_int, [c_u64, c_double, c_void_p, c_size_t]),
    "sj_corpus_batch": (c_int, [c_void_p, c_size_t, c_u64p, c_int, c_int, c_void_p, c_void_p]),
    "sj_blake3": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "sj_gemm_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_gemm": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int,
                        c_int, c_float, c_void_p, c_int, c_int, c_int, c_float, c_int, c_void_p]),
    "sj_gemm_grouped": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p]),
    "sj_moe_capacity": (c_int, [c_int, c_int, c_int]),
    "sj_route_topk": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "sj_route_pack": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "sj_route_capacity": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_moe_aux": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_float, c_double, c_void_p, c_void_p, c_int, c_float,
                           c_void_p, c_void_p]),
    "sj_moe_aux_workspace": (c_size_t, [c_int, c_int]),
    "sj_moe_dispatch": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "sj_moe_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "sj_moe_combine_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                   c_void_p]),
    "sj_route_topk_bwd": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                  c_void_p]),
    "sj_moe_dispatch_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_sgemm": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int,
                         c_void_p, c_int, c_void_p, c_int, c_int, c_void_p]),
    "sj_embedding_fwd_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "sj_rmsnorm_fwd_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "sj_cross_entropy_f32": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_int,
                                     c_void_p, c_double, c_void_p]),
    "sj_swiglu_bwd_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_attn_f32_fwd": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_attn_f32_workspace": (c_size_t, [c_int, c_int, c_int]),
    "sj_attn_f32_bwd": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                c_int, c_int, c_int, c_void_p, c_void_p]),
    "sj_attn_cached": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                               c_int, c_int, c_int, c_void_p]),
    "sj_copy_rows": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_int, c_size_t, c_void_p]),
    "sj_rows_sum_f32": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p]),
    "sj_scale_to_bf16": (c_int, [c_void_p, c_int, c_float, c_void_p, c_void_p]),
    "sj_value_head_fwd": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p,
                                  c_float, c_void_p, c_void_p, c_void_p, c_double, c_void_p]),
    "sj_value_head_bwd": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p,
                                  c_void_p, c_void_p, c_int, c_void_p]),
    "sj_ipc_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "sj_ipc_free": (c_int, [c_void_p]),
    "sj_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "sj_ipc_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "sj_ipc_close": (c_int, [c_void_p]),
    "sj_ep_receive_capacity": (c_int, [c_int, c_int, c_int, c_int]),
    "sj_ep_route_pack": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_size_t, c_void_p,
                                 c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_ep_dispatch": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                               c_size_t, c_void_p, c_void_p]),
    "sj_ep_barrier": (c_int, [c_int, c_int, c_void_p, c_size_t, c_void_p, c_int, c_void_p]),
    "sj_ep_combine": (c_int, [c_void_p, c_int, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                              c_int, c_int, c_void_p]),
    "sj_ep_combine_bwd": (c_int, [c_void_p, c_int, c_int, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_ep_dispatch_bwd": (c_int, [c_void_p, c_int, c_size_t, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                   c_int, c_void_p]),
    "sj_gemm_bias": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int,
                             c_int, c_int, c_float, c_void_p, c_void_p, c_int, c_void_p]),
    "sj_bert_embed": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                              c_void_p, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_bert_attention": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p]),
    "sj_rmsnorm_fwd": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "sj_rmsnorm_bwd": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_int, c_int, c_void_p]),
    "sj_rmsnorm_bwd_ex": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_int, c_int, c_int, c_void_p]),
    "sj_rmsnorm_workspace": (c_size_t, [c_int, c_int]),
    "sj_rmsnorm_noalloc_limit": (c_size_t, []),
    "sj_rmsnorm_bwd_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int, c_int, c_void_p]),
    "sj_embedding_fwd":(c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_embedding_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "sj_rope": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_void_p]),
    "sj_swiglu_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_swiglu_bwd_live": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "sj_patch_pool_fwd": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_patch_pool_bwd": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_patch_broadcast_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                       c_void_p]),
    "sj_patch_broadcast_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_cross_entropy": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_int, c_void_p,
                                 c_double, c_void_p]),
    "sj_cast": (c_int, [c_void_p, c_int, c_void_p, c_int, c_size_t, c_void_p]),
    "sj_add": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_float, c_int, c_void_p]),
    "sj_attn_gqa_fwd": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "sj_attn_gqa_bwd": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                c_int, c_int, c_int, c_float, c_void_p, c_void_p]),
    "sj_rope_table": (c_int, [c_void_p, c_int, c_int, c_int, c_float, c_void_p]),
    "sj_attn_workspace": (c_size_t, [c_int, c_int, c_int, c_int]),
    "sj_cv_orthonormalize": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_cv_transport": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "sj_cv_feature": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p,
                              c_void_p]),
    "sj_cv_block_terms": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_double,
                                  c_void_p]),
    "sj_cv_deferred_update": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_float, c_size_t, c_void_p]),
    "sj_cv_bind": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "sj_cv_scatter_rows": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    "sj_cv_gather_rows": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_float, c_void_p]),
    "sj_cv_outer": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_float, c_int, c_float, c_void_p, c_void_p]),
    "sj_sumsq_partials": (c_int, [c_size_t]),
    "sj_grad_sumsq": (c_int, [c_void_p, c_size_t, c_void_p, c_void_p]),
    "sj_optim_prepare": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_float, c_float, c_int, c_int, c_float, c_float,
                                 c_float, c_int, c_float, c_void_p]),
    "sj_adamw": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_float,
                         c_float, c_float, c_float, c_void_p]),
    "sj_sgd": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_float, c_void_p]),
    "sj_param_indices": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                 c_void_p]),
    "sj_param_indices_host": (c_int, [c_u64, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                      c_void_p]),
    "sj_param_basis_workspace": (c_size_t, [c_int, c_int, c_int]),
    "sj_param_basis": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_float,
                               c_void_p, c_void_p, c_void_p]),
    "sj_param_prepare": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_float, c_void_p,
                                 c_void_p, c_void_p]),
    "sj_param_materialize": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_int,
                                     c_int, c_void_p]),
}

# status codes (include/sejong.h)
SJ_OK, SJ_ERR_SHAPE, SJ_ERR_CAPACITY, SJ_ERR_CUDA, SJ_ERR_NCCL, SJ_ERR_TIMEOUT, SJ_ERR_ARGUMENT, SJ_ERR_UNSUPPORTED = range(8)
SJ_F32, SJ_F64, SJ_F16, SJ_I32, SJ_BF16 = range(5)
EPI_STORE, EPI_ACCUM, EPI_RESIDUAL, EPI_SWIGLU, EPI_ROPE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL = range(8)


class SejongError(RuntimeError):
    """A failing C-ABI call: `code` is the SJ_ERR_* status (mirrors sejong_core::Error)."""

    def __init__(self, code, message):
        super().__init__(f"[{code}] {message}")
        self.code = code


_lib = None


def load():
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m sejong_b200.build` "
                          "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name, *args):
    """Invoke a status-returning entry point and raise SejongError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != SJ_OK:
        raise SejongError(rc, f"{name}: {lib.sj_last_error().decode(errors='replace')}")
    return rc
