"""ctypes loader for libmsgl.so with the argument types of include/msgl_kernels.h."""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROOT = os.path.dirname(PKG)
# the in-tree build; MSGL_LIB names another build of the same library (e.g. a debug build)
LIB_PATH = os.environ.get("MSGL_LIB") or os.path.join(PKG, "libmsgl.so")
HEADERS = [os.path.join(ROOT, "include", f) for f in ("msgl_kernels.h", "msgl_engine.h")]

P, I, I64, F, SZ, U64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t, C.c_uint64

# entry point -> (restype, argtypes)
SIGNATURES = {
    "msgl_version": (C.c_char_p, []),
    "msgl_last_error": (C.c_char_p, []),
    "msgl_device_error": (I, [P, P, I, P]),
    "msgl_kernel_launches": (C.c_ulonglong, []),
    "msgl_launch_rmsnorm": (I, [P, P, P, I, I, F, I, P]),
    "msgl_launch_rope": (I, [P, P, P, P, I, I, I, I, I, P]),
    "msgl_launch_index_gather": (I, [P, P, P, I, I, I, I, P]),
    "msgl_launch_store_kv_page": (I, [P, P, P, P, P, I, I, I, I, I, P]),
    "msgl_add_rmsnorm": (I, [P, P, P, I, I, F, I, P]),
    "msgl_embed_rmsnorm": (I, [P, P, I, I, I, P, F, P, P, P]),
    "msgl_qknorm_rope_store_kv": (I, [P, P, P, P, I64, P, P, P, P, P, I, I, I, I, F, P]),
    "msgl_paged_attention_workspace_size": (SZ, [I, I, I, I, I]),
    "msgl_paged_attention_decode": (I, [P, P, P, I64, P, I, P, I, I, I, I, I, I, F, P, P, SZ, P]),
    "msgl_paged_attention_extend": (I, [P, P, P, I64, P, I, P, P, I, I, I, I, I, I, F, P, P]),
    "msgl_paged_attention_cascade_workspace_size": (SZ, [I, I, I, I, I, I]),
    "msgl_paged_attention_decode_cascade": (I, [P, P, P, I64, P, I, P, I, I, I, I, I, I, I, F, P, P, SZ, P]),
    "msgl_paged_attention_decode_noalloc": (I, [P, P, P, I64, P, I, P, I, I, I, I, I, I, F, P, P]),
    "msgl_gemm_workspace_size": (SZ, [I, I, I]),
    "msgl_gemm_bf16": (I, [P, P, P, I, I, I, I, P, SZ, P]),
    "msgl_pack_gate_up": (I, [P, P, I, I, P]),
    "msgl_gemm_gate_up_silu": (I, [P, P, P, I, I, I, P, SZ, P]),
    "msgl_gemm_partials_splits": (I, [I, I, I]),
    "msgl_decode_advance": (I, [P, P, P, P, P, I, P, P, P, I, I, P]),
    "msgl_sample": (I, [P, I, I, P, P, P, U64, U64, P, P]),
    "msgl_gemm_bf16_partials": (I, [P, P, P, I, I, I, I, P]),
    "msgl_add_partials_rmsnorm": (I, [P, I, P, P, P, I, I, F, P]),
    "msgl_qknorm_rope_store_kv_partials": (I, [P, I, P, P, P, I64, P, P, P, P, P, I, I, I, I, F, P]),
    "msgl_lm_head_argmax": (I, [P, P, I, I, I, P, P, P, SZ, P]),
    "msgl_argmax": (I, [P, I, I, I, P, P]),
    "msgl_fill_normal_bf16": (I, [P, I64, U64, U64, F, F, P]),
    "msgl_moe_route_topk": (I, [P, I, I, I, I, P, P, P]),
    "msgl_moe_route_topk_partials": (I, [P, I, I, I, I, I, P, P, P]),
    "msgl_moe_permute": (I, [P, I, I, I, P, P, P, P]),
    "msgl_grouped_gemm_workspace_size": (SZ, [I, I]),
    "msgl_grouped_gemm_bf16": (I, [P, P, P, P, I, I, I, I, P, SZ, P]),
    "msgl_grouped_gemm_bf16_reuse_tiles": (I, [P, P, P, P, I, I, I, I, P, SZ, P]),
    "msgl_grouped_gemm_gate_up_silu": (I, [P, P, P, P, I, I, I, I, P, SZ, P]),
    "msgl_moe_combine": (I, [P, P, P, I, I, I, P, P]),
    "msgl_moe_combine_add_rmsnorm": (I, [P, P, P, I, I, I, P, P, F, P, P]),
    "msgl_lm_head_argmax_partial": (I, [P, P, I, I, I, I, P, P, SZ, P]),
    "msgl_tp_unique_id_size": (SZ, []),
    "msgl_tp_get_unique_id": (I, [P]),
    "msgl_tp_init": (I, [I, I, P, P]),
    "msgl_tp_destroy": (I, [P]),
    "msgl_tp_rank": (I, [P]),
    "msgl_tp_world": (I, [P]),
    "msgl_tp_all_reduce_sum": (I, [P, P, I64, P]),
    "msgl_tp_all_gather": (I, [P, P, C.c_size_t, P]),
    "msgl_tp_allreduce_add_rmsnorm": (I, [P, P, P, P, I, I, F, I, P]),
    "msgl_tp_argmax_combine": (I, [P, P, P, I, P]),
    "msgl_tp_enable_p2p": (I, [P, SZ, P]),
    "msgl_tp_p2p_buffer": (I, [P, I, P, P]),
    "msgl_tp_fused_allreduce_add_rmsnorm": (I, [P, P, P, P, P, I, I, F, I, P]),
    "msgl_tp_fused_allreduce_add_rmsnorm_2shot": (I, [P, P, P, P, P, I, I, F, I, P]),
    "msgl_tp_shard_plan": (I, [I, I, I, I, I, I, P]),
    # executor (msgl_engine.h)
    "msgl_model_create": (I, [P, P]),
    "msgl_model_destroy": (I, [P]),
    "msgl_model_random_init": (I, [P, U64, F, P]),
    "msgl_model_set_weight": (I, [P, C.c_char_p, P, I64, P]),
    "msgl_model_weight_bytes": (I64, [P]),
    "msgl_model_load_safetensors": (I, [P, C.c_char_p, P]),
    "msgl_safetensors_index": (I, [C.c_char_p, P, P]),
    "msgl_model_get_config": (I, [P, P]),
    "msgl_model_decode_steps": (I, [P, P, I, P, P, P, I, P]),
    "msgl_radix_create": (I, [I, P]),
    "msgl_radix_destroy": (I, [P]),
    "msgl_radix_match": (I, [P, P, I, P, I, P, P]),
    "msgl_radix_insert": (I, [P, P, I, P, P, P, P, P]),
    "msgl_radix_lock": (I, [P, I64, I]),
    "msgl_radix_evict": (I, [P, I, P, P]),
    "msgl_radix_size": (I, [P, P, P]),
    "msgl_model_alloc_kv": (I, [P, I, I, P]),
    "msgl_model_kv_pool": (I, [P, I, P, P, P]),
    "msgl_model_forward": (I, [P, P, P, P, I, P]),
    "msgl_model_step_host": (I, [P, P, P, I, P]),
    "msgl_model_step_host_async": (I, [P, P, P, I, P, P]),
    "msgl_model_step_wait": (I, [P, U64]),
    "msgl_model_decode_steps_stop": (I, [P, P, I, P, P, P, P, I, P]),
    "msgl_decode_advance_masked": (I, [P, P, P, P, P, I, P, P, P, P, I, I, P]),
    "msgl_decode_finish": (I, [P, P, P, P, P, I, P, P, I, P]),
    "msgl_model_debug_hidden": (I, [P, P, P]),
    "msgl_model_set_num_layers_run": (I, [P, I]),
    "msgl_model_set_tp": (I, [P, P]),
}

_LIB = None


class MsglError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"msgl error {code}: {msg}")
        self.code = code


def header_symbols() -> list[str]:
    """Names of every entry point declared with MSGL_API in include/*.h."""
    names = []
    for h in HEADERS:
        if os.path.exists(h):
            names += re.findall(r"^MSGL_API[^(]*?\b(msgl_\w+)\s*\(", open(h).read(), flags=re.M)
    return names


def lib():
    """The loaded libmsgl (ctypes.CDLL). Raises if the in-tree library has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} not built: run `python mini-sglang-cpp_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int) -> None:
    if rc != 0:
        raise MsglError(rc, lib().msgl_last_error().decode())
