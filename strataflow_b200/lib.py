"""ctypes binding of libsfk.so (include/sfk.h).

The library is required: importing the engine or an op on a machine where the
shared object is missing raises immediately.  There is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libsfk.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "sfk.h")

SFK_OK = 0
SFK_ERR_INVALID_ARGUMENT, SFK_ERR_UNSUPPORTED, SFK_ERR_OUT_OF_MEMORY, SFK_ERR_RUNTIME = 1, 3, 4, 7
TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_K = 0, 1, 8, 12, 14, 15
KV_F32, KV_F16 = 0, 1
(T_TOK_EMBD, T_OUTPUT_NORM, T_OUTPUT, T_ATTN_NORM, T_ATTN_Q, T_ATTN_K, T_ATTN_V, T_ATTN_OUT,
 T_FFN_NORM, T_FFN_GATE_INP, T_FFN_GATE_EXPS, T_FFN_UP_EXPS, T_FFN_DOWN_EXPS) = range(13)
LAYERED = set(range(T_ATTN_NORM, 13))


class SfkError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"sfk status {status}: {msg}")
        self.status = status


class Hparams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "n_embd", "n_head", "n_head_kv", "n_layer", "n_ff", "n_expert", "n_expert_used", "n_vocab", "n_ctx")] + [
        ("rms_eps", C.c_float), ("freq_base", C.c_float)] + [(n, C.c_int32) for n in (
            "type_embd", "type_attn", "type_ffn_gu", "type_ffn_down", "type_output", "kv_type", "max_batch",
            "ep_size", "ep_rank", "head_dim", "expert_slots", "kv_window")]


EP_HANDLE_BYTES = 64  # SFK_EP_HANDLE_BYTES


class Stats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "weight_bytes_hbm", "kv_bytes_hbm", "scratch_bytes_hbm", "steps", "kernels_per_step",
        "active_bytes_per_token", "pool_slots", "pool_hits", "pool_misses", "pool_evictions", "h2d_expert_bytes",
        "prefetch_warmed", "prefetch_used", "kv_window_pages", "kv_pages_evicted", "kv_staged_bytes")]


class Sampling(C.Structure):
    """sfk_sampling: the reference's sf_sampling_params plus the eos token."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int32), ("seed", C.c_uint64),
                ("max_tokens", C.c_int32), ("eos_token", C.c_int32)]


TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)

P, I32, I64, U64, SZ, F = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_size_t, C.c_float
U32 = C.c_uint32
_SIGS = {
    "sfk_last_error": (C.c_char_p, []),
    "sfk_status_str": (C.c_char_p, [I32]),
    "sfk_engine_create": (I32, [C.c_int, C.POINTER(Hparams), C.POINTER(P)]),
    "sfk_engine_free": (None, [P]),
    "sfk_engine_stream": (P, [P]),
    "sfk_weights_put": (I32, [P, C.c_int, C.c_int, C.c_int, P, P, SZ]),
    "sfk_expert_put": (I32, [P, C.c_int, C.c_int, P, SZ]),
    "sfk_weights_get": (I32, [P, C.c_int, C.c_int, P, SZ]),
    "sfk_weights_synth": (I32, [P, U64]),
    "sfk_tensor_bytes": (SZ, [P, C.c_int, C.c_int]),
    "sfk_kv_reset": (I32, [P]),
    "sfk_forward": (I32, [P, I32, I32, P, P]),
    "sfk_forward_batch": (I32, [P, I32, P, P, P, P]),
    "sfk_decode_greedy": (I32, [P, I32, I32, P]),
    "sfk_prefill": (I32, [P, I32, P, I32, I32, P, P]),
    "sfk_sampling_defaults": (Sampling, []),
    "sfk_generate": (I32, [P, P, I32, C.POINTER(Sampling), P, I32, C.POINTER(I32), TOKEN_CB, P]),
    "sfk_sample_logits": (I32, [P, I32, C.POINTER(Sampling), I32, C.POINTER(I32), P]),
    "sfk_hidden_get": (I32, [P, P, SZ]),
    "sfk_route_get": (I32, [P, P, P, SZ]),
    "sfk_debug_get": (I32, [P, I32, P, SZ]),
    "sfk_get_stats": (I32, [P, C.POINTER(Stats)]),
    "sfk_time_kernels": (I32, [P, I32, I32, P, I32]),
    "sfk_dev_row_bytes": (I64, [C.c_int, I64]),
    "sfk_repack": (I32, [C.c_int, P, P, I64, I64, P]),
    "sfk_unpack": (I32, [C.c_int, P, P, I64, I64, P]),
    "sfk_dequantize": (I32, [C.c_int, P, P, I64, P]),
    "sfk_quantize_act": (I32, [C.c_int, P, I32, I64, P, P]),
    "sfk_mul_mat": (I32, [C.c_int, P, I64, I64, P, I32, P, P]),
    "sfk_mul_mat_tc": (I32, [C.c_int, P, I64, I64, P, I32, P, P]),
    "sfk_mul_mat_id": (I32, [C.c_int, P, I32, I64, I64, P, I32, P, I32, I32, P, P]),
    "sfk_mul_mat_id_tc": (I32, [C.c_int, P, I32, I64, I64, P, I32, P, I32, I32, P, P]),
    "sfk_moe_ffn": (I32, [C.c_int, C.c_int, P, P, P, I32, I64, I64, P, P, P, P, I32, I32, P, P]),
    "sfk_moe_ffn_noalloc": (I32, [C.c_int, C.c_int, P, P, P, I32, I64, I64, P, P, P, P, I32, I32, P, P]),
    "sfk_attn_decode_paged": (I32, [P, P, P, I32, I32, P, I32, P, I32, I32, I32, I32, P, P]),
    "sfk_ep_handle": (I32, [P, P, SZ]),
    "sfk_ep_connect": (I32, [P, P, I32]),
    "sfk_strata_open": (I32, [C.c_char_p, C.POINTER(P)]),
    "sfk_strata_close": (None, [P]),
    "sfk_strata_hparams": (I32, [P, C.POINTER(Hparams)]),
    "sfk_strata_n_tensors": (I64, [P]),
    "sfk_strata_tensor_info": (I32, [P, I64, C.c_char_p, SZ, C.POINTER(I32), P, C.POINTER(U64), C.POINTER(I32)]),
    "sfk_strata_read_trunk": (I32, [P, C.c_char_p, P, SZ]),
    "sfk_strata_bundle_bytes": (SZ, [P, I32]),
    "sfk_strata_read_bundle": (I32, [P, I32, I32, P, SZ]),
    "sfk_strata_load": (I32, [P, P]),
    "sfk_strata_pack": (I32, [C.c_char_p, C.c_char_p]),
    "sfk_embed": (I32, [P, P, P, I32, P]),
    "sfk_decode_layer_attn": (I32, [P, I32, P, I32, P]),
    "sfk_decode_layer_moe": (I32, [P, I32, I32, P, P, P]),
    "sfk_lm_head": (I32, [P, P, I32, P, P]),
    "sfk_pool_create": (I32, [U32, U32, U32, U32, C.POINTER(P)]),
    "sfk_pool_free": (None, [P]),
    "sfk_pool_acquire": (I64, [P, U32, U32, C.POINTER(I32)]),
    "sfk_pool_resident": (I32, [P, U32, U32]),
    "sfk_pool_stratified": (I32, [P]),
    "sfk_pool_layer_capacity": (U32, [P, U32]),
    "sfk_pool_has_free_slot_in_layer": (I32, [P, U32]),
    "sfk_pool_set_layer_weights": (I32, [P, P, U32]),
    "sfk_pool_pin": (I32, [P, U32]),
    "sfk_pool_unpin_all": (I32, [P]),
    "sfk_pool_stats": (I32, [P, P]),
    "sfk_predictor_create": (I32, [U32, U32, C.POINTER(P)]),
    "sfk_predictor_free": (None, [P]),
    "sfk_predictor_observe": (I32, [P, U32, U32]),
    "sfk_predictor_predict": (U32, [P, U32, U32, P]),
    "sfk_predictor_accuracy": (C.c_double, [P]),
    "sfk_predictor_layer_activity": (I32, [P, P, U32]),
}

_lib = None


def header_functions() -> list[str]:
    """Function names declared in include/sfk.h."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(sfk_[a-z0-9_]+)\s*\(", txt)))


def load() -> C.CDLL:
    """Load libsfk.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m strataflow_b200.build` "
                              "(the CUDA extension is required; there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != SFK_OK:
        raise SfkError(status, load().sfk_last_error().decode())
