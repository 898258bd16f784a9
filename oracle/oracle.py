"""ctypes binding of the CPU oracle (oracle/sf_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path.  Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg may
import this module.  The product package (strataflow_b200) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libsf_oracle.so")

F32, F16, Q8_0, Q4_K, Q6_K, Q8_K = 0, 1, 8, 12, 14, 15
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q8_K: (256, 292)}

(T_TOK_EMBD, T_OUTPUT_NORM, T_OUTPUT, T_ATTN_NORM, T_ATTN_Q, T_ATTN_K, T_ATTN_V, T_ATTN_OUT,
 T_FFN_NORM, T_FFN_GATE_INP, T_FFN_GATE_EXPS, T_FFN_UP_EXPS, T_FFN_DOWN_EXPS) = range(13)
LAYERED = set(range(T_ATTN_NORM, 13))


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def row_bytes(qtype: int, n: int) -> int:
    qk, bs = BLOCK[qtype]
    assert n % qk == 0
    return n // qk * bs


class Hparams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "n_embd", "n_head", "n_head_kv", "n_layer", "n_ff", "n_expert", "n_expert_used", "n_vocab", "n_ctx")] + [
        ("rms_eps", C.c_float), ("freq_base", C.c_float)] + [(n, C.c_int32) for n in (
            "type_embd", "type_attn", "type_ffn_gu", "type_ffn_down", "type_output", "kv_f16", "fp32_mode",
            "head_dim", "ep_size", "ep_head_par")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, I64, F, U64, SZ = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64, C.c_size_t
        sig = {
            "sfo_fp32_to_fp16": (C.c_uint16, [F]),
            "sfo_fp16_to_fp32": (F, [C.c_uint16]),
            "sfo_row_bytes": (SZ, [I, I64]),
            "sfo_dequantize": (I, [I, P, P, I64]),
            "sfo_quantize_q8_0": (I, [P, P, I64]),
            "sfo_quantize_q8_K": (I, [P, P, I64]),
            "sfo_quantize_weights": (I, [I, P, P, I64, I64]),
            "sfo_synth_f32": (None, [U64, I64, I64, F, P]),
            "sfo_mul_mat": (I, [I, P, I64, I64, P, P, I]),
            "sfo_rms_norm": (None, [P, P, I64, F, P]),
            "sfo_rope_normal": (None, [P, I, I, I, F]),
            "sfo_soft_max": (None, [P, P, I64, F]),
            "sfo_top_k_desc": (None, [P, I64, I, P]),
            "sfo_moe_ffn": (I, [I, I, P, P, P, I, I, I, I, I, P, P, P, P, P, P, I]),
            "sfo_router": (None, [P, I, I, P, I, P, P, P]),
            "sfo_attn_decode": (None, [P, P, P, I, I, I, I, P]),
            "sfo_model_create": (P, [P]),
            "sfo_model_free": (None, [P]),
            "sfo_set_fp32_mode": (None, [P, I]),
            "sfo_sample": (C.c_int32, [P, I64, C.c_float, C.c_int32, C.c_float, U64, C.c_int32]),
            "sfo_tensor_bytes": (SZ, [P, I, I, P, P]),
            "sfo_tensor_data": (P, [P, I, I]),
            "sfo_model_synth": (I, [P, U64]),
            "sfo_seq_create": (P, [P]),
            "sfo_seq_free": (None, [P]),
            "sfo_seq_reset": (None, [P]),
            "sfo_seq_fill_kv": (I, [P, I, U64]),
            "sfo_forward": (C.c_int32, [P, P, C.c_int32, C.c_int32, P]),
            "sfo_seq_hidden": (P, [P, I]),
            "sfo_seq_ids": (P, [P, I]),
            "sfo_argmax": (C.c_int32, [P, I]),
            "sfo_tensor_seed": (U64, [U64, I, I]),
            "sfo_set_threads": (None, [I]),
            "sfo_seq_timing": (None, [P, P, P]),
            "sfo_seq_debug": (P, [P, I, I]),
            "sfo_expf": (F, [F]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def set_threads(n: int) -> None:
    lib().sfo_set_threads(int(n))


def dequantize(qtype: int, data: np.ndarray, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, np.float32)
    assert lib().sfo_dequantize(qtype, _p(data), _p(out), n) == 0
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(row_bytes(Q8_0, x.size), np.uint8)
    assert lib().sfo_quantize_q8_0(_p(x), _p(out), x.size) == 0
    return out


def quantize_q8_K(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(row_bytes(Q8_K, x.size), np.uint8)
    assert lib().sfo_quantize_q8_K(_p(x), _p(out), x.size) == 0
    return out


def quantize_weights(qtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    nrows, ncols = x.reshape(-1, x.shape[-1]).shape
    out = np.empty(nrows * row_bytes(qtype, ncols), np.uint8)
    assert lib().sfo_quantize_weights(qtype, _p(x), _p(out), nrows, ncols) == 0
    return out


def synth_f32(seed: int, offset: int, n: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().sfo_synth_f32(C.c_uint64(seed), offset, n, std, _p(out))
    return out


def expf(x: float) -> float:
    return float(lib().sfo_expf(float(x)))


def mul_mat(qtype: int, w: np.ndarray, nrows: int, ncols: int, x: np.ndarray, fp32_mode=0) -> np.ndarray:
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(nrows, np.float32)
    assert lib().sfo_mul_mat(qtype, _p(w), nrows, ncols, _p(x), _p(y), int(fp32_mode)) == 0
    return y


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    lib().sfo_rms_norm(_p(x), _p(w), x.size, eps, _p(y))
    return y


def rope_normal(x, n_head, head_dim, pos, base):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().sfo_rope_normal(_p(x), n_head, head_dim, pos, base)
    return x


def router(w_r, x, k):
    w_r = np.ascontiguousarray(w_r, dtype=np.float32)
    E, d = w_r.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.empty(k, np.int32)
    wts = np.empty(k, np.float32)
    probs = np.empty(E, np.float32)
    lib().sfo_router(_p(w_r), E, d, _p(x), k, _p(ids), _p(wts), _p(probs))
    return ids, wts, probs


def moe_ffn(type_gu, type_down, gate, up, down, n_expert, d, F, x, res, ids, wts, fp32_mode=False):
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.shape[0]
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    k = ids.shape[1]
    wts = np.ascontiguousarray(wts, dtype=np.float32)
    out = np.empty((b, d), np.float32)
    gu = np.empty((b, k, F), np.float32)
    resp = None
    if res is not None:
        res = np.ascontiguousarray(res, dtype=np.float32)
        resp = _p(res)
    rc = lib().sfo_moe_ffn(type_gu, type_down, _p(gate), _p(up), _p(down), n_expert, d, F, b, k,
                           _p(x), resp, _p(ids), _p(wts), _p(out), _p(gu), int(fp32_mode))
    assert rc == 0
    return out, gu


def attn_decode(q, k, v, n_head, n_head_kv, head_dim):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    n_kv = k.shape[0]
    out = np.empty(n_head * head_dim, np.float32)
    lib().sfo_attn_decode(_p(q), _p(k), _p(v), n_kv, n_head, n_head_kv, head_dim, _p(out))
    return out


def tensor_seed(seed: int, tid: int, layer: int) -> int:
    return int(lib().sfo_tensor_seed(C.c_uint64(seed), tid, layer))


@dataclass
class ModelConfig:
    """Shape of a llama-arch MoE decode model (engine.h EngineHParams)."""
    n_embd: int
    n_head: int
    n_head_kv: int
    n_layer: int
    n_ff: int
    n_expert: int
    n_expert_used: int
    n_vocab: int
    n_ctx: int
    rms_eps: float = 1e-5
    freq_base: float = 10000.0
    type_embd: int = Q8_0
    type_attn: int = Q8_0
    type_ffn_gu: int = Q8_0
    type_ffn_down: int = Q8_0
    type_output: int = Q8_0
    kv_f16: bool = False
    fp32_mode: bool = False
    head_dim: int = 0   # 0: n_embd / n_head
    ep_size: int = 0    # expert parallelism's fp32 order over ep_size ranks (0 / 1: one GPU)
    ep_head_par: int = 0  # ... with the output projection split by heads

    def to_c(self) -> Hparams:
        h = Hparams()
        for name, _ in Hparams._fields_:
            setattr(h, name, getattr(self, name))
        return h


class Model:
    """Oracle model: weights in GGUF block layout + one or more sequences."""

    def __init__(self, cfg: ModelConfig, seed: int | None = None):
        self.cfg = cfg
        self._hp = cfg.to_c()
        self.h = lib().sfo_model_create(C.byref(self._hp))
        if not self.h:
            raise ValueError("oracle: bad hparams")
        if seed is not None:
            assert lib().sfo_model_synth(self.h, C.c_uint64(seed)) == 0

    def __del__(self):
        if getattr(self, "h", None):
            lib().sfo_model_free(self.h)
            self.h = None

    def tensor(self, tid: int, layer: int = 0) -> tuple[np.ndarray, int, tuple]:
        """(bytes view, ggml type, ne) of one tensor (a view into oracle memory)."""
        t = C.c_int()
        ne = (C.c_int64 * 3)()
        nb = lib().sfo_tensor_bytes(self.h, tid, layer, C.byref(t), ne)
        if nb == 0:
            raise KeyError((tid, layer))
        ptr = lib().sfo_tensor_data(self.h, tid, layer)
        arr = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint8)), shape=(nb,))
        return arr, t.value, (ne[0], ne[1], ne[2])

    def tensors(self):
        for tid in range(13):
            for layer in range(self.cfg.n_layer if tid in LAYERED else 1):
                yield tid, layer

    def new_seq(self) -> "Seq":
        return Seq(self)

    def set_fp32_mode(self, mode: int) -> None:
        """fp32 order of later forwards' quantized mul_mats (sfo_set_fp32_mode)."""
        lib().sfo_set_fp32_mode(self.h, int(mode))


class Seq:
    def __init__(self, model: Model):
        self.m = model
        self.h = lib().sfo_seq_create(model.h)
        if not self.h:
            raise MemoryError("oracle: seq alloc")

    def __del__(self):
        if getattr(self, "h", None):
            lib().sfo_seq_free(self.h)
            self.h = None

    def reset(self):
        lib().sfo_seq_reset(self.h)

    def fill_kv(self, n_pos: int, seed: int = 0) -> None:
        """Positions 0..n_pos-1 of the KV cache get seeded values (a stand-in
        for a fed prompt, for timing decode steps at a long context)."""
        assert lib().sfo_seq_fill_kv(self.h, int(n_pos), C.c_uint64(seed)) == 0

    def forward(self, token: int, pos: int) -> tuple[int, np.ndarray]:
        logits = np.empty(self.m.cfg.n_vocab, np.float32)
        am = lib().sfo_forward(self.m.h, self.h, int(token), int(pos), _p(logits))
        if am < 0:
            raise ValueError("oracle forward failed")
        return am, logits

    def timing(self) -> tuple[float, float]:
        """(seconds in the layer loop, seconds in embedding + head) so far."""
        a, b = C.c_double(), C.c_double()
        lib().sfo_seq_timing(self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def debug(self, il: int, which: int, n: int) -> np.ndarray:
        """Layer il intermediates of the last forward (see sfo_seq_debug)."""
        ptr = lib().sfo_seq_debug(self.h, il, which)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_float)), shape=(n,)).copy()

    def hidden(self, il: int) -> np.ndarray:
        ptr = lib().sfo_seq_hidden(self.h, il)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_float)), shape=(self.m.cfg.n_embd,)).copy()

    def ids(self, il: int) -> np.ndarray:
        ptr = lib().sfo_seq_ids(self.h, il)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_int32)),
                                     shape=(self.m.cfg.n_expert_used,)).copy()


def sample(logits: np.ndarray, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0,
           step: int = 0) -> int:
    """Token sampling of the generate loop (sfo_sample)."""
    lg = np.ascontiguousarray(logits, np.float32)
    return int(lib().sfo_sample(_p(lg), lg.size, float(temperature), int(top_k), float(top_p), int(seed), int(step)))


def greedy(model: Model, prompt: list[int], n_gen: int, want_logits=False, prompt_fp32_mode=None):
    """Prompt one token per position, then n_gen greedy tokens (the reference's
    tests/test_engine_oracle.cpp:182-207 drive pattern).  prompt_fp32_mode:
    the fp32 order of the prompt tokens' mul_mats (2: the per-block order of a
    batched prefill), the model's own order for the generated tokens."""
    seq = model.new_seq()
    pos = 0
    logits_all = []
    tok = None
    last = None
    if prompt_fp32_mode is not None:
        model.set_fp32_mode(prompt_fp32_mode)
    try:
        for t in prompt:
            tok, last = seq.forward(t, pos)
            pos += 1
    finally:
        if prompt_fp32_mode is not None:
            model.set_fp32_mode(int(model.cfg.fp32_mode))
    if want_logits:
        logits_all.append(last)
    out = []
    for _ in range(n_gen):
        out.append(tok)
        tok, last = seq.forward(tok, pos)
        pos += 1
        if want_logits:
            logits_all.append(last)
    return out, logits_all
