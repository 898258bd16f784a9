"""Operator-level entry points over torch CUDA tensors (device memory only).

Each call forwards device pointers to libsfk.so (include/sfk.h) on the tensor's
current CUDA stream.  Mirrors the ggml ops the reference's decode path issues
(src/model/engine/engine.cpp): ggml_get_rows dequant (:2712), ggml_mul_mat
(:1882-1889,1905,2994), ggml_mul_mat_id (:1967-1970), the fused expert segment
(:1956-1989) and the decode attention (:1751-1761).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import lib as L


def _ptr(t: torch.Tensor):
    assert t.is_cuda and t.is_contiguous()
    return C.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def dev_row_bytes(qtype: int, K: int) -> int:
    return int(L.load().sfk_dev_row_bytes(qtype, K))


def repack(qtype: int, gguf: torch.Tensor, nrows: int, K: int) -> torch.Tensor:
    """GGUF rows (uint8 CUDA tensor) -> device-layout weight tensor."""
    out = torch.empty(nrows * dev_row_bytes(qtype, K), dtype=torch.uint8, device=gguf.device)
    L.check(L.load().sfk_repack(qtype, _ptr(gguf), _ptr(out), nrows, K, _stream(gguf)))
    return out


def unpack(qtype: int, dev: torch.Tensor, nrows: int, K: int, gguf_bytes: int) -> torch.Tensor:
    out = torch.empty(gguf_bytes, dtype=torch.uint8, device=dev.device)
    L.check(L.load().sfk_unpack(qtype, _ptr(dev), _ptr(out), nrows, K, _stream(dev)))
    return out


def dequantize(qtype: int, gguf: torch.Tensor, n: int) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=gguf.device)
    L.check(L.load().sfk_dequantize(qtype, _ptr(gguf), _ptr(out), n, _stream(gguf)))
    return out


def quantize_act(act_type: int, x: torch.Tensor) -> torch.Tensor:
    """[b][K] f32 -> GGUF Q8_K (292 B / 256) or Q8_0 (34 B / 32) blocks."""
    b, K = x.shape
    nbytes = (K // 256) * 292 if act_type == L.TYPE_Q8_K else (K // 32) * 34
    out = torch.empty(b * nbytes, dtype=torch.uint8, device=x.device)
    L.check(L.load().sfk_quantize_act(act_type, _ptr(x), b, K, _ptr(out), _stream(x)))
    return out


def mul_mat(qtype: int, w_dev: torch.Tensor, rows: int, K: int, x: torch.Tensor) -> torch.Tensor:
    b = x.shape[0]
    y = torch.empty((b, rows), dtype=torch.float32, device=x.device)
    L.check(L.load().sfk_mul_mat(qtype, _ptr(w_dev), rows, K, _ptr(x), b, _ptr(y), _stream(x)))
    return y


def mul_mat_tc(qtype: int, w_dev: torch.Tensor, rows: int, K: int, x: torch.Tensor) -> torch.Tensor:
    """The same product for any number of activation rows on the tensor cores
    (sfk_mul_mat_tc): y [n][rows]."""
    n = x.shape[0]
    y = torch.empty((n, rows), dtype=torch.float32, device=x.device)
    L.check(L.load().sfk_mul_mat_tc(qtype, _ptr(w_dev), rows, K, _ptr(x), n, _ptr(y), _stream(x)))
    return y


def mul_mat_id(qtype: int, w_dev: torch.Tensor, n_expert: int, rows: int, K: int, x: torch.Tensor,
               ids: torch.Tensor) -> torch.Tensor:
    """x: [b][K] (broadcast over each token's experts) or [b][k][K]."""
    b, k = ids.shape
    per_pair = 1 if x.dim() == 3 else 0
    y = torch.empty((b, k, rows), dtype=torch.float32, device=x.device)
    L.check(L.load().sfk_mul_mat_id(qtype, _ptr(w_dev), n_expert, rows, K, _ptr(x), per_pair, _ptr(ids), b, k,
                                    _ptr(y), _stream(x)))
    return y


def mul_mat_id_tc(qtype: int, w_dev: torch.Tensor, n_expert: int, rows: int, K: int, x: torch.Tensor,
                  ids: torch.Tensor) -> torch.Tensor:
    """mul_mat_id on the tensor cores (sfk_mul_mat_id_tc), for batches of
    many routed pairs; the same arguments and result layout as mul_mat_id."""
    b, k = ids.shape
    per_pair = 1 if x.dim() == 3 else 0
    y = torch.empty((b, k, rows), dtype=torch.float32, device=x.device)
    L.check(L.load().sfk_mul_mat_id_tc(qtype, _ptr(w_dev), n_expert, rows, K, _ptr(x), per_pair, _ptr(ids), b, k,
                                       _ptr(y), _stream(x)))
    return y


def moe_ffn(type_gu: int, type_down: int, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, n_expert: int,
            d: int, F: int, x: torch.Tensor, res: torch.Tensor | None, ids: torch.Tensor,
            w: torch.Tensor) -> torch.Tensor:
    b, k = ids.shape
    out = torch.empty((b, d), dtype=torch.float32, device=x.device)
    L.check(L.load().sfk_moe_ffn(type_gu, type_down, _ptr(gate), _ptr(up), _ptr(down), n_expert, d, F, _ptr(x),
                                 _ptr(res) if res is not None else None, _ptr(ids), _ptr(w), b, k, _ptr(out),
                                 _stream(x)))
    return out


def attn_decode_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, page_table: torch.Tensor,
                      positions: torch.Tensor, n_head: int, n_head_kv: int, head_dim: int) -> torch.Tensor:
    b = q.shape[0]
    kv_type = L.KV_F16 if k_pages.dtype == torch.float16 else L.KV_F32
    out = torch.empty((b, n_head * head_dim), dtype=torch.float32, device=q.device)
    L.check(L.load().sfk_attn_decode_paged(_ptr(q), _ptr(k_pages), _ptr(v_pages), kv_type, k_pages.shape[0],
                                           _ptr(page_table),
                                           page_table.shape[1], _ptr(positions), b, n_head, n_head_kv, head_dim,
                                           _ptr(out), _stream(q)))
    return out


def sample_logits(logits: torch.Tensor, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0,
                  step: int = 0) -> int:
    """The generate loop's device sampler on f32 logits [V] (sfk_sample_logits)."""
    sp = L.Sampling(float(temperature), float(top_p), int(top_k), int(seed), 0, -1)
    tok = C.c_int32()
    L.check(L.load().sfk_sample_logits(_ptr(logits), int(logits.numel()), C.byref(sp), int(step), C.byref(tok),
                                       _stream(logits)))
    return tok.value
