"""Host-side mirror of StrataFlow's engine::Engine for the B200 decode path.

Reference interface (Coaade-Inc/strataflow, src/model/engine/engine.h):
  Engine::load(path, expert_slots, kv_window, trunk_pool_layers, backend)  :153
  Engine::forward(token, pos, std::vector<float>& logits) -> bool          :241
  Engine::reset_kv()                                                       :245
  EngineHParams                                                             :41

Here `Engine.load` takes the model shape (the GGUF hparams the reference reads
at engine.cpp:1077-1087) and fills the HBM tier either from the seeded
synthetic generator (on the device) or from GGUF tensor bytes; `forward`
returns the logits (raising on failure where the reference returns false).
All arithmetic runs in libsfk.so; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, asdict

import numpy as np

from . import lib as L


@dataclass
class ModelConfig:
    """Model shape (EngineHParams) plus the quant type of each weight class."""
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
    type_embd: int = L.TYPE_Q8_0
    type_attn: int = L.TYPE_Q8_0
    type_ffn_gu: int = L.TYPE_Q8_0
    type_ffn_down: int = L.TYPE_Q8_0
    type_output: int = L.TYPE_Q8_0
    kv_type: int = L.KV_F32
    max_batch: int = 1
    ep_size: int = 1   # expert-parallel ranks (one engine per GPU)
    ep_rank: int = 0
    head_dim: int = 0  # 0: n_embd / n_head
    expert_slots: int = 0  # HBM expert slots; 0: every expert resident (Engine::load's expert_slots)
    kv_window: int = 0     # resident KV tokens per sequence; 0: the whole context (Engine::load's kv_window)

    @property
    def hd(self) -> int:
        """The attention head width in use."""
        return self.head_dim if self.head_dim > 0 else self.n_embd // self.n_head

    def to_c(self) -> L.Hparams:
        h = L.Hparams()
        for name, _ in L.Hparams._fields_:
            setattr(h, name, getattr(self, name))
        return h

    def replace(self, **kw) -> "ModelConfig":
        d = asdict(self)
        d.update(kw)
        return ModelConfig(**d)


# The BASELINE.json configurations (shapes only; weights are seeded synthetic).
def tiny_config(**kw) -> ModelConfig:
    """4 layers, d 256, 8q/4kv heads (hd 32), 8 experts top-2,
    FFN 512, vocab 4096, Q8_0 weights, RoPE base 1e4, context 80."""
    c = ModelConfig(n_embd=256, n_head=8, n_head_kv=4, n_layer=4, n_ff=512, n_expert=8, n_expert_used=2,
                    n_vocab=4096, n_ctx=80, rms_eps=1e-5, freq_base=10000.0)
    return c.replace(**kw)


def mixtral_config(**kw) -> ModelConfig:
    """Mixtral-8x7B shape -- 32 layers, d 4096, 32q/8kv heads
    (hd 128), 8 experts top-2, FFN 14336, vocab 32000, RoPE base 1e6; experts
    Q4_K, attention / embedding / output Q6_K, router F32."""
    c = ModelConfig(n_embd=4096, n_head=32, n_head_kv=8, n_layer=32, n_ff=14336, n_expert=8, n_expert_used=2,
                    n_vocab=32000, n_ctx=1024, rms_eps=1e-5, freq_base=1e6, type_embd=L.TYPE_Q6_K,
                    type_attn=L.TYPE_Q6_K, type_ffn_gu=L.TYPE_Q4_K, type_ffn_down=L.TYPE_Q4_K,
                    type_output=L.TYPE_Q6_K, kv_type=L.KV_F16)
    return c.replace(**kw)


def trillion_config(**kw) -> ModelConfig:
    """~1T-parameter llama-arch MoE -- 61 layers, d 7168, 64q/8kv
    heads (hd 128), 384 experts top-8, FFN 2048, vocab 160000; experts Q4_K,
    trunk Q8_0 (RoPE base unspecified there: 1e4), f16 KV, context 1280 (a
    1024-token prompt + 128 decode steps); meant for expert parallelism
    (ep_size 4 or 8: ~156 or ~84 GB per GPU)."""
    c = ModelConfig(n_embd=7168, n_head=64, n_head_kv=8, n_layer=61, n_ff=2048, n_expert=384, n_expert_used=8,
                    n_vocab=160000, n_ctx=1280, rms_eps=1e-5, freq_base=10000.0, head_dim=128, type_embd=L.TYPE_Q8_0,
                    type_attn=L.TYPE_Q8_0, type_ffn_gu=L.TYPE_Q4_K, type_ffn_down=L.TYPE_Q4_K,
                    type_output=L.TYPE_Q8_0, kv_type=L.KV_F16)
    return c.replace(**kw)


class Engine:
    """One model resident in HBM plus its paged KV cache (max_batch sequences)."""

    def __init__(self, cfg: ModelConfig, device: int = 0):
        self.cfg = cfg
        self._lib = L.load()
        self._hp = cfg.to_c()
        h = C.c_void_p()
        L.check(self._lib.sfk_engine_create(device, C.byref(self._hp), C.byref(h)))
        self.h = h

    @classmethod
    def load(cls, cfg: ModelConfig, seed: int | None = None, tensors=None, device: int = 0) -> "Engine":
        """Create the engine and fill its HBM tier: from the seeded generator
        (`seed`) or from an iterable of (tensor_id, layer, ggml_type, ne,
        bytes) in GGUF layout (`tensors`)."""
        eng = cls(cfg, device)
        if seed is not None:
            L.check(eng._lib.sfk_weights_synth(eng.h, C.c_uint64(seed)))
        if tensors is not None:
            for tid, layer, qtype, ne, data in tensors:
                eng.put(tid, layer, qtype, ne, data)
        return eng

    @classmethod
    def load_strata(cls, path: str, n_ctx: int = 0, max_batch: int = 1, kv_type: int = L.KV_F16,
                    ep_size: int = 1, ep_rank: int = 0, device: int = 0, expert_slots: int = 0) -> "Engine":
        """Engine::load of a .strata file (engine.cpp:983-1137 with
        load_strata_weights): the model shape from the file's GGUF metadata,
        every trunk tensor and expert bundle uploaded to the HBM tier (or,
        with expert_slots below n_layer * n_expert, to the pinned host store
        behind a pool of that many HBM slots).  n_ctx <= 0 takes the file's
        llama.context_length."""
        from .strata import StrataFile
        with StrataFile(path) as f:
            base = L.Hparams()
            base.n_ctx, base.max_batch, base.kv_type, base.ep_size, base.ep_rank = n_ctx, max_batch, kv_type, \
                ep_size, ep_rank
            base.expert_slots = expert_slots
            hp = f.hparams(base)
            cfg = ModelConfig(**{n: getattr(hp, n) for n, _ in L.Hparams._fields_})
            eng = cls(cfg, device)
            try:
                f.load_into(eng)
            except Exception:
                eng.close()
                raise
        return eng

    def close(self):
        if getattr(self, "h", None):
            self._lib.sfk_engine_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def stream(self) -> int:
        """cudaStream_t (as an int) every call of this engine is ordered on."""
        return int(self._lib.sfk_engine_stream(self.h) or 0)

    # -- expert parallelism ---------------------------------------------------
    def ep_handle(self) -> bytes:
        """This rank's exchange-buffer handle (to be passed to every rank)."""
        buf = (C.c_uint8 * L.EP_HANDLE_BYTES)()
        L.check(self._lib.sfk_ep_handle(self.h, buf, L.EP_HANDLE_BYTES))
        return bytes(buf)

    def ep_connect(self, handles) -> None:
        """Open every rank's exchange buffer (handles in rank order)."""
        blob = b"".join(handles)
        L.check(self._lib.sfk_ep_connect(self.h, blob, len(handles)))

    def ep_connect_group(self, group=None) -> None:
        """Exchange handles over a torch.distributed group and connect."""
        import torch.distributed as dist
        hs = [None] * dist.get_world_size(group)
        dist.all_gather_object(hs, self.ep_handle(), group=group)
        self.ep_connect(hs)

    def time_kernels(self, n_seq: int = 1, iters: int = 32) -> dict:
        """Average device ms of each kernel class of one step (sfk_time_kernels)."""
        ms = (C.c_float * 8)()
        L.check(self._lib.sfk_time_kernels(self.h, n_seq, iters, ms, 8))
        names = ["embed", "qkv", "attention", "o_proj", "router", "gate_up", "down", "lm_head"]
        return {n: float(v) for n, v in zip(names, ms)}

    # -- weights -----------------------------------------------------------
    def tensor_bytes(self, tid: int, layer: int = 0) -> int:
        return int(self._lib.sfk_tensor_bytes(self.h, tid, layer))

    def put(self, tid: int, layer: int, qtype: int, ne, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data).view(np.uint8)
        ne_c = (C.c_int64 * 3)(*(list(ne) + [1, 1, 1])[:3])
        L.check(self._lib.sfk_weights_put(self.h, tid, layer, qtype, ne_c, data.ctypes.data_as(C.c_void_p),
                                          data.nbytes))

    def put_expert(self, layer: int, expert: int, bundle: np.ndarray) -> None:
        bundle = np.ascontiguousarray(bundle).view(np.uint8)
        L.check(self._lib.sfk_expert_put(self.h, layer, expert, bundle.ctypes.data_as(C.c_void_p), bundle.nbytes))

    def get(self, tid: int, layer: int = 0) -> np.ndarray:
        n = self.tensor_bytes(tid, layer)
        out = np.empty(n, np.uint8)
        L.check(self._lib.sfk_weights_get(self.h, tid, layer, out.ctypes.data_as(C.c_void_p), n))
        return out

    # -- decode --------------------------------------------------------------
    def reset_kv(self) -> None:
        L.check(self._lib.sfk_kv_reset(self.h))

    def forward(self, token: int, pos: int, want_logits: bool = True):
        """Engine::forward: one token at `pos`; returns (argmax, logits)."""
        logits = np.empty(self.cfg.n_vocab, np.float32) if want_logits else None
        am = C.c_int32()
        L.check(self._lib.sfk_forward(self.h, int(token), int(pos),
                                      logits.ctypes.data_as(C.c_void_p) if want_logits else None, C.byref(am)))
        return am.value, logits

    def forward_batch(self, tokens, positions, want_logits: bool = True):
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        n = tokens.size
        logits = np.empty((n, self.cfg.n_vocab), np.float32) if want_logits else None
        am = np.empty(n, np.int32)
        L.check(self._lib.sfk_forward_batch(self.h, n, tokens.ctypes.data_as(C.c_void_p),
                                            positions.ctypes.data_as(C.c_void_p),
                                            logits.ctypes.data_as(C.c_void_p) if want_logits else None,
                                            am.ctypes.data_as(C.c_void_p)))
        return am, logits

    def prefill(self, tokens, pos0: int = 0, seq: int = 0, want_logits: bool = True):
        """Batched prompt prefill (sfk_prefill): tokens at positions pos0..;
        returns (argmax, logits) of the last prompt token.  Decoding then
        continues with decode_greedy / forward."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.n_vocab, np.float32) if want_logits else None
        am = C.c_int32()
        L.check(self._lib.sfk_prefill(self.h, int(seq), tokens.ctypes.data_as(C.c_void_p), int(tokens.size), int(pos0),
                                      logits.ctypes.data_as(C.c_void_p) if want_logits else None, C.byref(am)))
        return am.value, logits

    def decode_greedy(self, n_steps: int, n_seq: int = 1, want_tokens: bool = True):
        """Greedy loop on the device; returns the tokens fed at each step
        ([n_steps][n_seq]); the first is the argmax of the previous step."""
        out = np.empty((n_steps, n_seq), np.int32) if want_tokens else None
        L.check(self._lib.sfk_decode_greedy(self.h, n_seq, n_steps,
                                            out.ctypes.data_as(C.c_void_p) if want_tokens else None))
        return out

    def route(self, n_seq: int = 1):
        """(ids, weights) of the last layer's routing in the last step."""
        k = self.cfg.n_expert_used
        ids = np.empty((n_seq, k), np.int32)
        w = np.empty((n_seq, k), np.float32)
        L.check(self._lib.sfk_route_get(self.h, ids.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p),
                                        ids.size))
        return ids, w

    def debug(self, which: int, n_seq: int = 1) -> np.ndarray:
        """Step buffers of the last layer (sfk_debug_get): 0 attention output,
        1 ffn_inp, 2 q after RoPE, 3 SwiGLU activation."""
        c = self.cfg
        n = {0: c.n_head * c.hd, 1: c.n_embd, 2: c.n_head * c.hd,
             3: c.n_expert_used * c.n_ff}[which] * n_seq
        out = np.empty(n, np.float32)
        L.check(self._lib.sfk_debug_get(self.h, which, out.ctypes.data_as(C.c_void_p), n))
        return out

    def hidden(self, n_seq: int = 1) -> np.ndarray:
        out = np.empty((n_seq, self.cfg.n_embd), np.float32)
        L.check(self._lib.sfk_hidden_get(self.h, out.ctypes.data_as(C.c_void_p), out.size))
        return out

    def stats(self) -> dict:
        s = L.Stats()
        L.check(self._lib.sfk_get_stats(self.h, C.byref(s)))
        return {n: int(getattr(s, n)) for n, _ in L.Stats._fields_}

    def generate_api(self, prompt, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, seed: int = 0,
                     max_tokens: int = 256, eos_token: int = -1, callback=None) -> list[int]:
        """sfk_generate: the reference's sf_generate on sequence 0 with every
        prompt token prefilled, then tokens greedy (temperature <= 0) or
        sampled on the device.  callback(token) -> truthy stops the loop."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        sp = L.Sampling(float(temperature), float(top_p), int(top_k), int(seed), int(max_tokens), int(eos_token))
        cap = max_tokens if max_tokens > 0 else 256
        out = np.empty(cap, np.int32)
        n = C.c_int32()
        cb = L.TOKEN_CB(lambda tok, _u: 1 if (callback is not None and callback(int(tok))) else 0)
        L.check(self._lib.sfk_generate(self.h, prompt.ctypes.data_as(C.c_void_p), int(prompt.size), C.byref(sp),
                                       out.ctypes.data_as(C.c_void_p), cap, C.byref(n), cb, None))
        return out[:n.value].tolist()

    def generate(self, prompt, n_gen: int, host_loop: bool = False):
        """The reference drive pattern (tests/test_engine_oracle.cpp:182-207):
        prompt tokens one position at a time, then n_gen greedy tokens.
        Returns (generated tokens, logits of each step when host_loop)."""
        pos = 0
        am = None
        logits_all = []
        last = None
        for t in prompt:
            am, last = self.forward(t, pos, want_logits=host_loop)
            pos += 1
        if host_loop:
            logits_all.append(last)
            out = []
            for _ in range(n_gen):
                out.append(am)
                am, last = self.forward(am, pos)
                logits_all.append(last)
                pos += 1
            return out, logits_all
        toks = self.decode_greedy(n_gen, 1)[:, 0].tolist()
        return toks, None
