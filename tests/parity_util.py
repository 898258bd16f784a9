"""Shared helpers of the GPU parity tests: the oracle model that matches an
engine's configuration, filled either from the seeded CPU generator or with
the engine's own resident weights (read back through sfk_weights_get straight
into the oracle's tensor buffers -- the generator equality itself is checked
separately, so large models need not be generated twice), and the north-star
logit tolerance (1e-3 relative L2, 1e-2 max-abs)."""
import ctypes as C

import numpy as np

from oracle import oracle as O

REL_L2, MAX_ABS = 1e-3, 1e-2


def oracle_cfg(cfg, **kw):
    d = {k: getattr(cfg, k) for k in ("n_embd", "n_head", "n_head_kv", "n_layer", "n_ff", "n_expert", "n_expert_used",
                                      "n_vocab", "n_ctx", "rms_eps", "freq_base", "type_embd", "type_attn",
                                      "type_ffn_gu", "type_ffn_down", "type_output", "head_dim")}
    d["kv_f16"] = cfg.kv_type == 1
    d.update(kw)
    return O.ModelConfig(**d)


def oracle_from_engine(eng, **kw) -> O.Model:
    """An oracle model holding exactly the engine's weights (GGUF bytes)."""
    from strataflow_b200 import lib as L
    om = O.Model(oracle_cfg(eng.cfg, **kw))
    for tid, layer in om.tensors():
        n = O.lib().sfo_tensor_bytes(om.h, tid, layer, None, None)
        assert n == eng.tensor_bytes(tid, layer), (tid, layer)
        ptr = O.lib().sfo_tensor_data(om.h, tid, layer)
        L.check(eng._lib.sfk_weights_get(eng.h, tid, layer, C.c_void_p(ptr), n))
    return om


def close(a, b):
    """(within tolerance, relative L2, max-abs) of logits a against oracle b."""
    rel = float(np.linalg.norm(a - b) / np.linalg.norm(b))
    mx = float(np.abs(a - b).max())
    return rel < REL_L2 and mx < MAX_ABS, rel, mx
