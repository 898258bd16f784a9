"""The per-layer entry points (sfk_embed, sfk_decode_layer_attn,
sfk_decode_layer_moe, sfk_lm_head): a host engine that keeps the reference's
own layer loop (attention segment, expert segment per layer,
engine.cpp:1854-1989) gets exactly the logits of the whole-step call, and the
routing of each expert segment."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from parity_util import oracle_cfg, close

pytestmark = pytest.mark.gpu


def _layer_chain(eng, tokens, positions, want_ids=False):
    import torch
    from strataflow_b200 import lib as L
    cfg = eng.cfg
    n = len(tokens)
    tok = np.ascontiguousarray(tokens, np.int32)
    pos = np.ascontiguousarray(positions, np.int32)
    hid = torch.empty((n, cfg.n_embd), dtype=torch.float32, device="cuda")
    logits = torch.empty((n, cfg.n_vocab), dtype=torch.float32, device="cuda")
    ids = torch.empty((cfg.n_layer, n, cfg.n_expert_used), dtype=torch.int32, device="cuda")
    w = torch.empty((cfg.n_layer, n, cfg.n_expert_used), dtype=torch.float32, device="cuda")
    lib = eng._lib
    vp = C.c_void_p
    L.check(lib.sfk_embed(eng.h, tok.ctypes.data_as(vp), pos.ctypes.data_as(vp), n, vp(hid.data_ptr())))
    for l in range(cfg.n_layer):
        L.check(lib.sfk_decode_layer_attn(eng.h, l, pos.ctypes.data_as(vp), n, vp(hid.data_ptr())))
        L.check(lib.sfk_decode_layer_moe(eng.h, l, n, vp(hid.data_ptr()), vp(ids[l].data_ptr()),
                                         vp(w[l].data_ptr())))
    am = np.empty(n, np.int32)
    L.check(lib.sfk_lm_head(eng.h, vp(hid.data_ptr()), n, vp(logits.data_ptr()), am.ctypes.data_as(vp)))
    torch.cuda.synchronize()
    return am, logits.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("kw", [{}, dict(type_ffn_gu=12, type_ffn_down=14, type_attn=14, type_output=14,
                                         type_embd=14, kv_type=1, max_batch=3)])
def test_layer_chain_equals_whole_step(cuda, kw):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(**kw)
    B = cfg.max_batch
    ref = E.Engine.load(cfg, seed=31)
    eng = E.Engine.load(cfg, seed=31)
    rng = np.random.default_rng(31)
    for e_ in (ref, eng):
        e_.reset_kv()
    for step in range(24):
        toks = rng.integers(0, cfg.n_vocab, B)
        pos = [step + 2 * t for t in range(B)]
        ra, rl = ref.forward_batch(toks, pos)
        a, lg, ids, w = _layer_chain(eng, toks, pos)
        assert np.array_equal(a, ra) and np.array_equal(lg, rl), step
        rid, rw = ref.route(B)                    # the last layer's routing of the whole step
        assert np.array_equal(ids[-1], rid) and np.array_equal(w[-1], rw)


def test_layer_chain_matches_oracle(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=32)
    om = O.Model(oracle_cfg(cfg), seed=32)
    seq = om.new_seq()
    eng.reset_kv()
    tok = 7
    for pos in range(20):
        am, lg, _, _ = _layer_chain(eng, [tok], [pos])
        ref_am, ref_lg = seq.forward(tok, pos)
        assert close(lg[0], ref_lg)[0] and am[0] == ref_am, pos
        tok = int(am[0])


def test_layer_chain_with_window_and_tier(cuda):
    """The same calls on an engine with a KV window and a bounded expert
    tier: still the resident engine's logits."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    ref = E.Engine.load(cfg, seed=33)
    eng = E.Engine.load(cfg.replace(kv_window=32, expert_slots=4), seed=33)
    for e_ in (ref, eng):
        e_.reset_kv()
    tok = 3
    for pos in range(60):
        ra, rl = ref.forward(tok, pos)
        am, lg, _, _ = _layer_chain(eng, [tok], [pos])
        assert am[0] == ra and np.array_equal(lg[0], rl), pos
        tok = ra
    assert eng.stats()["kv_pages_evicted"] > 0


def test_layer_calls_reject_bad_arguments(cuda):
    import torch
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=1)
    hid = torch.zeros((1, cfg.n_embd), device="cuda")
    vp = C.c_void_p
    pos = np.zeros(1, np.int32)
    assert eng._lib.sfk_decode_layer_attn(eng.h, cfg.n_layer, pos.ctypes.data_as(vp), 1,
                                          vp(hid.data_ptr())) == L.SFK_ERR_INVALID_ARGUMENT
    assert eng._lib.sfk_decode_layer_moe(eng.h, 0, 0, vp(hid.data_ptr()), None, None) == L.SFK_ERR_INVALID_ARGUMENT
    pos[0] = cfg.n_ctx
    assert eng._lib.sfk_decode_layer_attn(eng.h, 0, pos.ctypes.data_as(vp), 1,
                                          vp(hid.data_ptr())) == L.SFK_ERR_INVALID_ARGUMENT
    assert eng._lib.sfk_lm_head(eng.h, None, 1, None, None) == L.SFK_ERR_INVALID_ARGUMENT
