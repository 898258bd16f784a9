"""The KV window on the GPU (kv_window: the reference's KvStore ring window
and lossless cold store, src/kv/kv_store.h:30-95, engine.cpp:1633-1762): a
sequence keeps only its last kv_window tokens' pages in HBM, the older pages
go to pinned host memory and come back for every layer's attention.  The
attention sees the same keys and values in the same order as with the whole
context resident, so the logits are bit-identical to the resident engine's,
past many evictions, in the decode loop, the host-buffer step, batched steps
and the chunked prefill."""
import numpy as np
import pytest

from oracle import oracle as O
from parity_util import oracle_cfg, close

pytestmark = pytest.mark.gpu

KQ = dict(type_ffn_gu=12, type_ffn_down=14, type_attn=14, type_output=14, type_embd=14, kv_type=1)


def _decode(eng, prompt, n, host_loop=True):
    eng.reset_kv()
    toks, logits = eng.generate(prompt, n, host_loop=host_loop)
    return toks, (np.stack(logits) if logits is not None and len(logits) else None)


@pytest.mark.parametrize("window,kw", [(32, {}), (48, KQ), (40, {})])
def test_window_decode_bit_identical_to_resident(cuda, window, kw):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(**kw)
    prompt = np.random.default_rng(window).integers(0, cfg.n_vocab, 9).tolist()
    n = cfg.n_ctx - len(prompt)
    ref = E.Engine.load(cfg, seed=21)
    rt, rl = _decode(ref, prompt, n)
    eng = E.Engine.load(cfg.replace(kv_window=window), seed=21)
    t, lg = _decode(eng, prompt, n)
    assert t == rt
    assert np.array_equal(lg, rl)
    st = eng.stats()
    pages = (window + 15) // 16
    assert st["kv_window_pages"] == pages
    assert st["kv_pages_evicted"] == (cfg.n_ctx - 1) // 16 + 1 - pages
    assert st["kv_staged_bytes"] > 0


def test_window_bounds_hbm_kv(cuda):
    """HBM holds the window's pages of every layer plus one layer's worth of
    staging (twice), not the whole context of every layer."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(n_ctx=2048, n_layer=8)
    full = E.Engine(cfg).stats()["kv_bytes_hbm"]
    win = E.Engine(cfg.replace(kv_window=64)).stats()["kv_bytes_hbm"]
    assert win < full / 2


def test_window_device_loop_and_oracle(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(kv_window=32)
    eng = E.Engine.load(cfg, seed=5)
    om = O.Model(oracle_cfg(cfg), seed=5)
    prompt = np.random.default_rng(5).integers(0, cfg.n_vocab, 6).tolist()
    ref_toks, ref_logits = O.greedy(om, prompt, 60, want_logits=True)
    eng.reset_kv()
    toks, logits = eng.generate(prompt, 60, host_loop=True)
    assert toks == ref_toks
    for a, b in zip(logits, ref_logits):
        assert close(a, b)[0]
    eng.reset_kv()
    dev, _ = eng.generate(prompt, 60, host_loop=False)
    assert dev == toks


def test_window_batched_sequences_at_different_positions(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(max_batch=2, **KQ)
    ref = E.Engine.load(cfg, seed=7)
    eng = E.Engine.load(cfg.replace(kv_window=32), seed=7)
    rng = np.random.default_rng(7)
    for e_ in (ref, eng):
        e_.reset_kv()
    # sequence 1 starts 11 positions later than sequence 0
    for i in range(cfg.n_ctx - 11):
        toks = rng.integers(0, cfg.n_vocab, 2)
        pos = [i + 11, i]
        ra, rl = ref.forward_batch(toks, pos)
        a, lg = eng.forward_batch(toks, pos)
        assert np.array_equal(a, ra) and np.array_equal(lg, rl), i


@pytest.mark.parametrize("window", [32, 64])
def test_window_prefill_chunks_bit_identical(cuda, window):
    """A prompt longer than the window: prefilled in chunks that fit it, with
    the earlier pages evicted between chunks -- the same logits as the
    resident engine's prefill, and the same continuation."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(**KQ)
    prompt = np.random.default_rng(window).integers(0, cfg.n_vocab, 70).tolist()
    ref = E.Engine.load(cfg, seed=8)
    ref.reset_kv()
    ra, rl = ref.prefill(prompt)
    rn = ref.decode_greedy(8)
    eng = E.Engine.load(cfg.replace(kv_window=window), seed=8)
    eng.reset_kv()
    a, lg = eng.prefill(prompt)
    assert a == ra and np.array_equal(lg, rl)
    assert np.array_equal(eng.decode_greedy(8), rn)


def test_window_with_bounded_expert_tier_and_generate(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab, 30).tolist()
    ref = E.Engine.load(cfg, seed=3)
    ref.reset_kv()
    want = ref.generate_api(prompt, temperature=0.7, top_k=30, seed=9, max_tokens=40)
    eng = E.Engine.load(cfg.replace(kv_window=32, expert_slots=5), seed=3)
    eng.reset_kv()
    assert eng.generate_api(prompt, temperature=0.7, top_k=30, seed=9, max_tokens=40) == want
    st = eng.stats()
    assert st["kv_pages_evicted"] > 0 and st["pool_misses"] > 0


def test_window_rejections(cuda):
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config()
    with pytest.raises(L.SfkError) as ei:
        E.Engine(cfg.replace(kv_window=16))            # one page
    assert ei.value.status == L.SFK_ERR_INVALID_ARGUMENT
    with pytest.raises(L.SfkError) as ei:
        E.Engine(cfg.replace(kv_window=32, ep_size=2, ep_rank=0))
    assert ei.value.status == L.SFK_ERR_UNSUPPORTED
    assert E.Engine(cfg.replace(kv_window=cfg.n_ctx)).stats()["kv_window_pages"] == 0
    eng = E.Engine.load(cfg.replace(kv_window=32), seed=1)
    eng.reset_kv()
    for pos in range(50):
        eng.forward(1, pos)
    # positions 0..15 (page 0) and 16..31 (page 1) have left the window
    with pytest.raises(L.SfkError) as ei:
        eng.forward(1, 20)
    assert ei.value.status == L.SFK_ERR_INVALID_ARGUMENT
    eng.forward(1, 40)                                  # a page still in the window may be rewritten
    with pytest.raises(L.SfkError):
        eng.prefill([1, 2, 3], pos0=10)
    eng.reset_kv()                                      # a reset brings every page back
    eng.forward(1, 0)
