"""The bounded expert tier on the GPU: an engine whose HBM holds only
`expert_slots` expert bundles (the reference's expert_slots, engine.cpp:
1386-1422) streams the rest from pinned host memory and must decode exactly
what the fully resident engine decodes -- bit-identical logits, since the
kernels and the bytes are the same -- and what the oracle decodes.  Pool
pressure, the stratified and global LRU pools, prefetch on and off, the
batched prefill's passes over the pool and the public generate path are
covered."""
import numpy as np
import pytest

from oracle import oracle as O
from parity_util import oracle_cfg, close

pytestmark = pytest.mark.gpu

KQ = dict(type_ffn_gu=12, type_ffn_down=14, type_attn=14, type_output=14, type_embd=14)


def _decode(eng, prompt, n):
    eng.reset_kv()
    toks, logits = eng.generate(prompt, n, host_loop=True)
    return toks, np.stack(logits)


@pytest.mark.parametrize("slots,kw", [(6, {}), (2, {}), (9, KQ), (31, {})])
def test_tier_decode_bit_identical_to_resident(cuda, slots, kw):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(**kw)
    prompt = np.random.default_rng(slots).integers(0, cfg.n_vocab, 12).tolist()
    ref = E.Engine.load(cfg, seed=11)
    rt, rl = _decode(ref, prompt, 20)
    eng = E.Engine.load(cfg.replace(expert_slots=slots), seed=11)
    t, lg = _decode(eng, prompt, 20)
    assert t == rt
    assert np.array_equal(lg, rl)
    st = eng.stats()
    assert st["pool_slots"] == slots
    steps = len(prompt) + 20 - 1
    acquires = st["pool_hits"] + st["pool_misses"]
    assert acquires >= steps * cfg.n_layer            # every layer's routed set, plus prefetches
    assert st["pool_misses"] > 0
    if slots <= 9:                                     # under pressure (31 slots may hold all it routes)
        assert st["pool_evictions"] > 0
    assert st["h2d_expert_bytes"] % st["pool_misses"] == 0
    assert st["weight_bytes_hbm"] < ref.stats()["weight_bytes_hbm"]


def test_tier_decode_matches_oracle(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(expert_slots=5)
    eng = E.Engine.load(cfg, seed=2)
    om = O.Model(oracle_cfg(cfg), seed=2)
    prompt = np.random.default_rng(2).integers(0, cfg.n_vocab, 10).tolist()
    ref_toks, ref_logits = O.greedy(om, prompt, 16, want_logits=True)
    eng.reset_kv()
    toks, logits = eng.generate(prompt, 16, host_loop=True)
    assert toks == ref_toks
    for a, b in zip(logits, ref_logits):
        assert close(a, b)[0]


def test_tier_device_greedy_loop(cuda):
    """The device-fed greedy loop (sfk_decode_greedy) reads each layer's
    routing back the same way."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 8).tolist()
    ref = E.Engine.load(cfg, seed=4)
    ref.reset_kv()
    want, _ = ref.generate(prompt, 24, host_loop=False)
    eng = E.Engine.load(cfg.replace(expert_slots=3), seed=4)
    eng.reset_kv()
    got, _ = eng.generate(prompt, 24, host_loop=False)
    assert got == want


@pytest.mark.parametrize("env", [{"SFK_POOL_GLOBAL_LRU": "1"}, {"SFK_PREFETCH": "0"}, {"SFK_PREFETCH": "2"},
                                 {"SFK_POOL_GLOBAL_LRU": "1", "SFK_PREFETCH": "2"}])
def test_tier_policies_change_traffic_not_tokens(cuda, monkeypatch, env):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    prompt = np.random.default_rng(6).integers(0, cfg.n_vocab, 10).tolist()
    base = E.Engine.load(cfg.replace(expert_slots=7), seed=6)
    bt, bl = _decode(base, prompt, 16)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    eng = E.Engine.load(cfg.replace(expert_slots=7), seed=6)
    t, lg = _decode(eng, prompt, 16)
    assert t == bt and np.array_equal(lg, bl)
    st = eng.stats()
    if env.get("SFK_PREFETCH") == "0":
        assert st["prefetch_warmed"] == 0
    elif env.get("SFK_PREFETCH") == "2":
        assert st["prefetch_warmed"] > 0 and st["prefetch_used"] <= st["prefetch_warmed"]


@pytest.mark.parametrize("slots", [2, 5])
def test_tier_prefill_passes_bit_identical(cuda, slots):
    """A prompt's routed experts in passes of what the pool holds: the same
    logits as the resident engine's one pass, then the same continuation."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(**KQ)
    prompt = np.random.default_rng(9).integers(0, cfg.n_vocab, 40).tolist()
    ref = E.Engine.load(cfg, seed=9)
    ref.reset_kv()
    ra, rl = ref.prefill(prompt)
    rn = ref.decode_greedy(8)
    eng = E.Engine.load(cfg.replace(expert_slots=slots), seed=9)
    eng.reset_kv()
    a, lg = eng.prefill(prompt)
    assert a == ra and np.array_equal(lg, rl)
    assert np.array_equal(eng.decode_greedy(8), rn)


def test_tier_generate_api(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    prompt = np.random.default_rng(12).integers(0, cfg.n_vocab, 16).tolist()
    ref = E.Engine.load(cfg, seed=12)
    ref.reset_kv()
    want = ref.generate_api(prompt, temperature=0.8, top_k=20, seed=3, max_tokens=12)
    eng = E.Engine.load(cfg.replace(expert_slots=4), seed=12)
    eng.reset_kv()
    assert eng.generate_api(prompt, temperature=0.8, top_k=20, seed=3, max_tokens=12) == want


def test_tier_weights_round_trip(cuda):
    """Expert tensors and bundles put into the pinned store read back as the
    same GGUF bytes, and decode like the resident engine given the same
    bytes."""
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config(**KQ)
    ref = E.Engine.load(cfg, seed=13)
    eng = E.Engine.load(cfg.replace(expert_slots=4), seed=13)
    for tid in (L.T_FFN_GATE_EXPS, L.T_FFN_UP_EXPS, L.T_FFN_DOWN_EXPS):
        for l in range(cfg.n_layer):
            assert np.array_equal(eng.get(tid, l), ref.get(tid, l)), (tid, l)
    # overwrite layer 1's expert 3 through the bundle path, in both engines
    rng = np.random.default_rng(0)
    g = ref.get(L.T_FFN_GATE_EXPS, 1).reshape(cfg.n_expert, -1)
    u = ref.get(L.T_FFN_UP_EXPS, 1).reshape(cfg.n_expert, -1)
    dn = ref.get(L.T_FFN_DOWN_EXPS, 1).reshape(cfg.n_expert, -1)
    bundle = np.concatenate([g[5], u[6], dn[7]])   # another expert's valid bytes
    ref.put_expert(1, 3, bundle)
    eng.put_expert(1, 3, bundle)
    assert np.array_equal(eng.get(L.T_FFN_GATE_EXPS, 1), ref.get(L.T_FFN_GATE_EXPS, 1))
    prompt = rng.integers(0, cfg.n_vocab, 8).tolist()
    rt, rl = _decode(ref, prompt, 12)
    t, lg = _decode(eng, prompt, 12)
    assert t == rt and np.array_equal(lg, rl)


def test_tier_rejects_a_pool_below_one_steps_experts(cuda):
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config()
    with pytest.raises(L.SfkError) as ei:
        E.Engine(cfg.replace(expert_slots=1))
    assert ei.value.status == L.SFK_ERR_INVALID_ARGUMENT
    with pytest.raises(L.SfkError) as ei:
        E.Engine(cfg.replace(expert_slots=3, max_batch=2))   # two tokens route up to 4 experts
    assert ei.value.status == L.SFK_ERR_INVALID_ARGUMENT
    with pytest.raises(L.SfkError) as ei:
        E.Engine(cfg.replace(expert_slots=4, ep_size=2, ep_rank=0))
    assert ei.value.status == L.SFK_ERR_UNSUPPORTED
    # at or above the whole working set: the resident engine
    eng = E.Engine(cfg.replace(expert_slots=cfg.n_layer * cfg.n_expert))
    assert eng.stats()["pool_slots"] == 0


def test_tier_batched_step(cuda):
    """b = 2 sequences per step: both sequences' routed experts held at once."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(max_batch=2)
    ref = E.Engine.load(cfg, seed=15)
    eng = E.Engine.load(cfg.replace(expert_slots=4), seed=15)
    rng = np.random.default_rng(15)
    for e_ in (ref, eng):
        e_.reset_kv()
    for pos in range(10):
        toks = rng.integers(0, cfg.n_vocab, 2)
        ra, rl = ref.forward_batch(toks, [pos, pos])
        a, lg = eng.forward_batch(toks, [pos, pos])
        assert np.array_equal(a, ra) and np.array_equal(lg, rl), pos
