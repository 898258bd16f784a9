"""GPU parity of the whole decode step (engine::Engine::forward) against the
CPU oracle, driven the way the reference's own oracle test drives libllama
(tests/test_engine_oracle.cpp:145-236: prompt one token per position, then
greedy tokens): identical greedy sequences, logits within 1e-3 relative L2 and
1e-2 max-abs (the reference's own engine-vs-libllama
gate is 1e-3 max-abs for F32, 2e-2 for Q8_0, test_engine_oracle.cpp:136,539).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


from parity_util import oracle_cfg as _oracle_cfg, close as _close  # noqa: E402


def _run_parity(cfg, seed, prompt, n_gen, oracle_model=None):
    from strataflow_b200 import engine as E
    eng = E.Engine.load(cfg, seed=seed)
    om = oracle_model or O.Model(_oracle_cfg(cfg), seed=seed)
    ref_toks, ref_logits = O.greedy(om, prompt, n_gen, want_logits=True)
    toks, logits = eng.generate(prompt, n_gen, host_loop=True)
    worst = (0.0, 0.0)
    for i, (a, b) in enumerate(zip(logits, ref_logits)):
        ok, rel, mx = _close(a, b)
        worst = (max(worst[0], rel), max(worst[1], mx))
        assert ok, (i, rel, mx)
    assert toks == ref_toks
    return eng, om, toks, worst


def test_synth_weights_bit_identical_to_oracle(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(n_layer=2, type_ffn_gu=12, type_ffn_down=12, type_attn=14, type_output=14, type_embd=14)
    eng = E.Engine.load(cfg, seed=3)
    om = O.Model(_oracle_cfg(cfg), seed=3)
    for tid, layer in om.tensors():
        got = eng.get(tid, layer)
        ref, _, _ = om.tensor(tid, layer)
        assert np.array_equal(got, ref), (tid, layer)


def test_weights_put_get_roundtrip(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(n_layer=1)
    om = O.Model(_oracle_cfg(cfg), seed=9)
    tensors = []
    for tid, l in om.tensors():
        data, qtype, ne = om.tensor(tid, l)
        tensors.append((tid, l, qtype, ne, data))
    eng = E.Engine.load(cfg, tensors=tensors)
    for tid, l in om.tensors():
        assert np.array_equal(eng.get(tid, l), om.tensor(tid, l)[0])


def test_expert_bundle_put(cuda):
    """A .strata expert bundle (gate|up|down, strata_format.h:122-130) lands in
    the stacked tensors at that expert's slice."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(n_layer=1)
    eng = E.Engine.load(cfg, seed=1)
    om = O.Model(_oracle_cfg(cfg), seed=2)
    g, _, _ = om.tensor(O.T_FFN_GATE_EXPS, 0)
    u, _, _ = om.tensor(O.T_FFN_UP_EXPS, 0)
    dn, _, _ = om.tensor(O.T_FFN_DOWN_EXPS, 0)
    E_ = cfg.n_expert
    gl, dl = g.size // E_, dn.size // E_
    e = 5
    eng.put_expert(0, e, np.concatenate([g[e * gl:(e + 1) * gl], u[e * gl:(e + 1) * gl], dn[e * dl:(e + 1) * dl]]))
    assert np.array_equal(eng.get(O.T_FFN_GATE_EXPS, 0)[e * gl:(e + 1) * gl], g[e * gl:(e + 1) * gl])
    assert np.array_equal(eng.get(O.T_FFN_DOWN_EXPS, 0)[e * dl:(e + 1) * dl], dn[e * dl:(e + 1) * dl])


def test_tiny_q8_0_greedy_parity(cuda):
    """16-token prompt (seed 1), 64 greedy tokens, context 80."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    prompt = np.random.default_rng(1).integers(0, cfg.n_vocab, 16).tolist()
    eng, om, toks, worst = _run_parity(cfg, 0, prompt, 64)
    assert len(toks) == 64


def test_tiny_kquant_greedy_parity(cuda):
    """K-quant variant (the reference's make_kquant_moe_gguf shape family):
    Q4_K experts, Q6_K attention / embedding / output."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(type_ffn_gu=12, type_ffn_down=12, type_attn=14, type_output=14, type_embd=14)
    prompt = np.random.default_rng(2).integers(0, cfg.n_vocab, 12).tolist()
    _run_parity(cfg, 7, prompt, 24)


def test_tiny_f16_kv_greedy_parity(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(kv_type=1)
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab, 10).tolist()
    _run_parity(cfg, 4, prompt, 20)


def test_device_greedy_loop_matches_host_loop(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=0)
    prompt = np.random.default_rng(1).integers(0, cfg.n_vocab, 16).tolist()
    host, _ = eng.generate(prompt, 32, host_loop=True)
    eng.reset_kv()
    dev, _ = eng.generate(prompt, 32, host_loop=False)
    assert dev == host


def test_batched_step_equals_single_sequences(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(max_batch=4, n_layer=2)
    eng = E.Engine.load(cfg, seed=5)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, cfg.n_vocab, 6).tolist() for _ in range(3)]
    # batched: 3 sequences stepped together
    for p in range(6):
        am_b, lg_b = eng.forward_batch([pr[p] for pr in prompts], [p, p, p])
    # single: each sequence alone on a fresh engine
    for s in range(3):
        e1 = E.Engine.load(cfg, seed=5)
        for p in range(6):
            am1, lg1 = e1.forward(prompts[s][p], p)
        assert am1 == am_b[s]
        assert np.abs(lg1 - lg_b[s]).max() <= 1e-6 * np.abs(lg1).max()
    # and the device greedy loop over the batch continues every sequence
    toks = eng.decode_greedy(5, 3)
    assert toks.shape == (5, 3) and (toks[0] == am_b).all()


@pytest.mark.parametrize("kw", [dict(n_layer=2), dict(n_layer=2, type_ffn_gu=12, type_ffn_down=14, type_attn=14)])
def test_router_kernel_equals_fused_routing(cuda, monkeypatch, kw):
    """Steps of more than two tokens route with the router kernel; forcing
    the gate/up kernel's fused routing prologue for them instead
    (SFK_FUSED_ROUTE_MAX_B) gives the same routing and logits bit for bit."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(max_batch=4, **kw)
    rng = np.random.default_rng(7)
    steps = [(rng.integers(0, cfg.n_vocab, 3), [p, p + 2, p + 5]) for p in range(8)]

    def run():
        eng = E.Engine.load(cfg, seed=9)
        eng.reset_kv()
        out = []
        for toks, pos in steps:
            am, lg = eng.forward_batch(toks, pos)
            ids, w = eng.route(3)
            out.append((am, lg, ids, w))
        return out

    kern = run()
    monkeypatch.setenv("SFK_FUSED_ROUTE_MAX_B", "16")
    fused = run()
    for (a0, l0, i0, w0), (a1, l1, i1, w1) in zip(kern, fused):
        assert np.array_equal(a0, a1) and np.array_equal(i0, i1)
        assert np.array_equal(w0.view(np.uint32), w1.view(np.uint32))
        assert np.array_equal(l0.view(np.uint32), l1.view(np.uint32))


def test_mixtral_width_two_layer_parity(cuda):
    """Mid-size model: every Mixtral-8x7B width (d 4096, 32q/8kv x 128,
    8 experts top-2, FFN 14336, vocab 32000, RoPE 1e6, Q4_K experts, Q6_K
    trunk, f16 KV) with 2 layers, 8-token prompt + 8 greedy tokens."""
    from strataflow_b200 import engine as E
    cfg = E.mixtral_config(n_layer=2, n_ctx=64)
    prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 8).tolist()
    eng, om, toks, worst = _run_parity(cfg, 4, prompt, 8)
    # spot-check generator equality at full width too
    for tid, layer in [(O.T_ATTN_Q, 1), (O.T_FFN_DOWN_EXPS, 0), (O.T_OUTPUT, 0)]:
        assert np.array_equal(eng.get(tid, layer), om.tensor(tid, layer)[0])


def test_forward_rejects_out_of_range_inputs(cuda):
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config(n_layer=1, n_ctx=16)
    eng = E.Engine.load(cfg, seed=0)
    with pytest.raises(L.SfkError):
        eng.forward(cfg.n_vocab, 0)
    with pytest.raises(L.SfkError):
        eng.forward(1, cfg.n_ctx)
    eng.forward(1, 0)
    with pytest.raises(L.SfkError):
        eng.decode_greedy(cfg.n_ctx, 1)   # would run past n_ctx
    am, _ = eng.forward(2, 1)             # the engine still works afterwards
    assert 0 <= am < cfg.n_vocab


def test_kernel_timing_entry_point(cuda, monkeypatch):
    """The launch chain's per-kernel timing (the persistent step kernel is
    switched off so the step runs as the chain of 2 + 5L launches)."""
    from strataflow_b200 import engine as E
    import ctypes as C
    monkeypatch.setenv("SFK_PERSISTENT", "0")
    cfg = E.tiny_config(n_layer=2)
    eng = E.Engine.load(cfg, seed=0)
    eng.forward(3, 0)
    ms = (C.c_float * 8)()
    from strataflow_b200 import lib as L
    L.check(eng._lib.sfk_time_kernels(eng.h, 1, 4, ms, 8))
    # up to 64 experts the gate/up kernel routes in its prologue: no router
    # kernel, and its timing slot reads 0
    router = 4  # K_ROUTER in the kernel-class order (embed, qkv, attn, o, router, gate/up, down, lm_head)
    assert ms[router] == 0.0
    assert all(v > 0 for i, v in enumerate(ms) if i != router)
    assert eng.stats()["kernels_per_step"] == 2 + 5 * cfg.n_layer


def test_standalone_router_kernel_parity(cuda, monkeypatch):
    """SFK_ROUTER_KERNEL=1: routing runs in its own kernel before gate/up
    (launch chain)."""
    from strataflow_b200 import engine as E
    monkeypatch.setenv("SFK_ROUTER_KERNEL", "1")
    monkeypatch.setenv("SFK_PERSISTENT", "0")
    cfg = E.tiny_config(n_layer=2, n_expert=72, n_expert_used=4)
    prompt = np.random.default_rng(8).integers(0, cfg.n_vocab, 8).tolist()
    eng, om, toks, worst = _run_parity(cfg, 9, prompt, 12)
    assert eng.stats()["kernels_per_step"] == 2 + 6 * cfg.n_layer


@pytest.mark.parametrize("n_expert,k", [(72, 4), (160, 2)])
def test_many_experts_fused_routing_parity(cuda, n_expert, k, monkeypatch):
    """Routing inside gate/up for larger expert counts (launch chain): 72
    experts fit the ring (router staged in every CTA); 160 do not (each CTA
    scores a few logits and the CTAs exchange them)."""
    from strataflow_b200 import engine as E
    monkeypatch.setenv("SFK_PERSISTENT", "0")
    cfg = E.tiny_config(n_layer=2, n_expert=n_expert, n_expert_used=k)
    prompt = np.random.default_rng(n_expert).integers(0, cfg.n_vocab, 8).tolist()
    eng, om, toks, worst = _run_parity(cfg, 9, prompt, 12)
    assert eng.stats()["kernels_per_step"] == 2 + 5 * cfg.n_layer


@pytest.mark.parametrize("kw", [dict(), dict(type_ffn_gu=12, type_ffn_down=12, type_attn=14, type_output=14,
                                             type_embd=14, kv_type=1)])
def test_persistent_step_matches_launch_chain(cuda, monkeypatch, kw):
    """The persistent step kernel (one cooperative launch per step) and the
    launch chain produce the same greedy tokens and logits within float
    rounding of each other, and both match the oracle (checked by
    _run_parity on the persistent path)."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(n_layer=3, **kw)
    prompt = np.random.default_rng(12).integers(0, cfg.n_vocab, 10).tolist()
    monkeypatch.setenv("SFK_PERSISTENT", "1")
    eng, om, toks, worst = _run_parity(cfg, 21, prompt, 16)
    assert eng.stats()["kernels_per_step"] == 1
    monkeypatch.setenv("SFK_PERSISTENT", "0")
    chain = E.Engine.load(cfg, seed=21)
    toks_c, logits_c = chain.generate(prompt, 16, host_loop=True)
    assert chain.stats()["kernels_per_step"] == 2 + 5 * cfg.n_layer
    assert toks_c == toks
    eng.reset_kv()
    toks_p, logits_p = eng.generate(prompt, 16, host_loop=True)
    for a, b in zip(logits_p, logits_c):
        assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()
