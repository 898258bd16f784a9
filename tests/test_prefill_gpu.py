"""GPU parity of the batched prompt prefill (sfk_prefill) against the CPU
oracle.

The reference feeds a prompt one position per Engine::forward call
(tests/test_engine_oracle.cpp:182-187); sfk_prefill runs every layer over the
whole prompt at once on the tensor cores.  The oracle drives the reference's
pattern (prompt token by token, then greedy tokens); the engine prefills the
prompt in one call and continues token by token.  The prefill's GEMMs add a
row's 256-column blocks in order (ggml's generic per-block fp32 order), the
decode kernels in their own unit order, so the oracle computes the prompt
tokens in the per-block order and the generated tokens in the decode order
(prompt_fp32_mode=2).  The two orders alone move a small random model's
logits by ~7e-3 relative L2 (activation codes re-quantized layer after
layer), which is why the order is matched rather than the tolerance widened.
Gates: the last prompt token's logits and every decode step's logits within
1e-3 relative L2 and 1e-2 max-abs, identical greedy tokens."""
import numpy as np
import pytest

from oracle import oracle as O
from parity_util import close, oracle_cfg, oracle_from_engine

pytestmark = pytest.mark.gpu


def _prefill_then_decode(eng, prompt, n_gen, pos0=0):
    """Prefill the prompt, then n_gen greedy tokens one forward at a time:
    (generated tokens, [last prompt logits] + each step's logits)."""
    am, last = eng.prefill(prompt, pos0=pos0)
    logits = [last]
    toks = []
    pos = pos0 + len(prompt)
    for _ in range(n_gen):
        toks.append(am)
        am, lg = eng.forward(am, pos)
        logits.append(lg)
        pos += 1
    return toks, logits


def _check(eng, om, prompt, n_gen):
    ref_toks, ref_logits = O.greedy(om, prompt, n_gen, want_logits=True, prompt_fp32_mode=2)
    eng.reset_kv()
    toks, logits = _prefill_then_decode(eng, prompt, n_gen)
    worst = (0.0, 0.0)
    for i, (a, b) in enumerate(zip(logits, ref_logits)):
        ok, rel, mx = close(a, b)
        worst = (max(worst[0], rel), max(worst[1], mx))
        assert ok, (i, rel, mx)
    assert toks == ref_toks
    return worst


def test_tiny_q8_0_prefill(cuda):
    """configs[0] (Q8_0 everywhere, F32 KV): 16-token prompt, 16 greedy tokens."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=1)
    om = O.Model(oracle_cfg(cfg), seed=1)
    prompt = np.random.default_rng(1).integers(0, cfg.n_vocab, 16).tolist()
    _check(eng, om, prompt, 16)


def test_tiny_kquant_prefill_ragged(cuda):
    """K-quant weights (Q4_K experts, Q6_K trunk), f16 KV; a 70-token prompt
    (one full 64-row tile and a ragged one; expert groups of uneven size)."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(type_ffn_gu=12, type_ffn_down=12, type_attn=14, type_output=14, type_embd=14, kv_type=1)
    eng = E.Engine.load(cfg, seed=5)
    om = O.Model(oracle_cfg(cfg), seed=5)
    prompt = np.random.default_rng(5).integers(0, cfg.n_vocab, 70).tolist()
    _check(eng, om, prompt, 8)


def test_prefill_continues_at_pos0(cuda):
    """Two prefills (positions 0..36, then 37..56) equal one prompt of 57."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(type_ffn_gu=12, type_ffn_down=12, type_attn=14, type_output=14, type_embd=14)
    eng = E.Engine.load(cfg, seed=6)
    om = O.Model(oracle_cfg(cfg), seed=6)
    prompt = np.random.default_rng(6).integers(0, cfg.n_vocab, 57).tolist()
    ref_toks, ref_logits = O.greedy(om, prompt, 4, want_logits=True, prompt_fp32_mode=2)
    eng.reset_kv()
    eng.prefill(prompt[:37])
    toks, logits = _prefill_then_decode(eng, prompt[37:], 4, pos0=37)
    for i, (a, b) in enumerate(zip(logits, ref_logits)):
        ok, rel, mx = close(a, b)
        assert ok, (i, rel, mx)
    assert toks == ref_toks


def test_prefill_then_device_greedy(cuda):
    """The device greedy loop continues from the prefill's argmax and next
    position (the state a token-by-token prompt leaves)."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=2)
    om = O.Model(oracle_cfg(cfg), seed=2)
    prompt = np.random.default_rng(2).integers(0, cfg.n_vocab, 24).tolist()
    ref_toks, _ = O.greedy(om, prompt, 24, prompt_fp32_mode=2)
    eng.reset_kv()
    eng.prefill(prompt, want_logits=False)
    toks = eng.decode_greedy(24, 1)[:, 0].tolist()
    assert toks == ref_toks


def test_mixtral_width_prefill(cuda):
    """Mixtral-8x7B width at 2 layers (Q4_K experts, Q6_K trunk, F32 router,
    f16 paged KV): a 72-token prompt prefilled at once against the oracle fed
    token by token, then 4 greedy tokens."""
    from strataflow_b200 import engine as E
    cfg = E.mixtral_config(n_layer=2, n_ctx=96)
    eng = E.Engine.load(cfg, seed=4)
    om = oracle_from_engine(eng)
    prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 72).tolist()
    _check(eng, om, prompt, 4)


def test_mixtral_width_prefill_three_tiles(cuda):
    """130 prompt tokens (three 64-row activation tiles, a ragged last one; 260
    routed pairs in uneven expert groups) at Mixtral width, 2 layers."""
    from strataflow_b200 import engine as E
    cfg = E.mixtral_config(n_layer=2, n_ctx=160)
    eng = E.Engine.load(cfg, seed=7)
    om = oracle_from_engine(eng)
    prompt = np.random.default_rng(7).integers(0, cfg.n_vocab, 130).tolist()
    _check(eng, om, prompt, 2)


def test_prefill_rejects_bad_arguments(cuda):
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=1)
    with pytest.raises(L.SfkError):
        eng.prefill([], pos0=0)
    with pytest.raises(L.SfkError):
        eng.prefill([1, 2, 3], pos0=cfg.n_ctx - 2)
    with pytest.raises(L.SfkError):
        eng.prefill([1, cfg.n_vocab], pos0=0)
    # the engine is still usable
    eng.reset_kv()
    eng.prefill([1, 2, 3])
