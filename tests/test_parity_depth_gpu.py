"""Oracle parity at the benchmarked shapes (GPU).

* the full 32-layer Mixtral-8x7B shape of the decode benchmark (configs[3]:
  Q4_K experts, Q6_K trunk, F32 router, f16 paged KV, seed 4): a 32-token
  prompt fed one position per step, then 16 greedy tokens, against the CPU
  oracle holding the same weights;
* batch 8 at Mixtral width (2 layers): eight sequences stepped together by
  sfk_forward_batch, each checked against its own oracle sequence, then
  continued by the device greedy loop;
* the ~1T shape's width on one GPU (configs[4]: d 7168, 64 query / 8 KV
  heads of 128, 384 experts top-8, FFN 2048, vocab 160000, Q8_0 trunk, Q4_K
  experts) at 2 layers.

Tolerances are the north star's: identical greedy tokens, logits within 1e-3
relative L2 and 1e-2 max-abs (the reference's own engine gates are token
equality and 1e-3 / 2e-2 max-abs, tests/test_engine_oracle.cpp:133,136,207,539).
The oracle receives the engine's resident weights (sfk_weights_get); that the
device generator writes the oracle generator's bytes is checked by
test_engine_gpu.py."""
import numpy as np
import pytest

from oracle import oracle as O
from parity_util import close, oracle_from_engine

pytestmark = pytest.mark.gpu


def _check_seq(eng, om, prompt, n_gen):
    ref_toks, ref_logits = O.greedy(om, prompt, n_gen, want_logits=True)
    toks, logits = eng.generate(prompt, n_gen, host_loop=True)
    worst = (0.0, 0.0)
    for i, (a, b) in enumerate(zip(logits, ref_logits)):
        ok, rel, mx = close(a, b)
        worst = (max(worst[0], rel), max(worst[1], mx))
        assert ok, (i, rel, mx)
    assert toks == ref_toks
    return toks, worst


@pytest.mark.parametrize("persistent", ["1", "0"])
def test_mixtral_full_depth_greedy_parity(cuda, monkeypatch, persistent):
    """The benchmark's model at full depth: 32 layers, 32-token prompt, 16
    greedy tokens, every step's logits against the oracle; on the persistent
    step kernel (the benchmarked path) and on the launch chain."""
    from strataflow_b200 import engine as E
    monkeypatch.setenv("SFK_PERSISTENT", persistent)
    cfg = E.mixtral_config(n_ctx=64)
    eng = E.Engine.load(cfg, seed=4)
    try:
        om = oracle_from_engine(eng)
        prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 32).tolist()
        toks, worst = _check_seq(eng, om, prompt, 16)
        assert eng.stats()["kernels_per_step"] == (1 if persistent == "1" else 2 + 5 * cfg.n_layer)
        print("mixtral 32L persistent=%s worst rel/max-abs" % persistent, worst)
        # the device greedy loop continues the same sequence as the host loop
        eng.reset_kv()
        dev, _ = eng.generate(prompt, 16, host_loop=False)
        assert dev == toks
    finally:
        eng.close()


def test_mixtral_width_batch8_parity(cuda):
    """b=8 at Mixtral width: eight sequences in one step, each against its own
    oracle sequence, then four device greedy steps of the whole batch."""
    from strataflow_b200 import engine as E
    B, P, n_dev = 8, 6, 4
    cfg = E.mixtral_config(n_layer=2, n_ctx=32, max_batch=B)
    eng = E.Engine.load(cfg, seed=4)
    try:
        om = oracle_from_engine(eng)
        rng = np.random.default_rng(40)
        prompts = [rng.integers(0, cfg.n_vocab, P).tolist() for _ in range(B)]
        seqs = [om.new_seq() for _ in range(B)]
        for p in range(P):
            am, lg = eng.forward_batch([pr[p] for pr in prompts], [p] * B)
            for s in range(B):
                ram, rlg = seqs[s].forward(prompts[s][p], p)
                ok, rel, mx = close(lg[s], rlg)
                assert ok, (p, s, rel, mx)
                assert am[s] == ram, (p, s)
        toks = eng.decode_greedy(n_dev, B)
        assert (toks[0] == am).all()
        for s in range(B):   # the oracle follows the device loop's tokens
            tok = int(toks[0, s])
            for i in range(n_dev):
                ram, _ = seqs[s].forward(tok, P + i)
                if i + 1 < n_dev:
                    assert int(toks[i + 1, s]) == ram, (i, s)
                    tok = ram
    finally:
        eng.close()


def test_trillion_width_two_layer_parity(cuda):
    """The ~1T shape's every width (d 7168, 64 heads x 128 over a 8192-wide
    attention, 8 KV heads, 384 experts top-8, FFN 2048, vocab 160000, Q8_0
    trunk, Q4_K experts) at 2 layers on one GPU: 8-token prompt, 8 greedy
    tokens."""
    from strataflow_b200 import engine as E
    cfg = E.trillion_config(n_layer=2, n_ctx=32)
    eng = E.Engine.load(cfg, seed=5)
    try:
        om = oracle_from_engine(eng)
        prompt = np.random.default_rng(5).integers(0, cfg.n_vocab, 8).tolist()
        toks, worst = _check_seq(eng, om, prompt, 8)
        print("1T-width 2L worst rel/max-abs", worst)
    finally:
        eng.close()
