"""The public generate path (GPU): sfk_generate -- the reference's sf_generate
(src/api/strataflow_api.cpp:308-335) with every prompt token prefilled -- and
the device sampler of its sf_sampling_params (include/strataflow/
strataflow.h:193-199), against the CPU oracle (sfo_sample and the oracle's
token-by-token drive)."""
import numpy as np
import pytest

from oracle import oracle as O
from parity_util import oracle_cfg

pytestmark = pytest.mark.gpu

CASES = [  # temperature, top_k, top_p
    (1.0, 0, 1.0), (0.7, 0, 1.0), (0.8, 40, 1.0), (1.0, 0, 0.9), (0.6, 50, 0.95), (1.3, 5, 0.5),
    (0.9, 1, 1.0), (2.0, 0, 0.3),
]


@pytest.mark.parametrize("V", [4096, 32000, 160000])
def test_sampler_matches_oracle(cuda, V):
    """The same token as the oracle for every (temperature, top_k, top_p,
    seed, step) tried, on logits of three vocabulary sizes."""
    import torch
    from strataflow_b200 import ops
    rng = np.random.default_rng(V)
    for trial in range(6):
        logits = (rng.standard_normal(V) * (1.0 + trial)).astype(np.float32)
        d = torch.from_numpy(logits).cuda()
        for (T, k, p) in CASES:
            for step in (0, 3):
                seed = 1000 * trial + step
                got = ops.sample_logits(d, T, top_k=k, top_p=p, seed=seed, step=step)
                ref = O.sample(logits, T, top_k=k, top_p=p, seed=seed, step=step)
                assert got == ref, (V, trial, T, k, p, step, got, ref)


def test_sampler_ties_and_top_k_one(cuda):
    """Tied probabilities at the top-k and nucleus cut-offs enter by index;
    top_k = 1 is the first maximum."""
    import torch
    from strataflow_b200 import ops
    logits = np.zeros(1000, np.float32)
    logits[[7, 70, 700]] = 3.0    # three tied maxima
    logits[[5, 50, 500]] = 2.0    # three tied seconds
    d = torch.from_numpy(logits).cuda()
    for (T, k, p) in [(1.0, 1, 1.0), (1.0, 2, 1.0), (1.0, 4, 1.0), (1.0, 0, 0.2), (0.5, 5, 0.7)]:
        for seed in range(12):
            assert ops.sample_logits(d, T, top_k=k, top_p=p, seed=seed) == \
                O.sample(logits, T, top_k=k, top_p=p, seed=seed)
    assert ops.sample_logits(d, 1.0, top_k=1) == 7


def test_sampler_distribution(cuda):
    """Draws over many steps follow the kept distribution (chi-square-like
    bound on a 6-token vocabulary)."""
    import torch
    from strataflow_b200 import ops
    logits = np.log(np.array([0.4, 0.3, 0.15, 0.1, 0.04, 0.01], np.float32))
    d = torch.from_numpy(logits).cuda()
    n = 2000
    counts = np.bincount([ops.sample_logits(d, 1.0, seed=11, step=s) for s in range(n)], minlength=6)
    expect = np.exp(logits) / np.exp(logits).sum() * n
    assert np.all(np.abs(counts - expect) < 5 * np.sqrt(expect) + 3), (counts, expect)
    # top_p 0.7 keeps the first two tokens only
    c2 = np.bincount([ops.sample_logits(d, 1.0, top_p=0.7, seed=5, step=s) for s in range(400)], minlength=6)
    assert c2[2:].sum() == 0 and c2[0] > 0 and c2[1] > 0


def _oracle_generate(om, prompt, n, T=0.0, k=0, p=1.0, seed=0, eos=-1):
    """The generate drive on the oracle: prompt in the prefill's fp32 order,
    then sample / argmax each step's logits, stop before eos."""
    seq = om.new_seq()
    om.set_fp32_mode(2)
    last = None
    for pos, t in enumerate(prompt):
        _, last = seq.forward(t, pos)
    om.set_fp32_mode(int(om.cfg.fp32_mode))
    out = []
    pos = len(prompt)
    for i in range(n):
        tok = O.sample(last, T, top_k=k, top_p=p, seed=seed, step=i)
        if tok == eos:
            break
        out.append(tok)
        if i + 1 == n:
            break
        _, last = seq.forward(tok, pos)
        pos += 1
    return out


def test_generate_greedy_matches_oracle(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=3)
    om = O.Model(oracle_cfg(cfg), seed=3)
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab, 20).tolist()
    eng.reset_kv()
    got = eng.generate_api(prompt, max_tokens=16)
    assert got == _oracle_generate(om, prompt, 16)


def test_generate_sampled_matches_oracle(cuda):
    from strataflow_b200 import engine as E
    cfg = E.tiny_config(type_ffn_gu=12, type_ffn_down=12, type_attn=14, type_output=14, type_embd=14, kv_type=1)
    eng = E.Engine.load(cfg, seed=8)
    om = O.Model(oracle_cfg(cfg), seed=8)
    prompt = np.random.default_rng(8).integers(0, cfg.n_vocab, 24).tolist()
    for (T, k, p, seed) in [(0.8, 40, 0.95, 7), (1.2, 0, 1.0, 3)]:
        eng.reset_kv()
        got = eng.generate_api(prompt, temperature=T, top_k=k, top_p=p, seed=seed, max_tokens=20)
        assert got == _oracle_generate(om, prompt, 20, T, k, p, seed), (T, k, p, seed)


def test_generate_stops(cuda):
    """eos is not emitted; the callback stops the loop; max_tokens caps it;
    the prompt continues at the sequence's next position."""
    from strataflow_b200 import engine as E
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=4)
    prompt = np.random.default_rng(4).integers(0, cfg.n_vocab, 12).tolist()
    eng.reset_kv()
    full = eng.generate_api(prompt, max_tokens=10)
    assert len(full) == 10
    eng.reset_kv()
    assert eng.generate_api(prompt, max_tokens=10, eos_token=full[3]) == full[:full.index(full[3])]
    eng.reset_kv()
    seen = []
    got = eng.generate_api(prompt, max_tokens=10, callback=lambda t: seen.append(t) or len(seen) >= 4)
    assert got == full[:4] and seen == full[:4]
    # a second call continues the same sequence, as a session would: the
    # first call fed the prompt (prefill) and all its tokens but the last
    # (decode steps); the second prefills its prompt after them
    eng.reset_kv()
    a = eng.generate_api(prompt, max_tokens=3)
    b = eng.generate_api(prompt[:5], max_tokens=3)
    om = O.Model(oracle_cfg(cfg), seed=4)
    seq = om.new_seq()
    pos = 0
    for toks, mode in ((prompt, 2), (a[:-1], 0), (prompt[:5], 2)):
        om.set_fp32_mode(mode)
        for t in toks:
            _, last = seq.forward(t, pos)
            pos += 1
    om.set_fp32_mode(0)
    ref = []
    for i in range(3):
        tok = O.sample(last, 0.0)
        ref.append(tok)
        if i < 2:
            _, last = seq.forward(tok, pos)
            pos += 1
    assert b == ref


def test_generate_rejects_bad_arguments(cuda):
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    cfg = E.tiny_config()
    eng = E.Engine.load(cfg, seed=1)
    with pytest.raises(L.SfkError):
        eng.generate_api([], max_tokens=4)
    with pytest.raises(L.SfkError):
        eng.generate_api([1] * (cfg.n_ctx + 1), max_tokens=4)
    eng.reset_kv()
    assert len(eng.generate_api([1, 2, 3], max_tokens=4)) == 4
