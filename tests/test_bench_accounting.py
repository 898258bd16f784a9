"""The benchmark's byte accounting (CPU): the per-rank bytes of the
expert-parallel ~1T decode with and without the attention heads split, and
with the lm_head scored in vocabulary slices (the device greedy loop) or
whole (SFK_VOCAB_SHARD=0)."""
import os

import bench
from strataflow_b200 import engine as E


def test_ep_rank_bytes_1t_shape(monkeypatch):
    monkeypatch.delenv("SFK_HEAD_PARALLEL", raising=False)
    monkeypatch.setenv("SFK_VOCAB_SHARD", "0")
    cfg = E.trillion_config()
    q8 = lambda K: K // 32 * 34   # noqa: E731
    q4 = lambda K: K // 256 * 144   # noqa: E731
    attn = (64 + 16) * 128 * q8(7168) + 7168 * q8(8192)            # 78.0 MB + 62.4 MB per layer
    router, lm_head = 4 * 7168 * 384, 160000 * q8(7168)
    expert = 2 * 2048 * q4(7168) + 7168 * q4(2048)                 # 24.77 MB
    got, split = bench.ep_rank_bytes(cfg, 4, 1)
    assert split
    assert got == 61 * (attn / 4 + router) + lm_head + 61 * 8 / 4 * expert
    assert abs(got / 1e9 - 7.05) < 0.01
    monkeypatch.setenv("SFK_HEAD_PARALLEL", "0")
    rep, split = bench.ep_rank_bytes(cfg, 4, 1)
    assert not split and rep == 61 * (attn + router) + lm_head + 61 * 8 / 4 * expert
    one, split = bench.ep_rank_bytes(cfg, 1, 1)                     # one GPU holds everything
    assert not split and one == 61 * (attn + router) + lm_head + 61 * 8 * expert
    # vocabulary slices: a quarter of the lm_head per rank
    monkeypatch.delenv("SFK_HEAD_PARALLEL", raising=False)
    monkeypatch.delenv("SFK_VOCAB_SHARD", raising=False)
    got, split = bench.ep_rank_bytes(cfg, 4, 1)
    assert split and got == 61 * (attn / 4 + router) + lm_head / 4 + 61 * 8 / 4 * expert
    assert abs(got / 1e9 - 6.13) < 0.01


def test_ep_rank_bytes_uses_config_head_width(monkeypatch):
    """A head width other than 128 (the tiny shape: d 256 / 8 heads = 32) is
    taken from the config, as the engine takes it."""
    monkeypatch.delenv("SFK_HEAD_PARALLEL", raising=False)
    monkeypatch.delenv("SFK_VOCAB_SHARD", raising=False)
    cfg = E.tiny_config(type_ffn_gu=12, type_ffn_down=12)
    q8 = lambda K: K // 32 * 34   # noqa: E731
    q4 = lambda K: K // 256 * 144   # noqa: E731
    hd = 32
    attn = (8 + 2 * 4) * hd * q8(256) + 256 * q8(8 * hd)
    expert = 2 * 512 * q4(256) + 256 * q4(512)
    got, split = bench.ep_rank_bytes(cfg, 2, 1)
    # 4 query heads x 32 columns per rank = 128 columns: not whole 256-column blocks, so no split
    assert not split
    assert got == 4 * (attn + 4 * 256 * 8) + 2048 * q8(256) + 4 * 2 / 2 * expert
