"""The benchmark's byte accounting (CPU): the per-rank bytes of the
expert-parallel ~1T decode with and without the attention heads split."""
import os

import bench
from strataflow_b200 import engine as E


def test_ep_rank_bytes_1t_shape(monkeypatch):
    monkeypatch.delenv("SFK_HEAD_PARALLEL", raising=False)
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
