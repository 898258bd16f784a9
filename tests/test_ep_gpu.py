"""Expert parallelism over two GPUs of one box: each rank holds half of every
layer's experts (and, when the heads split into whole 256-column blocks, half
of the attention heads with their KV), the ranks add their partial outputs
through peer memory after every layer.  The decode must match the CPU oracle
run in expert parallelism's fp32 order (`ep_size`, `ep_head_par`: each rank's
partial summed over its own experts / head columns, rank 0 adding the
residual, partials added in rank order -- the only arithmetic that differs
from one GPU): identical greedy tokens, every step's logits within the
north-star 1e-3 relative L2 / 1e-2 max-abs, the same logits on both ranks
(bit-identical: the ranks add the same partials in the same order), and the
device greedy loop continuing with the oracle's tokens; steps that return no
logits (the device loop, host steps without logits) score each rank's slice
of the vocabulary and exchange the argmax.  Skipped on a box
with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, cfg_kw, seed, prompt, n_gen, q, env=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), **(env or {}))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        from strataflow_b200 import engine as E
        cfg = E.tiny_config(**cfg_kw).replace(ep_size=world, ep_rank=rank)
        eng = E.Engine.load(cfg, seed=seed, device=rank)
        eng.ep_connect_group()
        toks, logits = eng.generate(prompt, n_gen, host_loop=True)
        dev = eng.decode_greedy(6, 1)[:, 0].tolist()   # device loop continues the sequence
        # host steps that return no logits: each rank scores its vocabulary
        # slice and the argmax is exchanged
        eng.reset_kv()
        for pos, t in enumerate(prompt):
            am, _ = eng.forward(t, pos, want_logits=False)
        nl = []
        for i in range(4):
            nl.append(int(am))
            am, _ = eng.forward(am, len(prompt) + i, want_logits=False)
        q.put((rank, toks, np.stack(logits), dev + [nl], None))
        dist.barrier()
        eng.close()
        dist.destroy_process_group()
    except Exception as ex:  # report instead of hanging the parent
        q.put((rank, None, None, None, repr(ex)))


WIDE = dict(n_layer=2, n_embd=512, n_head=16, n_head_kv=4)   # heads split into whole 256-column blocks


def _head_par(cfg, world, env):
    """The engine's rule for splitting the attention heads (sfk_engine_create)."""
    if (env or {}).get("SFK_HEAD_PARALLEL") == "0":
        return 0
    return int(cfg.n_head % world == 0 and cfg.n_head_kv % world == 0 and (cfg.n_head // world) * cfg.hd % 256 == 0)


@pytest.mark.parametrize("cfg_kw,env", [
    (dict(n_layer=2), {}),                                                   # routing inside gate/up
    (dict(n_layer=2, type_ffn_gu=12, type_ffn_down=12, n_expert=16, n_expert_used=4), {}),
    (dict(n_layer=2, n_expert=72, n_expert_used=4), {}),                     # router staged per CTA
    (dict(n_layer=2, n_expert=160, n_expert_used=2), {}),                    # logits exchanged between CTAs
    (WIDE, {"SFK_HEAD_PARALLEL": "0"}),                                      # trunk replicated
    (WIDE, {}),                                                              # heads split over the ranks
    # the router kernel (steps of more than two tokens take it), building each
    # rank's slot lists for its own experts
    (dict(n_layer=2), {"SFK_ROUTER_KERNEL": "1"}),
    (dict(n_layer=2, n_expert=72, n_expert_used=4), {"SFK_ROUTER_KERNEL": "1"}),
])
def test_expert_parallel_two_ranks_match_oracle(cuda, cfg_kw, env):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import oracle as O
    from parity_util import close, oracle_cfg
    from strataflow_b200 import engine as E
    seed, n_gen, n_dev = 11, 10, 6
    prompt = np.random.default_rng(3).integers(0, 4096, 8).tolist()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, cfg_kw, seed, prompt, n_gen, q, env)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, toks, logits, dev, err = q.get(timeout=300)
        assert err is None, err
        res[rank] = (toks, logits, dev)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = E.tiny_config(**cfg_kw)
    om = O.Model(oracle_cfg(cfg, ep_size=2, ep_head_par=_head_par(cfg, 2, env)), seed=seed)
    ref_toks, ref_logits = O.greedy(om, prompt, n_gen + n_dev, want_logits=True)
    assert res[0][0] == res[1][0] == ref_toks[:n_gen]
    assert np.array_equal(res[0][1].view(np.uint32), res[1][1].view(np.uint32))
    for i in range(n_gen + 1):
        ok, rel, mx = close(res[0][1][i], ref_logits[i])
        assert ok, (i, rel, mx)
    # the device loop's first token is the argmax of the last host step
    assert res[0][2][:-1] == res[1][2][:-1] == ref_toks[n_gen:n_gen + n_dev]
    assert res[0][2][-1] == res[1][2][-1] == ref_toks[:4]
