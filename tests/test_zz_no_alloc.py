"""sfk_moe_ffn_noalloc: the fused expert FFN for callers that cannot allocate.

A caller whose device memory is already fully owned -- an engine that gave all
of HBM to its own pools, a process whose allocations all go through another
framework's allocator, a loop that cannot afford cudaMalloc's device-wide
synchronization -- calls sfk_moe_ffn_noalloc instead of sfk_moe_ffn.  It keeps
its scratch in a fixed array inside the library instead of allocating.  These
tests call it through the C ABI and check it against sfk_moe_ffn; the fused
FFN is bit-exact everywhere else in the suite, so equality is exact here too.

This file is collected last on purpose: a run that stops at its first failure
has already run every other test by the time it gets here.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q4_K, Q6_K = 12, 14


def _f16(v):
    return np.asarray(v, np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)


def _blocks(qtype, nrows, K, rng):
    """Random valid GGUF blocks: random code bits, small finite f16 scales."""
    if qtype == Q4_K:
        b = rng.integers(0, 256, size=(nrows * K // 256, 144), dtype=np.uint8)
        b[:, 0:2] = _f16(np.abs(rng.standard_normal(len(b))) * 2e-5 + 1e-6)
        b[:, 2:4] = _f16(np.abs(rng.standard_normal(len(b))) * 2e-5)
    else:
        b = rng.integers(0, 256, size=(nrows * K // 256, 210), dtype=np.uint8)
        b[:, 208:210] = _f16(rng.standard_normal(len(b)) * 5e-6)
    return b.reshape(-1)


def _case(qtype, E, d, F, b, k, seed):
    import torch
    from strataflow_b200 import ops
    rng = np.random.default_rng(seed)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    gate = ops.repack(qtype, dev(_blocks(qtype, E * F, d, rng)), E * F, d)
    up = ops.repack(qtype, dev(_blocks(qtype, E * F, d, rng)), E * F, d)
    down = ops.repack(qtype, dev(_blocks(qtype, E * d, F, rng)), E * d, F)
    x = dev(rng.standard_normal((b, d)).astype(np.float32))
    res = dev(rng.standard_normal((b, d)).astype(np.float32))
    ids = dev(np.stack([rng.choice(E, k, replace=False) for _ in range(b)]).astype(np.int32))
    lg = rng.standard_normal((b, k))
    w = dev((np.exp(lg) / np.exp(lg).sum(1, keepdims=True)).astype(np.float32))
    return gate, up, down, x, res, ids, w


def _call_noalloc(qtype, gate, up, down, E, d, F, x, res, ids, w, b, k):
    import torch
    from strataflow_b200 import lib as L
    out = torch.empty((b, d), dtype=torch.float32, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    L.check(L.load().sfk_moe_ffn_noalloc(qtype, qtype, P(gate), P(up), P(down), E, d, F, P(x), P(res), P(ids),
                                         P(w), b, k, P(out), stream))
    return out.cpu().numpy()


@pytest.mark.parametrize("qtype,E,d,F,b,k", [
    (Q4_K, 8, 4096, 14336, 1, 2),   # Mixtral expert shape, batch 1
    (Q6_K, 8, 1024, 2048, 3, 2),
])
def test_noalloc_matches_allocating_moe_ffn_twice(cuda, qtype, E, d, F, b, k):
    from strataflow_b200 import ops
    gate, up, down, x, res, ids, w = _case(qtype, E, d, F, b, k, seed=d + b)
    ref = ops.moe_ffn(qtype, qtype, gate, up, down, E, d, F, x, res, ids, w).cpu().numpy()
    for _ in range(2):   # the second call reuses the scratch the first left behind
        got = _call_noalloc(qtype, gate, up, down, E, d, F, x, res, ids, w, b, k)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    import torch
    from strataflow_b200 import lib as L
    one = torch.zeros(16, dtype=torch.float32, device="cuda")
    P = C.c_void_p(one.data_ptr())
    # b=16 tokens x 8 experts x F=14336 needs ~9 MB of scratch, over the 4 MiB area
    rc = L.load().sfk_moe_ffn_noalloc(Q4_K, Q4_K, P, P, P, 8, 4096, 14336, P, None, P, P, 16, 8, P, None)
    assert rc == 1
    assert b"fixed area" in L.load().sfk_last_error()
