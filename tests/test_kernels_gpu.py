"""GPU parity of the operator-level entry points against the CPU oracle.

Bit-exact: dequantization, activation quantization, repack/unpack, mul_mat,
mul_mat_id and the fused expert FFN (the oracle restates the kernels' fp32
accumulation order, and SiLU uses the shared exp).  Attention accumulates its
dots and sums in double like ggml's F32 path; the order of those double sums
differs from the oracle's, which changes the float result only when a double
lands within ~1e-16 of a float rounding boundary, hence the 1e-6 bound there.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")


def _torch():
    import torch
    return torch


def _f16(v):
    return np.asarray(v, np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)


def rand_blocks(qtype, nrows, K, rng):
    """Random valid blocks (all code bits random, f16 scales finite)."""
    rb = O.row_bytes(qtype, K)
    buf = rng.integers(0, 256, size=(nrows * rb,), dtype=np.uint8)
    if qtype == O.Q4_K:
        b = buf.reshape(-1, 144)
        b[:, 0:2] = _f16(np.abs(rng.standard_normal(len(b))) * 2e-5 + 1e-6)
        b[:, 2:4] = _f16(np.abs(rng.standard_normal(len(b))) * 2e-5)
    elif qtype == O.Q6_K:
        b = buf.reshape(-1, 210)
        b[:, 208:210] = _f16(rng.standard_normal(len(b)) * 5e-6)
    elif qtype == O.Q8_0:
        b = buf.reshape(-1, 34)
        b[:, 0:2] = _f16(rng.standard_normal(len(b)) * 1.5e-4)
    return buf


def to_dev(a):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def repacked(qtype, gguf, nrows, K):
    from strataflow_b200 import ops
    return ops.repack(qtype, to_dev(gguf), nrows, K)


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.mark.parametrize("name,qtype", [("q4_k", O.Q4_K), ("q6_k", O.Q6_K), ("q8_0", O.Q8_0)])
def test_dequantize_bit_exact_vs_golden(cuda, gold, name, qtype):
    from strataflow_b200 import ops
    blocks = gold[name + "_blocks"].reshape(-1)
    exp = gold[name + "_deq"]
    got = ops.dequantize(qtype, to_dev(blocks), exp.size).cpu().numpy()
    same = (got.view(np.uint32) == exp.view(np.uint32)) | (np.isnan(got) & np.isnan(exp))
    assert same.all(), int((~same).sum())


@pytest.mark.parametrize("qtype", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_dequantize_bit_exact_vs_oracle_large(cuda, qtype):
    from strataflow_b200 import ops
    rng = np.random.default_rng(int(qtype))
    n = 4096 * 64
    blocks = rand_blocks(qtype, 64, 4096, rng)
    got = ops.dequantize(qtype, to_dev(blocks), n).cpu().numpy()
    ref = O.dequantize(qtype, blocks, n)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("act", [O.Q8_K, O.Q8_0])
def test_quantize_act_bit_exact(cuda, act):
    from strataflow_b200 import ops
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((5, 4096)) * rng.choice([1e-3, 1.0, 30.0], (5, 1))).astype(np.float32)
    x[1, 256:512] = 0.0
    x[2, 40], x[2, 41] = 77.0, -77.0  # |x| tie: the first index sets the sign
    got = ops.quantize_act(act, to_dev(x)).cpu().numpy()
    ref = np.concatenate([(O.quantize_q8_K(r) if act == O.Q8_K else O.quantize_q8_0(r)) for r in x])
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("qtype,K", [(O.Q4_K, 4096), (O.Q4_K, 14336), (O.Q6_K, 4096), (O.Q6_K, 7168),
                                     (O.Q8_0, 256), (O.Q8_0, 7168)])
def test_repack_roundtrip(cuda, qtype, K):
    from strataflow_b200 import ops
    rng = np.random.default_rng(K)
    nrows = 37
    g = rand_blocks(qtype, nrows, K, rng)
    dev = ops.repack(qtype, to_dev(g), nrows, K)
    assert dev.numel() == nrows * ops.dev_row_bytes(qtype, K)
    back = ops.unpack(qtype, dev, nrows, K, g.size).cpu().numpy()
    assert np.array_equal(back, g)


@pytest.mark.parametrize("qtype,rows,K,b", [(O.Q4_K, 1000, 4096, 1), (O.Q4_K, 300, 14336, 3), (O.Q6_K, 6144, 4096, 1),
                                            (O.Q6_K, 130, 7168, 8), (O.Q8_0, 512, 256, 1), (O.Q8_0, 77, 7168, 16)])
def test_mul_mat_matches_oracle(cuda, qtype, rows, K, b):
    from strataflow_b200 import ops
    rng = np.random.default_rng(rows + K + b)
    w = rand_blocks(qtype, rows, K, rng)
    x = rng.standard_normal((b, K)).astype(np.float32)
    y = ops.mul_mat(qtype, repacked(qtype, w, rows, K), rows, K, to_dev(x)).cpu().numpy()
    ref = np.stack([O.mul_mat(qtype, w, rows, K, x[t]) for t in range(b)])
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), np.abs(y - ref).max() / np.abs(ref).max()


@pytest.mark.parametrize("qtype,b,k,per_pair", [(O.Q4_K, 1, 2, 0), (O.Q4_K, 4, 2, 0), (O.Q6_K, 3, 2, 1),
                                                (O.Q8_0, 2, 4, 0)])
def test_mul_mat_id_matches_oracle(cuda, qtype, b, k, per_pair):
    from strataflow_b200 import ops
    torch = _torch()
    rng = np.random.default_rng(100 + b * k)
    E, rows, K = 8, 512, 4096
    w = rand_blocks(qtype, E * rows, K, rng)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(b)]).astype(np.int32)
    x = rng.standard_normal((b, k, K) if per_pair else (b, K)).astype(np.float32)
    y = ops.mul_mat_id(qtype, repacked(qtype, w, E * rows, K), E, rows, K, to_dev(x),
                       torch.from_numpy(ids).cuda()).cpu().numpy()
    rb = O.row_bytes(qtype, K) * rows
    ref = np.zeros((b, k, rows), np.float32)
    for t in range(b):
        for j in range(k):
            e = ids[t, j]
            ref[t, j] = O.mul_mat(qtype, w[e * rb:(e + 1) * rb], rows, K, x[t, j] if per_pair else x[t])
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


def _moe_case(type_gu, type_dn, E, d, F, b, k, seed):
    rng = np.random.default_rng(seed)
    gate = rand_blocks(type_gu, E * F, d, rng)
    up = rand_blocks(type_gu, E * F, d, rng)
    down = rand_blocks(type_dn, E * d, F, rng)
    x = rng.standard_normal((b, d)).astype(np.float32)
    res = rng.standard_normal((b, d)).astype(np.float32)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(b)]).astype(np.int32)
    logits = rng.standard_normal((b, k)).astype(np.float32)
    w = (np.exp(logits) / np.exp(logits).sum(1, keepdims=True)).astype(np.float32)
    return gate, up, down, x, res, ids, w


@pytest.mark.parametrize("type_gu,type_dn,E,d,F,b,k", [
    (O.Q4_K, O.Q4_K, 8, 4096, 14336, 1, 2),      # config 2 shape, b = 1
    (O.Q4_K, O.Q4_K, 8, 4096, 14336, 4, 2),      # config 2 shape, b = 4
    (O.Q6_K, O.Q6_K, 8, 1024, 2048, 2, 2),
    (O.Q8_0, O.Q8_0, 8, 256, 512, 3, 2),         # tiny-model shape
    (O.Q4_K, O.Q4_K, 16, 1024, 2048, 2, 8),      # many experts per token
])
def test_moe_ffn_matches_oracle(cuda, type_gu, type_dn, E, d, F, b, k):
    from strataflow_b200 import ops
    torch = _torch()
    gate, up, down, x, res, ids, w = _moe_case(type_gu, type_dn, E, d, F, b, k, seed=E + d + b)
    out = ops.moe_ffn(type_gu, type_dn, repacked(type_gu, gate, E * F, d), repacked(type_gu, up, E * F, d),
                      repacked(type_dn, down, E * d, F), E, d, F, to_dev(x), to_dev(res),
                      torch.from_numpy(ids).cuda(), to_dev(w)).cpu().numpy()
    ref, _ = O.moe_ffn(type_gu, type_dn, gate, up, down, E, d, F, x, res, ids, w)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), \
        np.linalg.norm(out - ref) / np.linalg.norm(ref - res)


def test_moe_ffn_repeated_calls_are_identical(cuda):
    """The SwiGLU re-quantization counters reset themselves between calls."""
    from strataflow_b200 import ops
    torch = _torch()
    E, d, F, b, k = 8, 1024, 2048, 2, 2
    gate, up, down, x, res, ids, w = _moe_case(O.Q4_K, O.Q4_K, E, d, F, b, k, seed=5)
    args = (O.Q4_K, O.Q4_K, repacked(O.Q4_K, gate, E * F, d), repacked(O.Q4_K, up, E * F, d),
            repacked(O.Q4_K, down, E * d, F), E, d, F, to_dev(x), None, torch.from_numpy(ids).cuda(), to_dev(w))
    a = ops.moe_ffn(*args).cpu().numpy()
    c = ops.moe_ffn(*args).cpu().numpy()
    assert np.array_equal(a, c)


def _paged_case(b, ctx, Hq, Hkv, hd, f16, seed):
    torch = _torch()
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((b, Hq, hd)).astype(np.float32)
    K = rng.standard_normal((b, ctx, Hkv, hd)).astype(np.float32)
    V = rng.standard_normal((b, ctx, Hkv, hd)).astype(np.float32)
    if f16:
        K = K.astype(np.float16).astype(np.float32)
        V = V.astype(np.float16).astype(np.float32)
    max_pages = (ctx + 15) // 16
    perm = rng.permutation(b * max_pages).astype(np.int32)
    ptab = perm.reshape(b, max_pages)
    kp = np.zeros((b * max_pages, Hkv, 16, hd), np.float32)
    vp = np.zeros_like(kp)
    for t in range(b):
        for p in range(max_pages):
            n = min(16, ctx - 16 * p)
            kp[ptab[t, p], :, :n] = K[t, 16 * p:16 * p + n].transpose(1, 0, 2)
            vp[ptab[t, p], :, :n] = V[t, 16 * p:16 * p + n].transpose(1, 0, 2)
    dt = torch.float16 if f16 else torch.float32
    dev = (to_dev(q), torch.from_numpy(kp).to(dt).cuda(), torch.from_numpy(vp).to(dt).cuda(),
           torch.from_numpy(ptab).cuda())
    return q, K, V, dev


@pytest.mark.parametrize("b,ctx,f16", [(1, 512, True), (8, 512, True), (1, 4096, True), (8, 4096, True),
                                       (1, 32768, True), (2, 700, False), (3, 1, False), (1, 17, True)])
def test_attn_paged_matches_oracle(cuda, b, ctx, f16):
    from strataflow_b200 import ops
    torch = _torch()
    Hq, Hkv, hd = 32, 8, 128
    q, K, V, (dq, dk, dv, dpt) = _paged_case(b, ctx, Hq, Hkv, hd, f16, seed=ctx + b)
    # sequences of unequal length: sequence t attends over 0..pos_t
    pos = np.array([ctx - 1 - (t * 37) % max(ctx, 1) for t in range(b)], np.int32)
    out = ops.attn_decode_paged(dq, dk, dv, dpt, torch.from_numpy(pos).cuda(), Hq, Hkv, hd).cpu().numpy()
    for t in range(b):
        n = pos[t] + 1
        ref = O.attn_decode(q[t].ravel(), K[t, :n], V[t, :n], Hq, Hkv, hd)
        assert np.abs(out[t] - ref).max() <= 1e-6 * np.abs(ref).max(), (t, np.abs(out[t] - ref).max())


def test_attn_paged_small_heads(cuda):
    from strataflow_b200 import ops
    torch = _torch()
    b, ctx, Hq, Hkv, hd = 2, 80, 8, 4, 32
    q, K, V, (dq, dk, dv, dpt) = _paged_case(b, ctx, Hq, Hkv, hd, False, seed=1)
    pos = np.array([79, 40], np.int32)
    out = ops.attn_decode_paged(dq, dk, dv, dpt, torch.from_numpy(pos).cuda(), Hq, Hkv, hd).cpu().numpy()
    for t in range(b):
        ref = O.attn_decode(q[t].ravel(), K[t, :pos[t] + 1], V[t, :pos[t] + 1], Hq, Hkv, hd)
        assert np.abs(out[t] - ref).max() <= 1e-6 * np.abs(ref).max()


@pytest.mark.parametrize("Hq,Hkv,hd,ctx,f16", [(64, 8, 128, 1024, True),   # GQA group of 8 (the 1T shape)
                                              (16, 4, 64, 300, False),
                                              (8, 8, 256, 100, True)])
def test_attn_paged_other_head_shapes(cuda, Hq, Hkv, hd, ctx, f16):
    from strataflow_b200 import ops
    torch = _torch()
    b = 2
    q, K, V, (dq, dk, dv, dpt) = _paged_case(b, ctx, Hq, Hkv, hd, f16, seed=hd + ctx)
    pos = np.array([ctx - 1, ctx // 3], np.int32)
    out = ops.attn_decode_paged(dq, dk, dv, dpt, torch.from_numpy(pos).cuda(), Hq, Hkv, hd).cpu().numpy()
    for t in range(b):
        ref = O.attn_decode(q[t].ravel(), K[t, :pos[t] + 1], V[t, :pos[t] + 1], Hq, Hkv, hd)
        assert np.abs(out[t] - ref).max() <= 1e-6 * np.abs(ref).max()


def test_attn_paged_rejects_page_outside_pool(cuda):
    """A page id past the pool is checked before any copy and reported."""
    from strataflow_b200 import lib as L
    from strataflow_b200 import ops
    torch = _torch()
    q, K, V, (dq, dk, dv, dpt) = _paged_case(1, 64, 8, 4, 32, False, seed=5)
    bad = dpt.clone()
    bad[0, 1] = dk.shape[0]          # one past the last page
    pos = torch.tensor([63], dtype=torch.int32, device="cuda")
    with pytest.raises(L.SfkError):
        ops.attn_decode_paged(dq, dk, dv, bad, pos, 8, 4, 32)
    out = ops.attn_decode_paged(dq, dk, dv, dpt, pos, 8, 4, 32).cpu().numpy()   # still usable
    ref = O.attn_decode(q[0].ravel(), K[0], V[0], 8, 4, 32)
    assert np.abs(out[0] - ref).max() <= 1e-6 * np.abs(ref).max()


def test_mul_mat_id_rejects_bad_expert_id(cuda):
    from strataflow_b200 import ops, lib as L
    torch = _torch()
    rng = np.random.default_rng(0)
    w = rand_blocks(O.Q8_0, 4 * 32, 256, rng)
    with pytest.raises(L.SfkError):
        ops.mul_mat_id(O.Q8_0, repacked(O.Q8_0, w, 128, 256), 4, 32, 256,
                       to_dev(np.ones((1, 256), np.float32)), torch.tensor([[0, 9]], dtype=torch.int32).cuda())
