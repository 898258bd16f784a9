"""The tensor-core (tcgen05 kind::i8) quantized GEMM against the CPU oracle
(GPU).  Its integer sub-block dots are exact and it adds 256-column blocks in
ggml's generic block order, so it must equal the oracle's block-order mode
(fp32_mode=2, the arithmetic of ggml's reference vec_dot_*_q8_K / q8_0) bit for
bit, at any token count -- one token, a partial 64-token tile, several tiles --
and for weight row counts that are not multiples of the 128-row tile."""
import numpy as np
import pytest

from oracle import oracle as O
from test_kernels_gpu import rand_blocks, repacked, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qtype,rows,K,n", [
    (O.Q4_K, 256, 4096, 1), (O.Q4_K, 300, 4096, 70), (O.Q4_K, 128, 14336, 130),
    (O.Q6_K, 256, 4096, 33), (O.Q6_K, 200, 4096, 64),
    (O.Q8_0, 128, 256, 5), (O.Q8_0, 130, 7168, 65),
])
def test_mul_mat_tc_matches_oracle_block_order(cuda, qtype, rows, K, n):
    from strataflow_b200 import ops
    rng = np.random.default_rng(rows * 7 + K + n)
    w = rand_blocks(qtype, rows, K, rng)
    x = rng.standard_normal((n, K)).astype(np.float32)
    y = ops.mul_mat_tc(qtype, repacked(qtype, w, rows, K), rows, K, to_dev(x)).cpu().numpy()
    ref = np.stack([O.mul_mat(qtype, w, rows, K, x[t], fp32_mode=2) for t in range(n)])
    bad = np.argwhere(y.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, (bad[:5], np.abs(y - ref).max() / np.abs(ref).max())


def test_mul_mat_tc_close_to_decode_kernel(cuda):
    """Against the decode GEMV (same activation codes, unit-order fp32 sums):
    equal up to the order of the fp32 additions."""
    from strataflow_b200 import ops
    rng = np.random.default_rng(5)
    rows, K, n = 512, 4096, 16
    w = rand_blocks(O.Q4_K, rows, K, rng)
    x = rng.standard_normal((n, K)).astype(np.float32)
    wd = repacked(O.Q4_K, w, rows, K)
    a = ops.mul_mat_tc(O.Q4_K, wd, rows, K, to_dev(x)).cpu().numpy()
    b = ops.mul_mat(O.Q4_K, wd, rows, K, to_dev(x)).cpu().numpy()
    assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()


def _ids(rng, b, k, E, skew=False):
    if skew:   # most pairs on one expert: several full tiles of it
        ids = np.stack([[0] + list(rng.choice(np.arange(1, E), k - 1, replace=False)) for _ in range(b)])
    else:
        ids = np.stack([rng.choice(E, k, replace=False) for _ in range(b)])
    return ids.astype(np.int32)


@pytest.mark.parametrize("qtype,E,rows,K,b,k,per_pair,skew", [
    (O.Q4_K, 8, 300, 4096, 40, 2, 0, False),
    (O.Q4_K, 8, 256, 4096, 1, 2, 0, False),
    (O.Q4_K, 8, 128, 4096, 150, 2, 0, True),
    (O.Q6_K, 16, 200, 4096, 33, 4, 1, False),
    (O.Q8_0, 64, 130, 512, 50, 8, 0, False),
])
def test_mul_mat_id_tc_matches_oracle_block_order(cuda, qtype, E, rows, K, b, k, per_pair, skew):
    """The expert-grouped tensor-core mul_mat_id: every (token, expert) pair's
    row equals the oracle's block-order product bit for bit, and the rows come
    back in pair order, for a single token, partial and full 64-row tiles of
    one expert, per-pair activations and 64 experts."""
    import torch
    from strataflow_b200 import ops
    rng = np.random.default_rng(E * 1000 + b * k + rows)
    w = rand_blocks(qtype, E * rows, K, rng)
    ids = _ids(rng, b, k, E, skew)
    x = rng.standard_normal((b, k, K) if per_pair else (b, K)).astype(np.float32)
    y = ops.mul_mat_id_tc(qtype, repacked(qtype, w, E * rows, K), E, rows, K, to_dev(x),
                          torch.from_numpy(ids).cuda()).cpu().numpy()
    rb = O.row_bytes(qtype, K) * rows
    for t in range(b):
        for j in range(k):
            e = ids[t, j]
            ref = O.mul_mat(qtype, w[e * rb:(e + 1) * rb], rows, K, x[t, j] if per_pair else x[t], fp32_mode=2)
            assert np.array_equal(y[t, j].view(np.uint32), ref.view(np.uint32)), (t, j, e)


def test_mul_mat_id_tc_close_to_decode_kernel(cuda):
    """Against the CUDA-core mul_mat_id (same activation codes, unit-order
    fp32 sums): equal up to the order of the fp32 additions."""
    import torch
    from strataflow_b200 import ops
    rng = np.random.default_rng(8)
    E, rows, K, b, k = 8, 512, 4096, 16, 2
    w = rand_blocks(O.Q4_K, E * rows, K, rng)
    wd = repacked(O.Q4_K, w, E * rows, K)
    ids = torch.from_numpy(_ids(rng, b, k, E)).cuda()
    x = to_dev(rng.standard_normal((b, K)).astype(np.float32))
    a = ops.mul_mat_id_tc(O.Q4_K, wd, E, rows, K, x, ids).cpu().numpy()
    c = ops.mul_mat_id(O.Q4_K, wd, E, rows, K, x, ids).cpu().numpy()
    assert np.abs(a - c).max() <= 1e-5 * np.abs(c).max()


def test_mul_mat_id_tc_rejects_bad_expert_id(cuda):
    import torch
    from strataflow_b200 import lib as L
    from strataflow_b200 import ops
    rng = np.random.default_rng(9)
    w = rand_blocks(O.Q8_0, 4 * 32, 256, rng)
    ids = torch.tensor([[0, 4]], dtype=torch.int32, device="cuda")
    with pytest.raises(L.SfkError) as ei:
        ops.mul_mat_id_tc(O.Q8_0, repacked(O.Q8_0, w, 128, 256), 4, 32, 256,
                          to_dev(rng.standard_normal((1, 256)).astype(np.float32)), ids)
    assert ei.value.status == L.SFK_ERR_RUNTIME
    # the status word is cleared: a valid call afterwards succeeds
    ok = torch.tensor([[0, 3]], dtype=torch.int32, device="cuda")
    ops.mul_mat_id_tc(O.Q8_0, repacked(O.Q8_0, w, 128, 256), 4, 32, 256,
                      to_dev(rng.standard_normal((1, 256)).astype(np.float32)), ok)
