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
