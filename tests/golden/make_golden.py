"""Generate the committed golden vectors that pin the CPU oracle.

The reference's arithmetic for this path lives in ggml (llama.cpp tag b11379),
an un-vendored submodule of the reference.  gguf-py 0.19.0 (installed in the
build container, absent on the GPU box) restates ggml's reference dequantizers
and its Q8_0 quantizer in numpy; its own header says Q8_0 is "bit-exact same
results as reference implementation in ggml-quants.c".  This script runs
gguf-py once and freezes inputs and outputs into golden.npz, so the tests can
check the oracle (and the CUDA dequantizer) anywhere without gguf-py.

    python tests/golden/make_golden.py        # rewrites tests/golden/golden.npz

Blocks are random bytes with the f16 scale fields replaced by finite values of
realistic magnitude, plus hand-made edge blocks (all-zero scales, extreme codes,
negative/subnormal f16 scales).
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _f16(vals) -> np.ndarray:
    return np.asarray(vals, dtype=np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)


def make(seed: int = 1234, nblk: int = 48) -> dict:
    import gguf
    from gguf import quants

    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {"gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")}

    # Q4_K: [d f16][dmin f16][scales 12][qs 128]
    q4 = rng.integers(0, 256, size=(nblk, 144), dtype=np.uint8)
    q4[:, 0:2] = _f16(rng.standard_normal(nblk) * 1e-3)
    q4[:, 2:4] = _f16(np.abs(rng.standard_normal(nblk)) * 1e-3)
    q4[0, 4:16] = 0                       # all-zero scales and mins
    q4[1, 4:16] = 0xFF                    # all scale/min bits set (63s)
    q4[2, 0:2] = _f16([6.0e-8])           # subnormal f16 d
    q4[3, 0:4] = _f16([-65504.0, 65504.0]).reshape(-1)
    out["q4_k_blocks"] = q4
    out["q4_k_deq"] = quants.dequantize(q4.reshape(-1), gguf.GGMLQuantizationType.Q4_K).astype(np.float32).ravel()

    # Q6_K: [ql 128][qh 64][scales 16 int8][d f16]
    q6 = rng.integers(0, 256, size=(nblk, 210), dtype=np.uint8)
    q6[:, 208:210] = _f16(rng.standard_normal(nblk) * 1e-3)
    q6[0, 192:208] = 0x80                 # scales = -128
    q6[1, 192:208] = 0x7F                 # scales = 127
    q6[2, 0:192] = 0xFF                   # every code = 63 -> +31
    q6[3, 0:192] = 0x00                   # every code = 0 -> -32
    out["q6_k_blocks"] = q6
    out["q6_k_deq"] = quants.dequantize(q6.reshape(-1), gguf.GGMLQuantizationType.Q6_K).astype(np.float32).ravel()

    # Q8_0: [d f16][qs 32 int8]
    nq8 = nblk * 8
    q8 = rng.integers(0, 256, size=(nq8, 34), dtype=np.uint8)
    q8[:, 0:2] = _f16(rng.standard_normal(nq8) * 1e-2)
    q8[0, 2:] = 0x80                      # -128 codes
    out["q8_0_blocks"] = q8
    out["q8_0_deq"] = quants.dequantize(q8.reshape(-1), gguf.GGMLQuantizationType.Q8_0).astype(np.float32).ravel()

    # Q8_0 quantizer (ggml quantize_row_q8_0_ref): activations incl. exact
    # half-way values, zeros and a zero block
    x = (rng.standard_normal(nblk * 256) * rng.choice([1e-3, 1.0, 50.0], nblk * 256)).astype(np.float32)
    x[:32] = 0.0
    x[32:64] = np.linspace(-127, 127, 32, dtype=np.float32)
    x[64:96] = (np.arange(32, dtype=np.float32) - 15.5) * 0.5
    out["q8_0_x"] = x
    out["q8_0_q"] = quants.quantize(x.reshape(-1, 32), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    return out


def main() -> None:
    arrs = make()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrs)
    print("wrote", os.path.join(HERE, "golden.npz"), {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
