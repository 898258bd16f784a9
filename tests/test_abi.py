"""CPU tests of the C-ABI library: it builds for sm_100a, loads, exports every
entry point declared in include/sfk.h, and its host-only helpers answer without
a GPU.  No kernel is launched here."""
import ctypes as C
import subprocess

import pytest

from strataflow_b200 import build as B
from strataflow_b200 import lib as L


@pytest.fixture(scope="module")
def sfk():
    B.build()
    return L.load()


def test_library_exports_every_header_function(sfk):
    names = L.header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(sfk, n)]
    assert not missing, missing
    # the ctypes signature table covers the whole header
    assert sorted(L._SIGS) == names


def test_exported_symbols_are_c_abi(sfk):
    out = subprocess.run(["nm", "-D", "--defined-only", B.LIB], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    for n in L.header_functions():
        assert n in exported, n          # unmangled extern "C" names
    assert not any(s.startswith("_ZN3sfk") for s in exported)  # internals stay hidden


def test_status_strings(sfk):
    assert sfk.sfk_status_str(0) == b"ok"
    assert sfk.sfk_status_str(7) == b"runtime error"
    assert isinstance(sfk.sfk_last_error(), bytes)


@pytest.mark.parametrize("qtype,K,gguf", [(12, 4096, 2304), (14, 4096, 3360), (8, 4096, 4352), (12, 14336, 8064),
                                          (14, 7168, 5888), (8, 256, 272)])
def test_device_row_bytes_match_gguf(sfk, qtype, K, gguf):
    # the device layout streams exactly the GGUF bytes (Q6_K pads d to 16 B)
    assert sfk.sfk_dev_row_bytes(qtype, K) == gguf
    assert sfk.sfk_dev_row_bytes(qtype, 100) == 0


def test_engine_create_rejects_bad_hparams_without_touching_a_gpu(sfk):
    hp = L.Hparams()
    out = C.c_void_p()
    rc = sfk.sfk_engine_create(0, C.byref(hp), C.byref(out))   # all-zero shape
    assert rc == L.SFK_OK + 1 and not out.value
    assert b"positive" in sfk.sfk_last_error()


def test_expert_parallel_shape_is_checked_before_any_gpu_work(sfk):
    """ep_size must divide n_expert and ep_rank lie in [0, ep_size)."""
    from strataflow_b200 import engine as E
    out = C.c_void_p()
    for kw in (dict(ep_size=3), dict(ep_size=2, ep_rank=2), dict(ep_size=16)):
        hp = E.tiny_config(**kw).to_c()   # 8 experts
        rc = sfk.sfk_engine_create(0, C.byref(hp), C.byref(out))
        assert rc == L.SFK_OK + 1 and not out.value, kw
        assert b"ep_size" in sfk.sfk_last_error()
