"""The .strata file reader (host side) over libsfk.so.

Mirrors the reference's StrataReader (src/tws/strata_file.h / .cpp): open a
packed file, read its model shape from the embedded GGUF metadata, read a
trunk tensor or a (layer, expert) bundle verbatim, and fill an engine's HBM
tier from it (Engine::load_strata_weights, src/model/engine/engine.cpp:556-830).
All parsing happens in the C++ library; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib as L


class StrataFile:
    """An open .strata file (sfk_strata_open).  Use as a context manager or
    call close()."""

    def __init__(self, path: str):
        self._lib = L.load()
        h = C.c_void_p()
        L.check(self._lib.sfk_strata_open(str(path).encode(), C.byref(h)))
        self.h = h
        self.path = str(path)

    def close(self) -> None:
        if getattr(self, "h", None):
            self._lib.sfk_strata_close(self.h)
            self.h = None

    def __enter__(self) -> "StrataFile":
        return self

    def __exit__(self, *a) -> None:
        self.close()

    def __del__(self):
        self.close()

    def hparams(self, base: L.Hparams | None = None) -> L.Hparams:
        """Model shape from the GGUF keys; engine options (n_ctx, kv_type,
        max_batch, ep_size, ep_rank) come from `base`."""
        hp = L.Hparams() if base is None else base
        L.check(self._lib.sfk_strata_hparams(self.h, C.byref(hp)))
        return hp

    def tensors(self) -> list[dict]:
        """The GGUF tensor table: name, type, ne, nbytes, expert."""
        out = []
        name = C.create_string_buffer(128)
        t, ex = C.c_int32(), C.c_int32()
        ne = (C.c_int64 * 4)()
        nb = C.c_uint64()
        for i in range(int(self._lib.sfk_strata_n_tensors(self.h))):
            L.check(self._lib.sfk_strata_tensor_info(self.h, i, name, 128, C.byref(t), ne, C.byref(nb), C.byref(ex)))
            out.append({"name": name.value.decode(), "type": t.value, "ne": tuple(ne), "nbytes": nb.value,
                        "expert": bool(ex.value)})
        return out

    def read_trunk(self, name: str, nbytes: int) -> np.ndarray:
        buf = np.empty(nbytes, np.uint8)
        L.check(self._lib.sfk_strata_read_trunk(self.h, name.encode(), buf.ctypes.data_as(C.c_void_p), nbytes))
        return buf

    def read_bundle(self, layer: int, expert: int) -> np.ndarray:
        """StrataReader::read_bundle: gate|up|down of one expert."""
        n = int(self._lib.sfk_strata_bundle_bytes(self.h, layer))
        buf = np.empty(n, np.uint8)
        L.check(self._lib.sfk_strata_read_bundle(self.h, layer, expert, buf.ctypes.data_as(C.c_void_p), n))
        return buf

    def load_into(self, engine) -> None:
        """Upload every trunk tensor and every expert bundle into `engine`."""
        L.check(self._lib.sfk_strata_load(self.h, engine.h))


def pack(gguf_path: str, strata_path: str) -> None:
    """sfk_strata_pack: a GGUF checkpoint into a .strata file (the reference's
    pack_gguf_to_strata, src/tws/strata_pack.cpp:251, without LZ
    compression); raises SfkError on a refused or unreadable input."""
    lib = L.load()
    L.check(lib.sfk_strata_pack(str(gguf_path).encode(), str(strata_path).encode()))
