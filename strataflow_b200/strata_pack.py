"""The strata-pack tool: convert a GGUF checkpoint into a .strata file.

    python -m strataflow_b200.strata_pack MODEL.gguf MODEL.strata

The reference ships this as tools/strata-pack over pack_gguf_to_strata
(src/tws/strata_pack.cpp:251); here the packing runs in libsfk.so
(sfk_strata_pack) and this module is its command line.  Weight bytes are
copied verbatim, so the .strata decodes exactly like its source GGUF.
"""
from __future__ import annotations

import argparse
import os
import sys

from . import lib as L
from .strata import StrataFile, pack


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m strataflow_b200.strata_pack", description=__doc__.splitlines()[0])
    ap.add_argument("gguf", help="source GGUF checkpoint")
    ap.add_argument("strata", help="output .strata file")
    a = ap.parse_args(argv)
    try:
        pack(a.gguf, a.strata)
        with StrataFile(a.strata) as f:   # the written file opens and parses
            n = len(f.tensors())
    except L.SfkError as ex:
        print(f"strata-pack: {ex}", file=sys.stderr)
        return 1
    size = os.path.getsize(a.strata)
    print(f"wrote {a.strata} ({size} bytes, {n} tensors)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
