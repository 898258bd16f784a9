"""The benchmark's reference arm under a multi-rank launch, on CPU: launched
the way a scaling run launches it (torchrun, two ranks on 127.0.0.1), every
rank exits 0 and rank 0 alone prints one JSON line carrying the contract's
keys, on the same metric and unit as the measured arm."""
import json
import os
import socket
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_arm_two_ranks_one_line():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference", "--gpus", "2",
           "--steps", "1", "--warmup", "0"]
    out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = lines[0]
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "tok/s"
    assert d["n_gpus"] == 2 and d["value"] > 0 and d["higher_is_better"] is True
    for k in ("steps", "warmup", "ms_per_step", "scaling", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
