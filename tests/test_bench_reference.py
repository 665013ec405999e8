"""The benchmark's reference arm (`bench.py --impl reference`), which times the
reference's CPU search paths on the host cores, keeps the JSON contract the
round-end runs read: one line from rank 0 with the metric, unit, value, a
`cpu_baseline` describing the run and an `e2e` object without host-device
traffic; under torchrun the other ranks exit 0 without output. CPU only, on a
small corpus."""

import json
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
ARGS = ["--impl", "reference", "--steps", "1", "--warmup", "3", "--rows", "5000"]


def _json_lines(text):
    return [json.loads(line) for line in text.splitlines() if line.startswith("{")]


def _check_line(d, n_gpus):
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "ms_per_step", "higher_is_better", "scaling", "vs_baseline", "dtype",
                "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["n_gpus"] == n_gpus and d["steps"] == 1 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["rows_per_gpu"] == 5000


def test_reference_arm_prints_one_contract_line():
    res = subprocess.run([sys.executable, "bench.py", *ARGS], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1
    _check_line(lines[0], 1)


def test_reference_arm_under_torchrun_prints_from_rank_0_only():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--gpus", "2", *ARGS]
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1
    _check_line(lines[0], 2)
