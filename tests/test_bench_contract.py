"""bench.py's reference arm keeps the JSON-line contract, on CPU.

The arm times the CPU restatement of the block (no GPU needed), so its line
can be checked here: one JSON line from rank 0, the metric of configuration 1,
exactly the requested steps, an ``e2e`` object with no host-device bytes and
a ``cpu_baseline`` that says what was timed.  Under torchrun with two ranks,
rank 0 alone prints, and the other rank exits 0 without work."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lines(out: str) -> list[dict]:
    return [json.loads(ln) for ln in out.splitlines() if ln.startswith("{")]


def _check_line(d: dict, n_gpus: int) -> None:
    assert d["impl"] == "reference"
    assert d["metric"] == "moe_block_decode_us_per_token" and d["unit"] == "us/token"
    assert d["higher_is_better"] is False and d["steps"] == 3 and d["warmup"] == 3
    assert d["n_gpus"] == n_gpus and d["value"] > 0
    assert d["config"]["workload"] == "config1 q8 decode T=1"
    assert d["e2e"] == {"value": d["value"], "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "rnb_cpu_fast.c" in cb["sample"]


def test_reference_arm_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check_line(lines[0], 1)


def test_reference_arm_two_ranks_one_line():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check_line(lines[0], 2)
