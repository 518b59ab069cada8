"""The bench's reference arm (`bench.py --impl reference`) on the host cores:
one JSON line with the contract's keys on a small config-2 shape, from rank 0
alone when launched with torchrun (gloo), the other ranks exiting 0 without
output. It needs no GPU and loads nothing of the library."""
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
SMALL = ["--impl", "reference", "--nodes", "200000", "--batch", "256", "--steps", "2", "--warmup", "3",
         "--cpu-file-gb", "0.2", "--no-cold"]


def _lines(out: str):
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def _check(line: dict, n_gpus: int):
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["n_gpus"] == n_gpus and line["steps"] == 2 and line["warmup"] == 3
    assert line["config"]["workload"].startswith("c2: 200000 nodes")
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and "sample" in cb
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *SMALL], capture_output=True, text=True,
                       timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 1)


def test_reference_arm_under_torchrun_prints_once():
    port = 29900 + os.getpid() % 90
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(REPO, "bench.py"), "--gpus", "2", *SMALL]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1  # rank 0 alone prints
    _check(lines[0], 2)
