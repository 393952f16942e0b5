"""bench.py's reference arm on the CPU (no GPU needed): the CPU restatement of
the reference engine timed at the GPU arm's positions, printed as the one
JSON line the benchmark contract asks for, alone and under torchrun with two
ranks (rank 0 prints, the other rank exits 0 without work).  A small sample
of the 3B 2-bit workload keeps each run to seconds."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = ["--impl", "reference", "--model", "3b-w2", "--steps", "2", "--warmup", "3", "--prompt", "8"]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _lines(out: str) -> list[dict]:
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def _check(line: dict, n_gpus: int):
    assert line["impl"] == "reference"
    assert line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["n_gpus"] == n_gpus and line["warmup"] == 3
    assert 1 <= line["steps"] <= 2 and line["value"] > 0
    assert abs(line["ms_per_step"] - 1000.0 / line["value"]) < 1e-6 * line["ms_per_step"]
    assert line["vs_baseline"] is None and line["dtype"] == "u2->f32"
    cfg = line["config"]
    assert cfg["workload"] == "qwen2.5-3b-w2-dense-cell" and cfg["prompt"] == 8
    assert cfg["positions"] == "11..12"  # prompt + warm-up steps, then the timed ones
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert "positions 11.." in cb["sample"]
    e2e = line["e2e"]
    assert e2e == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, "bench.py"] + ARGS, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check(lines[0], 1)
    assert lines[0]["config"]["parallelism"] == "replicas x1"


def test_reference_arm_under_torchrun_prints_once():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--gpus", "2"]
    r = subprocess.run(cmd + ARGS, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check(lines[0], 2)
    assert lines[0]["config"]["parallelism"] == "replicas x2"
