"""The bench.py JSON contract, checked on the CPU through the reference arm.

`bench.py --impl reference` times the reference's own CPU MatMulNBits (built from its sources
into oracle/_ref, or the C restatement) and prints the line the driver reads; its keys and
types are the same as the GPU arm's. Under torchrun only rank 0 prints.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(*args, env=None):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, timeout=600,
                       cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    return lines


def test_reference_arm_prints_one_contract_line():
    lines = _run("--impl", "reference", "--steps", "2", "--warmup", "1", "--cpu-seconds", "0")
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key, typ in (("metric", str), ("value", float), ("unit", str), ("n_gpus", int), ("steps", int),
                     ("warmup", int), ("ms_per_step", float), ("higher_is_better", bool), ("scaling", str),
                     ("dtype", str), ("data", str), ("config", dict), ("cpu_baseline", dict), ("e2e", dict)):
        assert isinstance(d[key], typ), key
    assert d["impl"] == "reference" and d["warmup"] >= 3 and d["value"] > 0
    assert d["metric"] == "MatMulNBits INT4 M=1 HBM GB/s" and d["unit"] == "GB/s"
    assert "workload" in d["config"]
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] in ("reference", "port")
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    assert _run("--impl", "reference", "--steps", "1", "--warmup", "1", "--cpu-seconds", "0", env=env) == []


def test_reference_arm_uses_every_host_thread_under_torchrun():
    """torchrun sets OMP_NUM_THREADS=1 for its workers; the reference arm still times the CPU
    kernel on all host threads, so a multi-GPU line is not compared with one CPU thread."""
    env = dict(os.environ, RANK="0", WORLD_SIZE="2", LOCAL_RANK="0", OMP_NUM_THREADS="1")
    d = json.loads(_run("--impl", "reference", "--steps", "1", "--warmup", "1", "--cpu-seconds", "0", env=env)[0])
    assert d["cpu_baseline"]["cores"] == os.cpu_count()
    assert d["scaling"] == "strong"
