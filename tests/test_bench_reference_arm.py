"""bench.py --impl reference on CPU: the reference arm runs without the
product library, uses every core of its affinity (whatever OMP_NUM_THREADS
says), and under torchrun only rank 0 works."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CMD = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--experts", "16", "--m", "8",
       "--steps", "1", "--warmup", "1"]


def test_reference_arm_loads_no_product_library():
    env = dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(CMD, env=env, capture_output=True, text=True, timeout=600, check=True)
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert not any("libb200moe" in p for p in line["libraries_loaded"]), line["libraries_loaded"]
    assert any("libcpumoe" in p for p in line["libraries_loaded"])
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(CMD, env=env, capture_output=True, text=True, timeout=120, check=True)
    assert r.stdout.strip() == ""
