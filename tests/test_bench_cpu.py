"""bench.py on CPU: the reference arm's JSON line carries the driver contract's keys, and the
algorithmic byte counts behind every roofline are the per-token formulas of the path."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_step_bytes_per_token_matches_the_configs():
    # fwd x, z in and y out; bwd dy, x, z in and dx, dz out; alpha written and read: 2 (5D + 3Dz) + 4K
    assert bench.step_bytes_per_token(2048, 2048, 16) == 32832    # config 2
    assert bench.step_bytes_per_token(4096, 4096, 32) == 65664    # config 5
    c = dict(D=2048, Dz=2048, K=16)
    assert bench.KERNEL_BYTES_PER_TOKEN["conv_backward"](c) == 6 * 2048 + 4 * 16
    assert bench.KERNEL_BYTES_PER_TOKEN["conv_forward"](c) == 4 * 2048 + 2 * 16


def test_decode_bytes_per_step_is_the_cache_and_state_traffic():
    c = bench.DECODE
    B, Dz, K, S = c["B"], c["Dz"], c["K"], c["S"]
    want = 0
    for _, D, _ in c["modules"]:
        want += 2 * B * (D + Dz + D + (S - 1) * D + S * D) + 2 * K * S * D + 2 * K * Dz
    assert bench.decode_bytes_per_step(c) == want


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT, check=True)
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"].startswith("config2")
