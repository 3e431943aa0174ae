"""bench.py's reference arm on the host (no GPU): the JSON line it prints keeps the bench contract.

The reference arm times the reference's own host implementation of the decode products
(oracle/_ref, the reference's gemv_i_thread) on a bounded sample, so it runs here; under torchrun
only rank 0 prints.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libq8ref.so")


def run_bench(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=600)


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="oracle/_ref not built (make -C oracle)")
def test_reference_arm_prints_one_contract_line():
    p = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["warmup"] >= 3  # the contract's minimum, whatever was asked
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_is_silent_on_other_ranks():
    p = run_bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1",
                  env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def check_gpu_line(d: dict) -> None:
    """The keys and relations of the bench line of the B200 arm (one GPU)."""
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "roofline", "e2e", "gpu_launches", "clocks"):
        assert k in d, k
    assert d["n_gpus"] == 1 and d["warmup"] >= 3 and d["value"] > 0 and d["gpu_launches"] > 0
    assert abs(d["value"] - d["config"]["bytes_per_step"] / d["ms_per_step"] / 1e6) <= 0.01 * d["value"]
    r = d["roofline"]
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] > 0
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    assert abs(r["achieved"] - d["value"]) <= 0.01 * d["value"]  # the roofline is the step's (one GPU)
    e = d["e2e"]
    assert e["unit"] == d["unit"] and e["value"] > 0 and e["h2d_bytes_per_step"] > 0 and e["d2h_bytes_per_step"] > 0
    assert {"sm_mhz", "sm_max_mhz", "reasons", "samples"} <= set(d["clocks"])


def test_gpu_line_checker_accepts_a_recorded_line():
    # a line bench.py printed on a B200 (trimmed to the keys the checker reads)
    d = {"metric": "Q8_0 weight-product GB/s, 9B decode step (M=1)", "value": 3700.2, "unit": "GB/s", "n_gpus": 1,
         "steps": 200, "warmup": 5, "ms_per_step": 2.0307, "higher_is_better": True, "scaling": "strong",
         "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": {"workload": "w", "bytes_per_step": 7513769472},
         "roofline": {"bound": "hbm", "achieved": 3700.2, "peak": 6536.4, "unit": "GB/s", "frac": 0.5661},
         "e2e": {"value": 1302.0, "unit": "GB/s", "h2d_bytes_per_step": 3162112, "d2h_bytes_per_step": 4277760},
         "gpu_launches": 51600, "clocks": {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 19}}
    check_gpu_line(d)


@pytest.mark.gpu
def test_bench_one_gpu_line():
    p = run_bench("--steps", "40", "--warmup", "3", "--no-prompt")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    check_gpu_line(json.loads(lines[0]))
