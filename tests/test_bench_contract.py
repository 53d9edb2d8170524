"""The JSON line `bench.py` prints is what a benchmark driver reads: one line
per run, with the keys below. The reference arm (the reference's CPU expert
tier, compiled from its source) runs on the CPU; this library's arm needs a
B200 and runs a short decode workload through the same code as the default
run."""

from __future__ import annotations

import json
import subprocess
import sys

import pytest

from conftest import ROOT


def _json_lines(out: str) -> list[dict]:
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def _run(args: list[str], timeout: int) -> dict:
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = _json_lines(proc.stdout)
    assert len(lines) == 1, proc.stdout[-2000:]
    return lines[0]


def test_reference_arm_line():
    from oracle import nvfp4 as O
    if not O.reference_available():
        pytest.skip("reference CPU tier not built (oracle/_ref)")
    line = _run(["--impl", "reference", "--tokens", "4", "--steps", "2", "--warmup", "1"], 900)
    assert line["impl"] == "reference"
    assert line["metric"] == "routed-expert tokens/s" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["steps"] >= 1 and line["ms_per_step"] > 0
    assert line["config"]["workload"].startswith("config1-decode") and "T=4" in \
        line["config"]["workload"]
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.gpu
def test_b200_arm_line(cuda):
    T = 8
    line = _run(["--tokens", str(T), "--steps", "5", "--warmup", "3", "--no-cpu-baseline",
                 "--no-extras", "--min-timed-s", "0"], 900)
    assert "impl" not in line or line["impl"] != "reference"
    assert line["metric"] == "routed-expert tokens/s" and line["n_gpus"] == 1
    assert line["steps"] == 5 and line["warmup"] == 3
    assert line["device_errors"] == 0 and line["value"] > 0
    assert line["value"] == pytest.approx(T / (line["ms_per_step"] * 1e-3), rel=1e-6)
    r = line["roofline"]
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] > 0
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"], rel=1e-6)
    assert 0 < r["frac"] < 1.2
    e = line["e2e"]
    # bf16 hidden rows up, int32 ids and fp32 weights up, bf16 rows back
    assert e["h2d_bytes_per_step"] == T * 4096 * 2 + T * 8 * 4 * 2
    assert e["d2h_bytes_per_step"] == T * 4096 * 2
    assert e["value"] > 0 and e["unit"] == "tokens/s"
    # the copies overlap the neighbouring steps; the serial form is reported beside them
    assert e["serial_copies"]["ms_per_step"] > 0
    assert line["gpu_launches"] > 0
    clk = line["clocks"]
    assert clk is not None and clk["sm_max_mhz"] > 0
