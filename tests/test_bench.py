"""bench.py's output contract: one JSON line with the keys the driver reads.

CPU: the reference arm (the oracle on host cores) on a small sample, argument
validation and the byte-counting helpers. GPU: this build's arm on a small
batch (roofline, clocks and launch count present and consistent).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import REPO, gpu_available

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
             "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


def _run(args, timeout=600):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py")] + args,
                         capture_output=True, text=True, timeout=timeout, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    line = _run(["--impl", "reference", "--steps", "1", "--warmup", "0", "--log-n", "8",
                 "--batch", "64"])
    assert BASE_KEYS <= set(line)
    assert line["impl"] == "reference" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["unit"] == "GB/s"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["config"]["n"] == 256 and line["config"]["batch_per_gpu"] == 64


def test_reference_arm_2d_and_multipass():
    l2 = _run(["--impl", "reference", "--kind", "2d", "--log-n", "5", "--batch", "2", "--steps",
               "1", "--warmup", "0"])
    assert l2["metric"].startswith("batched 2D") and "2 pass(es)" in l2["config"]["bytes_counted"]
    l1 = _run(["--impl", "reference", "--log-n", "16", "--batch", "2", "--steps", "1",
               "--warmup", "0"])
    assert "2 pass(es)" in l1["config"]["bytes_counted"]


def test_argument_validation():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--kind", "2d",
                          "--log-n", "15"], capture_output=True, text=True, cwd=REPO)
    assert out.returncode != 0 and "--kind 2d needs --log-n <= 14" in out.stderr


def test_byte_counting_helpers():
    sys.path.insert(0, REPO)
    import bench

    assert bench.passes_counted("1d", 12) == 1
    assert bench.passes_counted("1d", 20) == 2
    assert bench.passes_counted("2d", 12) == 2
    assert bench.elems_per_item(12, "2d") == 1 << 24
    assert "fft_rows_pf_kernel<14" in bench.rows_kernel_name(14)
    assert "fft_rows_kernel<12,4" in bench.rows_kernel_name(12)
    cfg = bench.workload_config(12, 65536)
    assert "2048 MiB" in cfg["l2"] and cfg["n"] == 4096


@pytest.mark.gpu
def test_gpu_arm_line():
    if not gpu_available():
        pytest.skip("no B200")
    line = _run(["--steps", "3", "--warmup", "3", "--batch", "4096", "--no-e2e",
                 "--no-cpu-baseline", "--no-extras"])
    assert BASE_KEYS <= set(line)
    assert line["n_gpus"] == 1 and line["gpu_launches"] == 6
    rf = line["roofline"]
    assert rf["bound"] == "hbm" and rf["unit"] == "GB/s" and 0 < rf["frac"] < 1.5
    assert abs(rf["frac"] - rf["achieved"] / rf["peak"]) < 1e-3
    assert line["clocks"]["sm_max_mhz"] is None or line["clocks"]["sm_max_mhz"] > 0
    assert line["roundtrip_max_rel_err"] < 1e-4
