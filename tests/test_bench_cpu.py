"""The benchmark's host-side contract, without a GPU: the roofline arithmetic,
the choice of the tensor peak from the clock record, and the JSON lines of the
two CPU reference arms (headline and routed workloads)."""

import json
import math
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_roofline_terms_of_the_headline_workload():
    c = bench.CFG
    flops, nbytes = bench.roofline_terms(c["B"], c["H"], c["N"], c["M"], c["d"], c["k"], 2)
    # the dense affinity of 128 slices of 16384 x 16384 x 64
    assert flops == 2.0 * 16384 * 16384 * 64 * 128
    assert math.isclose(flops / 1e12, 4.398, rel_tol=1e-3)
    # read Q, K, V, dO; write O, dQ, dK, dV (bf16); int32 indices and fp32 LSE
    assert nbytes == ((5 * 16384 + 6 * 16384) * 64 * 2 + 8 * 16384 * 65) * 128
    assert math.isclose(nbytes / 1e9, 4.04, rel_tol=2e-3)


@pytest.mark.parametrize("clocks, key", [
    ({"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}, "bf16_tflops"),
    ({"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}, "bf16_tflops_sustained"),
    ({"sm_mhz": 1300.0, "sm_max_mhz": 1965.0, "reasons": []}, "bf16_tflops_sustained"),
    ({"samples": 0}, "bf16_tflops"),
])
def test_tensor_peak_follows_the_clock_record(clocks, key):
    assert bench.tensor_peak_key(clocks) == key


def test_peaks_and_traffic_files_parse():
    peaks = bench.load_peaks()
    assert peaks["hbm_gbs"] > 0 and peaks["bf16_tflops"] >= peaks["bf16_tflops_sustained"] > 0
    traffic = bench.load_traffic()
    assert traffic.get("forward_B16_H8_N16384_k64", 0) > 1.6e9  # at least the compulsory bytes


def _json_line(args, timeout=600):
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                         timeout=timeout, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


def _check_reference_line(line, metric):
    assert line["impl"] == "reference" and line["metric"] == metric
    assert line["value"] > 0 and line["unit"] == bench.UNIT and line["higher_is_better"] is True
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": bench.UNIT, "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["steps"] == 1 and line["warmup"] == 3  # the warm-up is raised to the minimum of 3


def test_reference_arm_prints_one_contract_line():
    line = _json_line(["--impl", "reference", "--steps", "1", "--warmup", "0", "--ref-rows", "8"])
    _check_reference_line(line, bench.METRIC)
    assert line["config"]["workload"] == bench.WORKLOAD and line["config"]["sample_rows"] == 8


def test_routed_reference_arm_prints_one_contract_line():
    line = _json_line(["--workload", "routed", "--impl", "reference", "--steps", "1", "--warmup", "0"])
    _check_reference_line(line, bench.ROUTED_METRIC)
    assert line["config"]["workload"] == bench.ROUTED_WORKLOAD
