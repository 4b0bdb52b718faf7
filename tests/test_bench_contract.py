"""The parts of bench.py's output contract that run without a GPU.

* The reference arm (``--impl reference``): the reference's CPU attention
  (the oracle port) timed on the host cores, printed as one JSON line with
  the keys the driver reads (metric, value, unit, higher_is_better,
  cpu_baseline describing the run, e2e with no copies).
* The roofline peak follows the regime the clock record shows: the burst
  bf16 figure when the SM clock held its maximum with no power capping, the
  sustained figure otherwise.
"""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0", "--skip-reference-gpu"],
        capture_output=True, text=True, check=True, timeout=600, cwd=str(ROOT)).stdout
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s"
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_roofline_peak_follows_the_clock_regime():
    pk = {"bf16_tflops": 1667.9, "bf16_tflops_sustained": 1387.1}
    at_max = {"sm_mhz": 1965, "sm_max_mhz": 1965, "reasons": []}
    capped = {"sm_mhz": 1965, "sm_max_mhz": 1965, "reasons": ["sw_power_cap"]}
    slow = {"sm_mhz": 1500, "sm_max_mhz": 1965, "reasons": []}
    assert bench.tensor_peak(pk, "measured", at_max) == (1667.9, "bf16_tflops (measured)")
    assert bench.tensor_peak(pk, "measured", capped)[0] == 1387.1
    assert bench.tensor_peak(pk, "measured", slow)[0] == 1387.1
    # a peaks file without the sustained figure falls back to the stated one
    assert bench.tensor_peak({"bf16_tflops": 1600.0}, "measured", capped)[0] == \
        bench.FALLBACK_PEAKS["bf16_tflops_sustained"]
