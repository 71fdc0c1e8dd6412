"""bench.py on the CPU: the reference arm's JSON line and rank rule, and how the clock
samples taken during a timed region are matched to the measured device.

The reference arm times the CPU oracle on host cores, so it runs without a GPU; the GPU
arm's line is checked on the B200 by the driver itself.
"""

import datetime
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

REQUIRED = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
            "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def run_bench(*args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert REQUIRED <= set(line)
    assert line["impl"] == "reference"
    assert line["steps"] == 1 and line["warmup"] >= 3  # fewer than 3 warm-up steps are raised to 3
    assert line["higher_is_better"] is True and line["scaling"] == "weak" and line["n_gpus"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    sys.path.insert(0, str(ROOT))
    import bench

    for key, val in bench.decode_config().items():  # the GPU arm's workload, sampled
        assert line["config"][key] == val, key
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert cb["unit"] == line["unit"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3",
                  env_extra={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_clock_samples_follow_the_device_by_pci_bus_id(tmp_path):
    sys.path.insert(0, str(ROOT))
    import bench

    rows = []
    for k, t in enumerate(("05:00:00.100", "05:00:00.200", "05:00:00.300")):
        # nvidia-smi index 0 is another GPU at 1000 MHz; index 1 is this device at 1965 MHz
        rows.append(f"2026/12/02 {t}, 0, 00000000:18:00.0, 1000, 1965, 100.0, 0x0, Not Active, Not Active, "
                    f"Not Active, Not Active")
        rows.append(f"2026/12/02 {t}, 1, 00000000:2A:00.0, {1965 - k}, 1965, 700.0, 0x4, Not Active, Not Active, "
                    f"Not Active, Active")
    ts = [datetime.datetime(2026, 12, 2, 5, 0, 0, 100000 * i).timestamp() for i in (1, 2, 3)]

    def sampler(bus, index):
        s = bench.ClockSampler.__new__(bench.ClockSampler)
        s.index, s.bus, s.proc, s.window = index, bus, None, (ts[0] - 0.01, ts[1] + 0.01)
        s.path = str(tmp_path / f"clocks_{index}_{bus}.csv")
        Path(s.path).write_text("\n".join(rows) + "\n")
        return s

    got = sampler((0, 0x2A, 0), 0).summary()  # CUDA ordinal 0 is nvidia-smi index 1
    assert got["sm_mhz"] == 1964.5 and got["samples"] == 2 and got["reasons"] == ["sw_power_cap"]
    got = sampler(None, 0).summary()  # no bus id: fall back to the ordinal
    assert got["sm_mhz"] == 1000.0 and got["reasons"] == []

