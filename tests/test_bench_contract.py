"""CPU: bench.py's reference arm prints the contract's JSON line (the
product arm needs a GPU and is exercised by the round-end bench run)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "gpu_launches"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["gpu_launches"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["config"]["m"] == 8192


def test_roofline_denominator_follows_the_timed_region():
    """20 steps of 8192^3 (~16 ms) compare with the burst peak, a ~1 s loop
    with the sustained one (the power cap has settled the clock by then)."""
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.roofline_denominator(0.016, 1655.2, 1386.1) == (1655.2, True)
    assert bench.roofline_denominator(0.9, 1655.2, 1386.1) == (1386.1, False)
    assert bench.roofline_denominator(0.9, 1655.2, None) == (1655.2, True)
