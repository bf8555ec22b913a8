"""CPU: the reference arm of bench.py prints one JSON line with the contract's keys.

The reference arm times the reference's CPU path for this hot path (its fp32 math-SDPA
parity oracle) on the host cores; here it runs on a small sequence so the test is quick.
"""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--S", "256",
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert "sampled" in d["config"]["workload"]


def test_warmup_below_three_is_rejected():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode != 0 and "warmup" in out.stderr
