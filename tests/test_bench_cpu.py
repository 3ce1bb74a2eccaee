"""The benchmark's reference arm runs on the host alone; its JSON line must carry
the keys the benchmark contract names (impl, metric, value, unit, cpu_baseline,
e2e with zero host-device bytes) on a small sample."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--ref-batch", "2"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    lines = [line for line in r.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "GB/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


def test_cpu_baseline_sample_repeats_until_its_minimum_time():
    sys.path.insert(0, str(ROOT))
    import bench

    gbs, seconds, desc = bench.cpu_decode_sample(1, "decode_1b", batch=1, heads=2, min_seconds=0.2)
    assert gbs > 0 and seconds >= 0.2
    assert "passes" in desc
