"""The bench.py contract on CPU: the reference arm (the reference's CPU implementation of the path, no GPU needed)
prints one JSON line with the keys the driver reads, and a workload without a timed reference arm says so."""
import json
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _run(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, timeout=240,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_quant_line():
    d = _run("--impl", "reference", "--workload", "quant", "--steps", "3", "--warmup", "3")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_gemm_line():
    d = _run("--impl", "reference", "--workload", "gemm", "--steps", "3", "--warmup", "3")
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
    assert d["config"]["M"] == 8192 and d["config"]["N"] == 14336 and d["config"]["K"] == 4096


def test_reference_arm_unavailable_workload():
    d = _run("--impl", "reference", "--workload", "w4a16", "--steps", "3", "--warmup", "3")
    assert d["impl"] == "reference" and "unavailable" in d
