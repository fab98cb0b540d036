"""bench.py's contract with the driver, checked without a GPU: the
configurations the default run also measures resolve to workloads, and the
reference arm prints one JSON line with the keys the driver reads."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_side_configs_resolve_to_workloads():
    import bench
    assert bench.SIDE_CONFIGS, "the default run measures the other configurations too"
    for name, overrides in bench.SIDE_CONFIGS:
        cls = bench.CONFIGS[name.split("_")[0]]
        for attr in ("batch", "workload", "step", "dominant", "cpu_sample"):
            assert hasattr(cls, attr), (name, attr)
        assert set(overrides) <= {"dtype", "width"}, name


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "cfg1", "--steps", "1",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["config"]["global_batch"] == d["config"]["per_gpu_batch"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference")
