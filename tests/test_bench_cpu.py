"""bench.py's reference arm on the CPU: the JSON line the driver reads, and
the rank > 0 behaviour under torchrun (exit 0, no output, no work)."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--model", "tiny-llama",
        "--steps", "1", "--warmup", "1", "--cpu-seconds", "1"]


def _env(**kw):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(kw)
    return env


def test_reference_arm_json_line():
    """The reference's own engine (installed under baseline/_ref) on a tiny decoder."""
    r = subprocess.run(ARGS, capture_output=True, text=True, timeout=600, env=_env(), cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if not os.path.isdir(os.path.join(REPO, "baseline", "_ref", "csaq")):
        assert "unavailable" in d
        return
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "CSAQInferenceEngine.generate" in cb["sample"] and "2 layers" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("tiny-llama-shaped decoder")


def test_reference_arm_other_ranks_exit_without_output():
    r = subprocess.run(ARGS, capture_output=True, text=True, timeout=600,
                       env=_env(RANK="1", WORLD_SIZE="2", LOCAL_RANK="1"), cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_cpu_baseline_samples_of_the_kernel_workloads():
    """The host-core legs of the gemm and calib workloads run one pass at budget 0."""
    sys.path.insert(0, REPO)
    import bench
    tf, desc = bench.cpu_gemm_sample(0.0)
    assert tf > 0 and desc.startswith("1 dequantise-then-matmul passes")
    gbs, desc = bench.cpu_salience_sample(0.0)
    assert gbs > 0 and desc.startswith("1 accumulation passes")
