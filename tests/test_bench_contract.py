"""The benchmark's reference arm on the CPU: `bench.py --impl reference` prints one JSON line with
the driver's keys, the same workload `config` as the GPU arm, a `cpu_baseline` describing the run
and an `e2e` object with no host<->device bytes (the reference arm runs on the host cores).
A small kv_len keeps the run to a second or two."""
import json
import subprocess
import sys

from conftest import ROOT

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _run(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_json_contract():
    import bench

    d = _run("--impl", "reference", "--steps", "2", "--warmup", "1", "--kv-len", "4096")
    assert REQUIRED <= set(d)
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["metric"] == bench.METRIC and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    # the same workload description as the GPU arm's line, so the driver compares like with like
    assert d["config"] == bench.workload_config(4096, 1)
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["unit"] == "GB/s"
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_only_rank0_prints():
    """Under torchrun the other ranks exit 0 without work or output."""
    import os

    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup",
                          "0", "--kv-len", "1024"], cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
