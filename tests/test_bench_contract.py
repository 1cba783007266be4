"""bench.py's reference arm (CPU only): the JSON line the driver reads, and the silent exit of ranks
other than 0 under torchrun. The GPU arm's line is checked by the GPU runs of bench.py itself."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra: dict, *args: str) -> subprocess.CompletedProcess:
    env = {**os.environ, **env_extra}
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def _json_lines(out: str) -> list[dict]:
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def test_reference_arm_line():
    sys.path.insert(0, ROOT)
    import bench

    p = _run({"RANK": "0", "WORLD_SIZE": "1"}, "--impl", "reference", "--steps", "1", "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = _json_lines(p.stdout)
    assert len(lines) == 1, p.stdout
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True  # the default workload is M = 8192
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] >= 1
    assert d["config"] == bench.workload_config("mlp_up_prefill", 8192, 1)  # the GPU arm's config object
    assert (d["config"]["m"], d["config"]["n"], d["config"]["k"]) == (8192, 57344, 8192)
    assert d["config"]["parallelism"] == "column-parallel N/1"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_silently():
    p = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--impl", "reference", "--steps", "1",
             "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    assert _json_lines(p.stdout) == []


def test_reference_arm_sharded_config_matches():
    """Under torchrun with 2 ranks, rank 0's line names the per-rank shard like the GPU arm does."""
    sys.path.insert(0, ROOT)
    import bench

    p = _run({"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"}, "--impl", "reference", "--steps", "1", "--warmup",
             "0", "--workload", "mlp_up_decode")
    assert p.returncode == 0, p.stderr[-2000:]
    (d,) = _json_lines(p.stdout)
    assert d["config"] == bench.workload_config("mlp_up_decode", 1, 2)
    assert d["config"]["n_per_gpu"] == 57344 // 2 and d["n_gpus"] == 2 and d["unit"] == "TB/s"
