"""bench.py's reference arm runs on the host cores (the oracle port), so its JSON contract is checked here without a
GPU: one line per workload with the keys the driver reads, `impl: reference`, an e2e object with no host copies,
and a cpu_baseline that names its kind, cores and sample. Ranks other than 0 of a multi-rank launch print nothing
and exit 0."""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def run_bench(*args, env=None):
    e = dict(os.environ, **(env or {}))
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], capture_output=True, text=True,
                       timeout=600, cwd=REPO, env=e)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.strip()]


def check_line(r):
    assert KEYS <= set(r), KEYS - set(r)
    assert r["impl"] == "reference"
    assert r["value"] > 0 and r["ms_per_step"] > 0 and r["higher_is_better"] is True
    assert r["e2e"]["h2d_bytes_per_step"] == 0 and r["e2e"]["d2h_bytes_per_step"] == 0
    assert r["e2e"]["value"] == r["value"] and r["e2e"]["unit"] == r["unit"]
    cb = r["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == pytest.approx(r["value"])
    assert r["config"]["workload"]


@pytest.mark.parametrize("workload", ["decode40", "batch64", "prefill4096", "prefill32k"])
def test_reference_arm_line(workload):
    import bench
    args = ("--no-decode40",) if workload == "prefill4096" else ()
    lines = run_bench("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "3", *args)
    assert len(lines) == 1
    check_line(lines[0])
    assert lines[0]["unit"] == "tokens/s"
    # the same config object as the GPU arm at the same N, so the two lines name the same work
    assert lines[0]["config"] == json.loads(json.dumps(bench.workload_config(workload, 1)))


def test_reference_arm_default_is_whole_steps():
    """The default workload (prefill4096) at N=1 times one whole 4096-token layer per step and attaches the
    decode40 arm (whole 40-layer tokens); the ms per step is what was measured (steps x ms fits the run)."""
    import time
    t0 = time.perf_counter()
    lines = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    wall = time.perf_counter() - t0
    assert len(lines) == 1
    r = lines[0]
    check_line(r)
    assert r["config"]["workload"].startswith("configs[3]")
    d = r["decode40"]
    check_line(d)
    assert d["config"]["workload"].startswith("configs[1]")
    assert (r["steps"] + r["warmup"]) * r["ms_per_step"] / 1e3 < wall
    assert (d["steps"] + d["warmup"]) * d["ms_per_step"] / 1e3 < wall


def test_reference_arm_typed_decode():
    lines = run_bench("--impl", "reference", "--workload", "typed-decode", "--ggml-type", "IQ4_XS", "--steps", "1",
                      "--warmup", "3")
    assert len(lines) == 1
    check_line(lines[0])
    assert lines[0]["config"]["ggml_type"] == "IQ4_XS"


def test_reference_arm_other_ranks_are_silent():
    """Under torchrun only rank 0 runs the reference arm; the others exit 0 without work."""
    lines = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3", "--no-decode40",
                      env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert lines == []
