"""bench.py's reference arm on the CPU: it runs the reference's own float32 forward (transformers
5.5.0 Qwen3_5TextModel, the module the reference's engine calls) on one bounded sample and prints
the one JSON line the driver parses, with the keys its contract names."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "requests/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0 and d["scaling"] == "strong"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "requests/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_cpu_sample_is_length_stratified_and_prefix_balanced():
    sys.path.insert(0, ROOT)
    import bench
    from fastdecisions_b200 import workloads as W
    reqs = W.config5_requests(256)
    ids = bench.cpu_sample_ids(reqs)
    lens = [reqs[i].ids.size for i in ids]
    assert len(set(ids)) == len(ids) >= 12 and max(lens) <= 2048
    assert min(lens) < 150 and max(lens) > 1000          # spans the length mix
    assert min(lens[:4]) < 400 and max(lens[:4]) > 700   # a short prefix already spans it
    assert ids == bench.cpu_sample_ids(reqs)             # deterministic


def test_parity_summary():
    sys.path.insert(0, ROOT)
    import numpy as np
    import bench
    ref = {0: np.array([0.5, 0.5, 0.0]), 3: np.array([0.2, 0.7, 0.1])}
    ours = {0: np.array([0.52, 0.48, 0.0]), 3: np.array([0.2, 0.69, 0.11]), 5: np.array([1.0, 0.0, 0.0])}
    p = bench.parity_summary(ours, ref)
    assert p["n"] == 2 and p["argmax_agree"] == "2/2"
    assert abs(p["max_dp_pp"] - 2.0) < 1e-9 and abs(p["mean_dp_pp"] - 1.5) < 1e-9
