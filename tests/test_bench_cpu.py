"""CPU tests of bench.py's reference arm, the line the driver reads beside the
GPU arm: for small samples of three workloads, `--impl reference` must print
one JSON line with the workload's metric and unit, impl "reference", a
cpu_baseline describing the run, and an e2e figure equal to the value with no
host-device copies."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_ref(*args):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3",
           *args]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


# --workload name -> the config's workload name
NAMES = {"decode": "sparse_mla_decode", "indexer_prefill": "indexer_prefill", "sparse_prefill": "sparse_prefill",
         "indexer_decode": "indexer_decode", "shard_merge": "shard_merge", "decode_layer": "decode_layer",
         "shard_merge_p2p": "shard_merge_p2p", "dsa_layer": "dsa_decode_layer"}


@pytest.mark.parametrize("workload,extra,unit", [
    ("decode", ["--ctx", "4096", "--cpu-rows", "1"], "tok/s"),
    ("indexer_decode", ["--ctx", "4096", "--cpu-rows", "1"], "tok/s"),
    ("shard_merge", ["--cpu-rows", "16"], "rows/s"),
    ("decode_layer", ["--ctx", "4096", "--cpu-rows", "1"], "tok/s"),
    ("dsa_layer", ["--ctx", "4096", "--cpu-rows", "1"], "tok/s"),
])
def test_reference_arm_json_line(workload, extra, unit):
    d = run_ref("--workload", workload, *extra)
    assert d["impl"] == "reference" and d["unit"] == unit and d["n_gpus"] == 1
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"] == NAMES[workload]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_workloads_registered_with_configs():
    sys.path.insert(0, ROOT)
    import bench

    assert set(bench.WORKLOADS) == set(NAMES)
    for name, cls in bench.WORKLOADS.items():
        wl = cls()
        cfg = wl.config()
        assert cfg["workload"] == NAMES[name]
        assert "model" not in cfg
        assert wl.metric and wl.unit
