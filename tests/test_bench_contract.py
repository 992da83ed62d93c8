"""The bench's CPU-side contract: the reference arm (``--impl reference``, the
oracle port timed on the host cores) prints one JSON line with every key the
driver reads; under a multi-rank launch only rank 0 runs and prints; fewer
than 3 warm-up steps are refused; both arms describe a workload with the same
``config`` dict; the default workload's 512 requests shard with equal counts."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")


def run(args, env_extra=None, timeout=900):
    env = {**os.environ, **(env_extra or {})}
    return subprocess.run([sys.executable, BENCH, *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_warmup_below_three_is_refused():
    p = run(["--impl", "reference", "--warmup", "2"])
    assert p.returncode == 2 and "--warmup must be at least 3" in p.stderr


def test_reference_arm_other_ranks_exit_quietly():
    p = run(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"],
            {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [line for line in p.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_the_contract_line():
    # the config-2 line (the default config-5 sample builds a 770M-parameter drafter on the host)
    p = run(["--impl", "reference", "--workload", "config2", "--steps", "1", "--warmup", "3", "--cpu-seconds", "0.5"],
            {"RANK": "0", "WORLD_SIZE": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [line for line in p.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["higher_is_better"] is True and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"].startswith("config2")


def test_both_arms_print_the_same_config_and_the_default_shards_evenly():
    import argparse
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", BENCH)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    from flashmap_b200.sharding import balanced_capacity, lpt_assign, request_costs

    for world in (1, 2, 4, 8):
        args = argparse.Namespace(workload="all", launch="auto", profile_small=False)
        a, b = bench.workload_config(args, world), bench.workload_config(args, world)
        assert a == b and a["requests"] == 512 and a["workload"].startswith("config5")
        lengths = bench.shard_lengths()
        assert len(lengths) == 512 and min(lengths) >= 1024 and max(lengths) <= 8192
        shares = lpt_assign(request_costs(lengths), world, balanced_capacity(512, world))
        assert sorted(i for s in shares for i in s) == list(range(512))
        assert {len(s) for s in shares} == {512 // world}
