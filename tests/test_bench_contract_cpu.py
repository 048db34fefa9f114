"""The reference arm of bench.py (the CPU restatement of the host reference,
timed on this machine's cores) keeps the bench line contract: one JSON line
with the BASELINE metric, a cpu_baseline block and a zero-copy e2e block;
under torchrun only rank 0 prints, and torchrun's OMP_NUM_THREADS=1 does not
shrink the sample to one core."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_reference(extra_env):
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env.update(extra_env)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--config", "2", "--steps", "1", "--warmup", "1"],
                          capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)


def test_reference_arm_line():
    with open(os.path.join(ROOT, "BASELINE.json")) as fh:
        metric = json.load(fh)["metric"]
    res = run_reference({"OMP_NUM_THREADS": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == metric
    assert line["unit"] == "GB/s" and line["value"] > 0 and line["higher_is_better"] is True
    cpu = line["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cpu)
    assert cpu["kind"] == "port" and cpu["value"] == line["value"]
    assert cpu["cores"] == len(os.sched_getaffinity(0))
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["config_index"] == 2


def test_reference_arm_other_ranks_print_nothing():
    res = run_reference({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""


def test_both_arms_build_the_same_config():
    """The GPU arm and the reference arm print the same `config` object for
    the same flags (both call bench.config_dict), at every world size."""
    import argparse
    sys.path.insert(0, ROOT)
    import bench
    res = run_reference({"WORLD_SIZE": "4", "RANK": "0", "LOCAL_RANK": "0"})
    assert res.returncode == 0, res.stderr[-2000:]
    ref = json.loads(res.stdout.strip().splitlines()[-1])["config"]
    args = argparse.Namespace(config=2, partitioned=False)
    assert ref == bench.config_dict(args, dict(bench.CONFIGS[2]), 4)
    for world in (1, 2, 8):
        c5 = bench.config_dict(argparse.Namespace(config=5, partitioned=False), dict(bench.CONFIGS[5]), world)
        assert c5["elements_total"] == 1 << 32 and c5["elements_per_gpu"] == (1 << 32) // world
        assert c5["parallelism"] == ("single" if world == 1 else f"partitioned1d{world}")
