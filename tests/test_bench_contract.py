"""bench.py's output contract, checked on the arm that runs without a GPU: the
reference arm (`--impl reference`) times the reference's own CPU moe_forward
and prints one JSON line with the same metric, unit and config keys as the
GPU arm; under torchrun only rank 0 prints."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=600)


def test_reference_arm_prints_one_contract_line(built):
    import bench
    p = _run()
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout
    r = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in r, key
    assert r["impl"] == "reference" and r["metric"] == bench.METRIC and r["unit"] == bench.UNIT
    assert r["value"] > 0 and r["steps"] == 1 and r["n_gpus"] == 1 and r["higher_is_better"] is True
    assert r["config"] == bench.bench_config(1)  # the GPU arm's config block
    assert r["sample_tokens_per_step"] >= 1
    cb = r["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == r["value"]
    assert r["e2e"] == {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only(built):
    p = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [l for l in p.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_loads_nothing_of_the_product(built):
    """The reference arm builds its inputs with the checkers' generator and
    times the reference build: neither the qmoe binding nor libqmoe.so may be
    loaded in its process."""
    code = (
        "import runpy, sys, json\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1']\n"
        f"runpy.run_path({os.path.join(ROOT, 'bench.py')!r}, run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'qmoe': 'qmoe' in sys.modules, 'lib': 'libqmoe' in maps,\n"
        "                  'ref': 'libmoe_ref' in maps or 'liboracle' in maps}))\n")
    p = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert r == {"qmoe": False, "lib": False, "ref": True}
