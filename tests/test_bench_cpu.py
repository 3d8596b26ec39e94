"""bench.py's reference arm on the host CPU: the contract line it prints, that
it loads no library code, and that under torchrun only rank 0 works."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

# runs bench.py as __main__, then reports whether the CUDA library was loaded
_RUNNER = (
    "import runpy, sys\n"
    "sys.argv = ['bench.py'] + sys.argv[1:]\n"
    "runpy.run_path('bench.py', run_name='__main__')\n"
    "print('LIBRARY-LOADED' if 'moe_serving_profile_b200._lib' in sys.modules else 'LIBRARY-NOT-LOADED')\n"
)


def _run(args, rank="0"):
    env = dict(os.environ, RANK=rank, WORLD_SIZE="2" if rank != "0" else "1")
    return subprocess.run([sys.executable, "-c", _RUNNER] + args, cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=300)


def test_reference_arm_prints_a_contract_line():
    r = _run(["--impl", "reference", "--workload", "qwen3-tiny", "--steps", "2", "--warmup", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert lines[-1] == "LIBRARY-NOT-LOADED"
    line = json.loads(lines[-2])
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 2 and line["warmup"] == 1
    assert line["config"]["workload"] == "qwen3-tiny"
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and "T=64" in cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    r = _run(["--impl", "reference", "--workload", "qwen3-tiny", "--steps", "1", "--warmup", "0"], rank="1")
    assert r.returncode == 0, r.stderr[-2000:]
    assert [ln for ln in r.stdout.splitlines() if ln.strip()] == ["LIBRARY-NOT-LOADED"]
