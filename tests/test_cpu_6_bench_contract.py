"""bench.py's reference arm on the host: one JSON line with the keys the
benchmark contract names, for both workloads (the reference's kernels compiled
for the host, a few small steps)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("model,unit", [("build_model", "images/s"), ("uwb_loc_v3", "samples/s")])
def test_reference_arm_json_line(model, unit):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--model", model,
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0 and d["steps"] == 1
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"]
    assert d["config"] == _config(model)
    assert d["cpu_baseline"]["cores"] == _host_cores()


def _config(model):
    sys.path.insert(0, str(ROOT))
    import bench
    return bench.config_of(bench.workload(False, model), 1)


def _host_cores():
    import os
    return len(os.sched_getaffinity(0))


def test_reference_arm_loads_no_gpu_code():
    """The reference arm builds its weights in numpy: neither this repository's
    package nor its CUDA library is loaded, and the thread count is every host
    core even when a launcher exported OMP_NUM_THREADS=1."""
    code = ("import sys; sys.path.insert(0, '.'); import bench; "
            "r = bench.cpu_reference_steps(False, 2, 1, 0); "
            "maps = open('/proc/self/maps').read(); "
            "print(r[1], 'opencl_tf' in sys.modules, 'libb2ocl' in maps)")
    import os
    env = dict(os.environ, OMP_NUM_THREADS="1")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    cores, pkg, lib = out.stdout.split()[-3:]
    assert int(cores) == _host_cores()
    assert pkg == "False" and lib == "False"
