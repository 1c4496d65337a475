"""The benchmark's reference arm runs the reference's own CPU operators and
nothing of this library: after a short run, libkllm_b200.so must not be
mapped into the process (the arm imports only the workload shapes)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROBE = r"""
import io, json, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"]
import bench
buf = io.StringIO()
bench._JSON_OUT = buf
bench.run_reference(bench.parse_args())
maps = open("/proc/self/maps").read()
line = json.loads(buf.getvalue().splitlines()[-1])
print(json.dumps({"mapped_product": "libkllm_b200" in maps, "torch": "torch" in sys.modules,
                  "line": line}))
"""


def _reference_built() -> bool:
    return os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libkllm_ref.so"))


@pytest.mark.skipif(not _reference_built(), reason="oracle/_ref (the compiled reference) is not built")
def test_reference_arm_does_not_map_the_product_library():
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", PROBE], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["mapped_product"] is False
    assert out["torch"] is False
    line = out["line"]
    assert line["impl"] == "reference"
    assert line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference"


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun only rank 0 runs the reference arm; every other rank exits
    0 at once, prints no line and joins no process group."""
    env = dict(os.environ, PYTHONPATH=ROOT, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2",
               MASTER_ADDR="127.0.0.1", MASTER_PORT="1")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
