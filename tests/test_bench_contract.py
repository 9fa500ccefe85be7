"""The reference arm of bench.py on the host (no GPU): one timed step of the
reference's CPU path through `bench.py --impl reference`, checked for the
JSON line the driver reads and for the libraries the process loaded -- the
reference's compiled kernels (or the oracle port), never this repository's
CUDA library or the CUDA runtime."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

DRIVER = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
libs = sorted({l.split()[-1] for l in maps.splitlines() if l.split()[-1].endswith(".so") or ".so." in l.split()[-1]})
print("LIBS " + json.dumps(libs))
"""


def test_reference_arm_line_and_libraries():
    out = subprocess.run([sys.executable, "-c", "import json\n" + DRIVER], cwd=ROOT, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    libs = json.loads(lines[-1][len("LIBS "):])
    line = json.loads(next(l for l in reversed(lines) if l.startswith("{")))
    assert line["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3
    assert line["config"]["seq_len"] == 128  # the GPU arm's prompt
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"]
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["unit"] == line["unit"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    names = [os.path.basename(p) for p in libs]
    assert not any(n.startswith("libq35b") for n in names), names
    assert not any(n.startswith("libcudart") or n.startswith("libcuda.") for n in names), names
    if cb["kind"] == "reference":
        assert any(n.startswith("libq35ref") for n in names), names


def test_reference_arm_under_torchrun_prints_once():
    """launched as the driver launches N > 1 (torchrun, two ranks on this
    host): rank 0 alone runs and prints its line, the other rank exits 0
    without work; no process group is needed for it"""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "3"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    assert lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2 and lines[0]["value"] > 0
