"""The C++ drop-in header (include/cusort_b200.cuh): every public template
instantiates and links against libcusort_b200 (CPU: compile and link only);
on a GPU the program runs every form on a small array and exits 0."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "cxx" / "header_use.cu"


def _build(tmp_path) -> Path:
    from libcusort_b200 import build as B
    lib = B.build()
    exe = tmp_path / "header_use"
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-I", str(ROOT / "include"), str(SRC),
           "-o", str(exe), "-L", str(lib.parent), "-lcusort_b200", f"-Xlinker=-rpath={lib.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


def test_header_compiles_and_links(tmp_path):
    assert _build(tmp_path).exists()


@pytest.mark.gpu
def test_header_program_runs(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    r = subprocess.run([str(_build(tmp_path))], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
