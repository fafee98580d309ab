"""Build the CUDA library in-tree: libcusort_b200/_lib/libcusort_b200.so.

Every .cu under csrc/ is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) in parallel, then linked into one
shared library with the CUDA runtime linked statically and NCCL dynamically.
Run as ``python -m libcusort_b200.build`` or through ``__graft_entry__.build()``.

Environment CUSORT_NVCC_DEFINES adds preprocessor definitions to every
compile (e.g. ``-DCUSORT_LOOKBACK_TIMER=1`` for the lookback-timer build that
``bench.py --lookback-stall`` reads); the definitions of the last build are
kept beside the library, so a change of them forces a rebuild.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
OBJ_DIR = PKG / "_build"
LIB = OUT_DIR / "libcusort_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr"]
STAMP = OUT_DIR / "defines.txt"


def extra_defines() -> list[str]:
    """-D flags from CUSORT_NVCC_DEFINES (anything else there is rejected)."""
    flags = os.environ.get("CUSORT_NVCC_DEFINES", "").split()
    bad = [f for f in flags if not f.startswith("-D")]
    if bad:
        raise ValueError(f"CUSORT_NVCC_DEFINES takes -D flags only, got {bad}")
    return flags


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def nccl_flags() -> list[str]:
    """Header + library location of NCCL (system install)."""
    inc = []
    for d in ("/usr/include", "/usr/local/cuda/include"):
        if Path(d, "nccl.h").exists():
            inc = ["-I" + d]
            break
    return inc


def _compile(src: Path, verbose: bool) -> tuple[Path, str]:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra_defines(), *nccl_flags(), "-Xptxas", "-v", "-c", str(src), "-o",
           str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    return obj, r.stderr


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    if (STAMP.read_text() if STAMP.exists() else "") != " ".join(extra_defines()):
        return False
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [PKG.parent / "include" / "cusort_b200.h", Path(__file__)]
    return all(p.stat().st_mtime <= t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    OBJ_DIR.mkdir(exist_ok=True)
    srcs = sources()
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = []
        for obj, log in ex.map(lambda s: _compile(s, verbose), srcs):
            objs.append(obj)
            logs.append(log)
    (OBJ_DIR / "ptxas.log").write_text("".join(logs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lnccl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    STAMP.write_text(" ".join(extra_defines()))
    if verbose:
        print("".join(logs))
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
