"""Build the sm_100a shared library ``pagelora_b200/lib/libpagelora_b200.so``.

The library is compiled in-tree with nvcc (no torch headers, no JIT cache):
every ``csrc/*.cu`` file is compiled for ``compute_100a``/``sm_100a`` and
linked into one shared object exporting the C ABI of
``include/pagelora_b200.h``.  ``python -m pagelora_b200.build`` rebuilds it;
``ensure_built()`` rebuilds only when a source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC_DIR = PKG_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libpagelora_b200.so"
OBJ_DIR = LIB_DIR / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=default",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _inputs() -> list[Path]:
    return sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def _obj_stale(src: Path, obj: Path, flags_file: Path, flags: str) -> bool:
    """An object is rebuilt when missing, older than its source or any shared
    header, or built with other flags."""

    if not obj.exists() or not flags_file.exists() or flags_file.read_text() != flags:
        return True
    built = obj.stat().st_mtime
    headers = sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))
    return any(p.stat().st_mtime > built for p in [src, *headers])


def build(verbose: bool = False, extra_flags: list[str] | None = None, *, force: bool = False) -> Path:
    """Compile all CUDA sources into the shared library and return its path.

    Each source is compiled to its own object file (in parallel: the files
    share no device symbols; objects newer than their inputs are kept unless
    ``force``), then nvcc links them into one shared object."""

    LIB_DIR.mkdir(parents=True, exist_ok=True)
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]
    objs, jobs = [], []
    for src in sources():
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [_nvcc(), *ARCH_FLAGS, *compile_flags, *(extra_flags or []), f"-I{INCLUDE_DIR}", "-c", "-o", str(obj),
               str(src)]
        flags_file = obj.with_suffix(".flags")
        objs.append(obj)
        if force or _obj_stale(src, obj, flags_file, " ".join(cmd)):
            jobs.append((cmd, flags_file))
    workers = max(1, min(len(jobs), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        logs = list(pool.map(lambda job: _run(job[0], verbose), jobs))
    for cmd, flags_file in jobs:
        flags_file.write_text(" ".join(cmd))
    if verbose:
        for log in logs:
            if log.strip():
                print(log, flush=True)
    _run([_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *(str(obj) for obj in objs)], verbose)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def ensure_built() -> Path:
    if is_stale():
        build()
    return LIB_PATH


if __name__ == "__main__":
    flags = ["-Xptxas", "-v"] if "--ptxas-info" in sys.argv else None
    print(build(verbose=True, extra_flags=flags, force="--force" in sys.argv))
