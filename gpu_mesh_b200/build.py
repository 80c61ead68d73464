"""Build the stage executor's CUDA library (sm_100a) in-tree.

``python -m gpu_mesh_b200.build`` compiles every ``csrc/*.cu`` into
``gpu_mesh_b200/lib/libmeshgpu_b200.so`` with nvcc.  Objects are cached under
``gpu_mesh_b200/lib/obj`` and rebuilt when a source or header is newer.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = LIB_DIR / "obj"
LIB_PATH = LIB_DIR / "libmeshgpu_b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the stage library")
    return cand


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    objs = []
    todo = []
    for src in sources:
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            todo.append((src, obj))

    def compile_one(item: tuple[Path, Path]) -> None:
        src, obj = item
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")

    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(compile_one, todo))
    if todo or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objs), "-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
