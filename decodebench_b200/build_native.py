"""Build the sm_100a kernel library ``decodebench_b200/_lib/libdbk.so`` in-tree.

Each ``csrc/*.cu`` is compiled separately (in parallel) with relocatable device
code, then device-linked into one shared library exporting the C ABI declared in
``include/dbk.h``. Run ``python -m decodebench_b200.build_native`` or call
:func:`build`; nvcc cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libdbk.so"
OBJ_DIR = ROOT / "_build" / "obj"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the decodebench_b200 kernels need CUDA 12.8+")


def _flags(verbose: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC",
                "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}"]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), ROOT / "include" / "dbk.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    srcs = _sources()
    objs = [OBJ_DIR / (s.stem + ".o") for s in srcs]

    def compile_one(pair):
        src, obj = pair
        if not force and not _stale(obj, src):
            return ""
        cmd = [cc, *_flags(verbose), "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        logs = list(ex.map(compile_one, zip(srcs, objs)))
    if verbose:
        for s, log in zip(srcs, logs):
            if log:
                print(f"== {s.name}\n{log}", file=sys.stderr)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objs),
               "-o", str(LIB), "-lcudart", "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
