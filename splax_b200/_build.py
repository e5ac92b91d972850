"""Build libsplax_b200.so (the CUDA kernels and the C ABI) in-tree with nvcc for sm_100a.

The files whose float arithmetic feeds integer outputs (project.cu, sort.cu) compile with
--fmad=false and IEEE division / square root, so tile counts, radii and sort keys reproduce
the C oracle bit for bit; the blend kernels keep FMA contraction. The CUDA runtime is linked
statically, so the library runs next to any torch build in the same process.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD_DIR = PKG / "_build"
LIB_PATH = PKG / "libsplax_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
          f"-I{INCLUDE}"]
EXACT = ["--fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false"]
SOURCES = {
    "project.cu": EXACT,
    "sort.cu": EXACT,
    "raster_fwd.cu": [],
    "raster_bwd.cu": [],
    "capi.cu": [],
    "project_noalloc.cu": [],
    "loss.cu": [],
    "ssim.cu": [],
    "optim.cu": [],
    "ply.cu": [],
    "collective.cu": [],
}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def _deps() -> list[Path]:
    return [*CSRC.glob("*.cu"), *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    newest = max(p.stat().st_mtime for p in _deps())
    return LIB_PATH.stat().st_mtime >= newest


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every .cu into _build/ in parallel and link libsplax_b200.so."""
    if not force and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(item):
        name, extra = item
        obj = BUILD_DIR / (name + ".o")
        cmd = [cc, *ARCH, *COMMON, *extra, "-c", str(CSRC / name), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {name}:\n{res.stderr}")
        if verbose or ptxas_info:
            print(res.stderr, end="")
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES.items()))
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(force=True, verbose=True, ptxas_info="-v" in sys.argv))
