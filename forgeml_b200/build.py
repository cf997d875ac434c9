"""Build the sm_100a shared library ``forgeml_b200/_lib/libforgeml_b200.so``.

The kernels are plain CUDA C++ behind an ``extern "C"`` ABI
(``include/forgeml_b200.h``); the Python packages load the library with
ctypes.  Built in-tree with nvcc (cross-compiles without a GPU):

    python -m forgeml_b200.build            # incremental
    python -m forgeml_b200.build --force    # rebuild everything
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
OBJ_DIR = OUT_DIR / "obj"
LIB_NAME = "libforgeml_b200.so"
SOURCES = ["common.cu", "gemm.cu", "layernorm.cu", "attention.cu", "sdpa_tc.cu", "nebula_ops.cu", "allreduce.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")
    return cand


def common_flags() -> list[str]:
    return [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-rdc=true",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        f"-I{PKG.parent / 'include'}",
    ]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list((PKG.parent / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: str, nvcc: str, force: bool, verbose: bool) -> Path:
    s = CSRC / src
    o = OBJ_DIR / (Path(src).stem + ".o")
    if not force and o.exists() and o.stat().st_mtime >= max(s.stat().st_mtime, _headers_mtime()):
        return o
    cmd = [nvcc, *common_flags(), "-c", str(s), "-o", str(o)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return o


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link the shared library."""
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, nvcc, force, verbose), SOURCES))
    lib = OUT_DIR / LIB_NAME
    if not force and lib.exists() and lib.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return lib
    cmd = [nvcc, *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", "-o", str(lib)]
    cmd += [str(o) for o in objs]
    cmd += ["-cudart", "static", "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
