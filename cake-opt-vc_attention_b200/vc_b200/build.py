"""Build the in-tree CUDA library ``libvc_b200.so`` for sm_100a with nvcc.

The library is a plain C-ABI shared object (see include/vc_b200.h); Python
loads it with ctypes.  Objects are compiled in parallel and relinked only when
a source or header is newer than the library.

    python -m vc_b200.build [--force] [--verbose]
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
ROOT = PKG.parent                       # cake-opt-vc_attention_b200/
REPO = ROOT.parent
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libvc_b200.so"
OBJ_DIR = ROOT / "_build"
SOURCES = ["capi.cu", "prep_qk.cu", "prep_hadamard.cu", "prep_v.cu", "cluster.cu", "attention.cu", "tensor_peak.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# Whole-program device code (no -rdc): ptxas honours setmaxnreg only then.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-v", "-diag-suppress=177"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    exe = shutil.which("nvcc") or str(Path(home) / "bin" / "nvcc")
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return exe


def _deps() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) +
                  list(INCLUDE.glob("*.h")))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = OBJ_DIR / (Path(src).stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(CSRC / src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr[-8000:]}")
    return str(obj), (r.stderr if verbose else "")


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", *objs, "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr[-8000:]}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
