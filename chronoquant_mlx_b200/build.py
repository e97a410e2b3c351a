"""Build libchronoquant_b200.so in-tree with nvcc for sm_100a.

    python -m chronoquant_mlx_b200.build [--force] [-j N] [--checks]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (in parallel), then
they link into ``chronoquant_mlx_b200/libchronoquant_b200.so``.  Objects are
rebuilt when their source or any ``csrc/*.cuh`` / ``include/*.h`` is newer.

``--checks`` builds the debug variant ``libchronoquant_b200_checks.so``
(objects under ``_build/checks/``) with ``-DCQ_CHECKS``: every page lookup
in the kernels is bounds-checked and a bad index is reported as device
error 7 (``cq_device_error``) instead of being followed.  The package loads
it instead of the release library when ``CQ_CHECKS=1`` is set at import.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libchronoquant_b200.so")
OUT_CHECKS = os.path.join(HERE, "libchronoquant_b200_checks.so")
BUILD = os.path.join(ROOT, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def build(force: bool = False, jobs: int = 8, verbose: bool = False, checks: bool = False) -> str:
    bdir = os.path.join(BUILD, "checks") if checks else BUILD
    out = OUT_CHECKS if checks else OUT
    os.makedirs(bdir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = _newest_header()
    cc = nvcc()
    flags = FLAGS + (["-DCQ_CHECKS"] if checks else [])

    def compile_one(src: str) -> str:
        obj = os.path.join(bdir, os.path.basename(src)[:-3] + ".o")
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr):
            return obj
        cmd = [cc, *ARCH, *flags, "-Xptxas", "-v", "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, srcs))
    newest_obj = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(out) or os.path.getmtime(out) < newest_obj:
        tmp = out + ".tmp"
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, out)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--checks", action="store_true", help="the bounds-checked debug variant")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v, checks=a.checks))


if __name__ == "__main__":
    main()
