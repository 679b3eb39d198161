"""Build libquack_b200.so in-tree with nvcc for sm_100a.

    python quack_b200/csrc/build.py            # incremental
    python quack_b200/csrc/build.py --force

Every translation unit is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; the GEMM instantiation file is
compiled once per (operand kind, output format) pair so the pairs build in parallel.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
OBJ_DIR = os.path.join(HERE, "build")
LIB_PATH = os.path.join(PKG, "libquack_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
]

HEADERS = ["qk_ptx.cuh", "qk_types.h", "qk_common.h", "gemm_blockscaled.cuh", "gemm_host.h",
           os.path.join("..", "..", "include", "quack_b200.h")]


def _units():
    units = [("capi.cu", "capi.o", []), ("quantize.cu", "quantize.o", []), ("gemm_api.cu", "gemm_api.o", []),
             ("peer.cu", "peer.o", []), ("tensormap.cu", "tensormap.o", [])]
    if os.path.exists(os.path.join(HERE, "noalloc.cu")):
        units.append(("noalloc.cu", "noalloc.o", []))
    for kind in (0, 1, 2):
        for qf in (0, 1, 2, 4):
            units.append(("gemm_inst.cu", f"gemm_k{kind}_q{qf}.o", [f"-DQK_KIND={kind}", f"-DQK_QF={qf}"]))
    return units


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _stale(src, obj):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(HERE, h) for h in HEADERS] + [os.path.abspath(__file__)]
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, defines=(), lib_path: str = LIB_PATH, obj_dir: str = OBJ_DIR) -> str:
    """Compile what is stale and link.  `defines` (e.g. ("QK_EPI_GROUPS=1",)) with a separate `lib_path` /
    `obj_dir` builds a variant library next to the default one (load it with QUACK_B200_LIB=path)."""
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = _nvcc()
    jobs = []
    objs = []
    extra = [f"-D{d}" for d in defines]
    for src, obj, defs in _units():
        s, o = os.path.join(HERE, src), os.path.join(obj_dir, obj)
        objs.append(o)
        if force or _stale(s, o):
            jobs.append([nvcc, *NVCC_FLAGS, *defs, *extra, "-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if jobs or not os.path.exists(lib_path) or force:
        run([nvcc, "-shared", "-o", lib_path, *objs, "-Xcompiler", "-fPIC"])
    return lib_path


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--define", action="append", default=[], help="extra -D for every unit (variant builds)")
    ap.add_argument("--out", default=LIB_PATH, help="library path (variant builds)")
    ap.add_argument("--objdir", default=OBJ_DIR)
    a = ap.parse_args()
    print(build(force=a.force, verbose=True, defines=tuple(a.define), lib_path=a.out, obj_dir=a.objdir))
