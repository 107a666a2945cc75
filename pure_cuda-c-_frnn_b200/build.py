"""Build the engine's shared library for sm_100a.

    python pure_cuda-c-_frnn_b200/build.py [--force] [--verbose]

Compiles every csrc/*.cu with nvcc (-gencode arch=compute_100a,code=sm_100a
-lineinfo -O3) and links frnn_cuda/libfrnn_b200.so in-tree, so the library
travels with the source tree.  Objects go to csrc/_build/.  Rebuilds only what
changed (source or any csrc/ header newer than the object).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(CSRC, "_build")
LIB = os.path.join(HERE, "frnn_cuda", "libfrnn_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", INCLUDE, "-I", CSRC] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "frnn_b200.h"))
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
          defines: list[str] | None = None, out: str | None = None) -> str:
    """Compile and link.  ``defines`` are extra -D macros (launch-policy
    knobs); with defines or ``out`` the objects go to a separate folder and the
    library to ``out``, leaving the default build untouched."""
    defines = defines or []
    lib = out or LIB
    tag = hashlib.sha1(repr((sorted(defines), os.path.abspath(lib))).encode()).hexdigest()[:10]
    obj_dir = OBJ if not (defines or out) else OBJ + "_" + tag
    os.makedirs(obj_dir, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    hdrs = _headers()
    cc = nvcc()
    jobs = []
    objs = []
    for f in srcs:
        src = os.path.join(CSRC, f)
        obj = os.path.join(obj_dir, f[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            cmd = [cc, "-c", src, "-o", obj] + NVCC_FLAGS + ["-D" + d for d in defines]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        p = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, p

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cmd, p in ex.map(run, jobs):
            if p.returncode != 0:
                failed.append((cmd, p))
            elif ptxas_verbose or verbose:
                sys.stderr.write(p.stderr)
    if failed:
        for cmd, p in failed:
            sys.stderr.write(" ".join(cmd) + "\n" + p.stdout + p.stderr + "\n")
        raise RuntimeError(f"nvcc failed for {len(failed)} file(s)")
    if force or jobs or _stale(lib, objs):
        cmd = [cc, "-shared", "-o", lib] + objs + ARCH + ["-lcudart", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError("link failed:\n" + p.stdout + p.stderr)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print register/spill usage")
    ap.add_argument("-D", dest="defines", action="append", default=[],
                    help="extra macro, e.g. -D FRNN_COOP_MIN_BLOCKS=6")
    ap.add_argument("--out", default=None, help="library path (default: in-tree frnn_cuda/)")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas, a.defines, a.out))
