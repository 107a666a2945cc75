"""Golden vectors for frnn_cuda.harness, from the reference's own benchmark script.

Run in a container that has the reference checkout (it is not needed to run the
tests):

    python tests/golden/harness/make_harness_golden.py /path/to/reference

It compiles only the definitions of gen_points, radius_for and calibrate_radius
from Tests/scripts/benchmark_vs_libfrnn.py (the module's top level, which runs
the GPU sweep, is not executed), evaluates them on small seeded cases and writes
tests/golden/harness/harness_golden.npz.
"""

import ast
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_functions(ref_root):
    path = os.path.join(ref_root, "Tests", "scripts", "benchmark_vs_libfrnn.py")
    tree = ast.parse(open(path).read(), path)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef)
            and n.name in ("gen_points", "radius_for", "calibrate_radius")]
    ns = {"np": np, "pi": math.pi, "gamma": math.gamma, "ceil": math.ceil, "K": 16,
          "print": lambda *a, **k: None}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FRNN_REF_ROOT")
    if not ref_root:
        sys.exit("usage: make_harness_golden.py REF_ROOT (or set FRNN_REF_ROOT): the reference checkout")
    ns = reference_functions(ref_root)
    out = {}
    cases = [("uniform", 3, 0.02, 2000, 3), ("lowrank", 3, 0.02, 3000, 12), ("lowrank", 3, 0.02, 2500, 16),
             ("lowrank", 5, 0.05, 1500, 8)]
    for t, (dist, intrinsic, noise, N, D) in enumerate(cases):
        ns.update(DIST=dist, INTRINSIC=intrinsic, LOWRANK_NOISE=noise)
        pts = ns["gen_points"](N, D, 1234)
        out[f"pts{t}"] = pts
        out[f"meta{t}"] = np.array([N, D, intrinsic, noise, dist == "uniform"], dtype=np.float64)
        if dist != "uniform":
            out[f"r{t}"] = np.array(ns["calibrate_radius"](pts, target=16))
    out["radius_for"] = np.array([[D, N, ns["radius_for"](D, N)] for D in (3, 12, 16, 128)
                                  for N in (200000, 1000000)], dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "harness_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "harness_golden.npz"))


if __name__ == "__main__":
    main()
