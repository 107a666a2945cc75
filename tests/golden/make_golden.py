"""Record the reference engine's outputs on tests/golden/cases.py (run on a B200).

    python tests/golden/make_golden.py OUT_DIR

Runs FRNNEngine.search_gpu of the reference (oracle/_ref/libfrnn_ref.so,
compiled from the reference's own sources by oracle/Makefile) on each case and
writes OUT_DIR/<case>.npz with the SoA points, K, radius, the path the
reference dispatcher takes and its SoA results.  The committed fixtures in
tests/golden/ were produced by this script; test_oracle_cpu.py checks the
oracle against them on any machine.
"""

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "pure_cuda-c-_frnn_b200"), os.path.join(ROOT, "oracle"), HERE):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import oracle  # noqa: E402
from cases import cases  # noqa: E402
from frnn_cuda import datagen  # noqa: E402


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    for name, pts, K, r in cases():
        soa = datagen.soa(pts)
        D, N = soa.shape
        _, _, valid, path = oracle.ref_search(soa, K, r)
        assert valid.all(), f"{name}: a point would be dropped by the reference grid"
        eng = oracle.RefEngine(N)
        t = torch.from_numpy(soa).cuda()
        eng.search_gpu(t.data_ptr(), N, D, K, r)
        idx, dist = eng.get_results(N, K)
        eng.close()
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), points_soa=soa, K=K,
                            radius=np.float64(r), ref_path=path, ref_idx=idx, ref_dist=dist)
        print(name, path, N, D, K, r, flush=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py OUT_DIR (the .npz files are then reviewed and copied here)")
    main(sys.argv[1])
