"""Result comparison helpers for the parity tests.

Two bars are used:

* ``assert_bit_exact`` -- engine vs the CPU oracle: both compute the same
  fp32 distances in the same order and rank by (d2, index), so index and
  distance arrays must be identical.

* ``compare_to_reference`` -- engine (or oracle) vs the reference engine,
  whose slot order is heap order and whose tie-break is its visit order.  The
  bar (from the project brief): neighbour index sets exact, except that ties
  at equal distance and points within 1e-6*r^2 of the radius boundary are
  excepted and counted; distances of shared neighbours within 1e-5 relative.
"""

from __future__ import annotations

import numpy as np

BOUNDARY_REL = 1e-6
DIST_RTOL = 1e-5


def assert_bit_exact(idx_a, dist_a, idx_b, dist_b, what=""):
    idx_a, idx_b = np.asarray(idx_a), np.asarray(idx_b)
    dist_a, dist_b = np.asarray(dist_a), np.asarray(dist_b)
    assert idx_a.shape == idx_b.shape, (idx_a.shape, idx_b.shape)
    bad = np.argwhere((idx_a != idx_b) | (dist_a.view(np.int32) != dist_b.view(np.int32)))
    if len(bad):
        k, q = bad[0]
        qs = np.unique(bad[:, 1])
        rows = "; ".join(f"q={int(x)} k={[int(y) for y in bad[bad[:, 1] == x, 0][:4]]} "
                         f"a={idx_a[:4, x].tolist()} b={idx_b[:4, x].tolist()}" for x in qs[:4])
        raise AssertionError(
            f"{what}: {len(bad)} mismatching slots in {len(qs)} queries; first at k={k} q={q}: "
            f"a=({idx_a[k, q]}, {dist_a[k, q]!r}) b=({idx_b[k, q]}, {dist_b[k, q]!r}); {rows}")


def sort_rows(idx: np.ndarray, dist: np.ndarray):
    """SoA (K, N) -> per-query rows sorted by (d2, idx); padding (-1) last."""
    idx = np.asarray(idx).T.copy()
    dist = np.asarray(dist).T.copy()
    key_d = np.where(idx < 0, np.inf, dist.astype(np.float64))
    key_i = np.where(idx < 0, np.iinfo(np.int64).max, idx.astype(np.int64))
    order = np.lexsort((key_i, key_d), axis=1)
    return np.take_along_axis(idx, order, 1), np.take_along_axis(dist, order, 1)


def compare_to_reference(idx_a, dist_a, idx_r, dist_r, pts_soa, r, valid=None, d2_f64=None):
    """Compare SoA results a (engine) with r (reference).  Returns a dict of
    counts; ``mismatch`` must be 0 for parity.  ``d2_f64(qi, pj)`` gives exact
    squared distances used to classify differences."""
    K, N = np.asarray(idx_a).shape
    a_i, a_d = sort_rows(idx_a, dist_a)
    b_i, b_d = sort_rows(idx_r, dist_r)
    r2 = float(np.float32(r) * np.float32(r))
    band = BOUNDARY_REL * r2
    stats = {"queries": 0, "identical": 0, "tie_excepted": 0, "boundary_excepted": 0,
             "dist_mismatch": 0, "mismatch": 0, "first_bad": None}
    rows = np.arange(N) if valid is None else np.nonzero(valid)[0]
    stats["queries"] = int(len(rows))
    # vectorised fast path: rows with identical index lists and close distances
    same = np.all(a_i[rows] == b_i[rows], axis=1)
    ad, bd = a_d[rows].astype(np.float64), b_d[rows].astype(np.float64)
    close = np.all(np.abs(ad - bd) <= DIST_RTOL * np.maximum(np.maximum(np.abs(ad), np.abs(bd)), 1e-30),
                   axis=1)
    stats["identical"] += int(np.sum(same & close))
    for q in rows[~(same & close)]:
        sa = set(int(x) for x in a_i[q] if x >= 0)
        sb = set(int(x) for x in b_i[q] if x >= 0)
        # distances of shared neighbours
        da = {int(i): float(d) for i, d in zip(a_i[q], a_d[q]) if i >= 0}
        db = {int(i): float(d) for i, d in zip(b_i[q], b_d[q]) if i >= 0}
        for j in sa & sb:
            x, y = da[j], db[j]
            if abs(x - y) > DIST_RTOL * max(abs(x), abs(y), 1e-30):
                stats["dist_mismatch"] += 1
                stats["first_bad"] = stats["first_bad"] or (int(q), j, x, y)
        if sa == sb:
            stats["identical"] += 1
            continue
        diff = sorted(sa ^ sb)
        # classify every differing index
        if d2_f64 is not None:
            exact = d2_f64(np.full(len(diff), q, np.int32), np.array(diff, np.int32))
        else:
            exact = np.array([da.get(j, db.get(j)) for j in diff], np.float64)
        near_boundary = np.abs(exact - r2) <= band
        if np.all(near_boundary):
            stats["boundary_excepted"] += 1
            continue
        # ties: a differing index must sit at the K-th (largest kept) distance
        kth_a = max(da.values()) if len(da) == K else None
        kth_b = max(db.values()) if len(db) == K else None
        ok = True
        for j, nb in zip(diff, near_boundary):
            if nb:
                continue
            dj = da.get(j, db.get(j))
            # equal distance up to the 1e-5 relative distance tolerance: the two
            # engines may round the same pair differently by an ulp
            tie = any(k is not None and abs(dj - k) <= DIST_RTOL * max(abs(k), 1e-30)
                      for k in (kth_a, kth_b))
            if not tie:
                ok = False
        if ok:
            stats["tie_excepted"] += 1
        else:
            stats["mismatch"] += 1
            stats["first_bad"] = stats["first_bad"] or (int(q), diff[:6])
    return stats
