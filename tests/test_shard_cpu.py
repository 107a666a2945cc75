"""The partition a sharded search applies (frnn_shard_partition), on the host.

The root cuts the cell-sorted queries at scan-tile starts so that every rank
gets about the same estimated work (the sum over its cells of
count * (count + 2)); these cases pin the cut rule without a GPU."""

import numpy as np
import pytest

import frnn_cuda


def cuts(work, N, nparts, starts=None):
    work = np.asarray(work, np.uint64)
    if starts is None:
        starts = np.linspace(0, N, len(work), endpoint=False).astype(np.int32)
    return frnn_cuda.shard_partition(work, starts, N, nparts)


def test_equal_work_equal_slices():
    b = cuts([10] * 8, 800, 4, starts=np.arange(0, 800, 100))
    assert b.tolist() == [0, 200, 400, 600, 800]


def test_bounds_cover_every_query_once():
    rng = np.random.default_rng(3)
    for nparts in (1, 2, 3, 5, 8, 64):
        tiles = int(rng.integers(1, 500))
        N = int(rng.integers(tiles, 10 * tiles + 1))
        starts = np.sort(rng.choice(N, tiles, replace=False)).astype(np.int32)
        starts[0] = 0
        work = rng.integers(0, 1000, tiles)
        b = cuts(work, N, nparts, starts)
        assert b[0] == 0 and b[-1] == N and len(b) == nparts + 1
        assert np.all(np.diff(b) >= 0)
        assert set(b[1:-1]).issubset(set(starts.tolist()) | {N})


def test_skewed_work_follows_the_work_not_the_count():
    # one dense region (a cluster) in the middle: its tiles carry most work
    work = [1] * 40 + [400] * 10 + [1] * 50
    b = cuts(work, 100_000, 4, starts=np.arange(0, 100_000, 1000))
    # all three cuts fall inside the dense tiles [40_000, 50_000)
    assert all(40_000 <= x <= 50_000 for x in b[1:-1]), b
    share = []
    cum = np.concatenate([[0], np.cumsum(work)])
    for r in range(4):
        share.append(cum[b[r + 1] // 1000] - cum[b[r] // 1000])
    assert max(share) <= 1.2 * (cum[-1] / 4) + 400, share


def test_more_ranks_than_tiles_leaves_empty_slices():
    b = cuts([5, 5], 10, 6, starts=[0, 5])
    assert b[0] == 0 and b[-1] == 10 and np.all(np.diff(b) >= 0)
    assert (np.diff(b) == 0).sum() >= 4


def test_rejects_bad_arguments():
    with pytest.raises(ValueError):
        frnn_cuda.shard_partition([1, 2], [0], 10, 2)
    with pytest.raises(ValueError):
        frnn_cuda.shard_partition([1], [0], 10, 0)


# The sharded tensor-core search that shares the symmetric filter: query
# block b (128 queries) filters the T - b tiles at or above it plus about
# 0.35 tile of re-rank; the ranks get equal shares, cut between pairs of
# blocks (frnn_shard_tc_partition).
def tc_block_work(N):
    T = (N + 127) // 128
    return (T - np.arange(T)) + 0.35


@pytest.mark.parametrize("N,nparts", [(1_000_000, 2), (1_000_000, 4), (1_000_000, 8), (300_001, 3),
                                      (65_536, 8), (9_001, 2), (1_000, 4), (0, 3), (5, 1)])
def test_tc_partition_covers_and_balances(N, nparts):
    b = frnn_cuda.shard_tc_partition(N, nparts)
    assert b[0] == 0 and b[-1] == N and (np.diff(b) >= 0).all(), b
    assert all(x % 256 == 0 for x in b[1:-1] if x < N), b
    w = tc_block_work(N)
    if N == 0 or nparts == 1:
        return
    blocks = [(lo // 128, (hi + 127) // 128) for lo, hi in zip(b[:-1], b[1:])]
    share = np.array([w[a:z].sum() for a, z in blocks]) / w.sum()
    # each cut is within one pair of blocks of its quantile
    pair = 2 * w[0] / w.sum()
    assert np.abs(np.cumsum(share)[:-1] - np.arange(1, nparts) / nparts).max() <= pair + 1e-12, share


def test_tc_partition_rejects_bad_arguments():
    for N, nparts in [(-1, 2), (100, 0), (100, 65)]:
        with pytest.raises((ValueError, frnn_cuda.FRNNError)):
            frnn_cuda.shard_tc_partition(N, nparts)
