"""The balanced split schedule of the tensor-core decode path, restated in
Python from its definition (csrc/mla_common.cuh: the cost line, each cluster's
quota, item ids b + cluster) and checked for the properties the kernels rely
on: every tile of every sequence is decoded exactly once, a sequence's item ids
are consecutive and below batch + clusters, no cluster exceeds its quota, and
the combine's id range for a sequence is exactly the ids its items used.
The fixed cost of an item is 2 tiles whatever the head count (item_cost_for:
the Q load is one 128-row box either way); schedules are checked at 16 and 128
heads."""
import numpy as np
import pytest

TILE = 96


def item_cost_for(num_heads):
    return 2


def cdiv(a, b):
    return -(-a // b)


def schedule(lens, clusters, ITEM_COST=2):
    tiles = [cdiv(n, TILE) for n in lens]
    cost = [t + ITEM_COST if t > 0 else 0 for t in tiles]
    off = np.concatenate([[0], np.cumsum(cost)]).astype(int)
    total = int(off[-1])
    q = max(1, cdiv(total, clusters))
    items = []  # (cluster, id, b, first_tile, last_tile_exclusive)
    for c in range(clusters):
        x0, x1 = min(c * q, total), min(c * q + q, total)
        for b, n in enumerate(lens):
            base = off[b] + ITEM_COST
            lo, hi = max(x0 - base, 0), min(x1 - base, tiles[b])
            if hi > lo:
                items.append((c, b + c, b, lo, hi))
    ranges = {}
    for b, t in enumerate(tiles):
        if t:
            base = off[b] + ITEM_COST
            ranges[b] = (b + base // q, b + (base + t - 1) // q + 1)
    return items, ranges, q, off


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("clusters", [1, 7, 74])
@pytest.mark.parametrize("num_heads", [16, 128])
def test_balanced_schedule_properties(seed, clusters, num_heads):
    ITEM_COST = item_cost_for(num_heads)
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in rng.integers(0, 9000, size=int(rng.integers(1, 300)))]
    items, ranges, q, off = schedule(lens, clusters, ITEM_COST)
    covered = {b: np.zeros(cdiv(n, TILE), dtype=int) for b, n in enumerate(lens)}
    per_cluster = {}
    for c, i, b, lo, hi in items:
        covered[b][lo:hi] += 1
        per_cluster[c] = per_cluster.get(c, 0) + (hi - lo) + ITEM_COST
        assert 0 <= i < len(lens) + clusters
    for b, cov in covered.items():
        assert np.all(cov == 1), f"sequence {b} tiles covered {cov}"
    ids = {}
    for c, i, b, lo, hi in items:
        ids.setdefault(b, []).append(i)
    for b, l in ids.items():
        l = sorted(l)
        assert l == list(range(l[0], l[-1] + 1)), "ids of one sequence are consecutive"
        assert ranges[b] == (l[0], l[-1] + 1), "combine range = the ids used"
    assert len({i for _, i, _, _, _ in items}) == len(items), "ids are unique"
    for c, load in per_cluster.items():
        assert load <= q + ITEM_COST, "a cluster's work is its quota plus at most one item's fixed cost"


def test_item_cost_is_two_tiles():
    assert item_cost_for(128) == 2 and item_cost_for(64) == 2 and item_cost_for(16) == 2


def test_balanced_schedule_single_sequence_matches_even_split():
    items, ranges, q, _ = schedule([131072], 74, item_cost_for(128))
    assert len(items) == 72 and max(hi - lo for *_, lo, hi in items) == q
