"""The host plan of a decode step (pkv_decode_plan) covers every page exactly once (CPU only).

A work item is {sequence, split << 8 | head_group, splits of the sequence,
workspace slot of split 0}; the kernel trusts these fields, so the plan must
name only sequences of the batch, head groups of the pool, splits inside each
sequence's pages, and give every (sequence, head group, split) its own slot.
"""

from __future__ import annotations

import numpy as np
import pytest


@pytest.mark.parametrize("hkv", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("seed", range(4))
def test_plan_covers_every_page_once(hkv, seed):
    from randomrepo_b200._lib import lib
    from randomrepo_b200.device import plan_decode

    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 300))
    lens = rng.integers(1, 5000, size=n).astype(np.int32)
    if seed == 0:
        lens[:3] = [1, 16, 17]
    pps, rows, n_items, n_combine = plan_decode(lens, hkv, int(rng.choice([1, 7, 148])), int(rng.choice([64, 128])))
    items, entries = rows[:n_items], rows[n_items:]
    assert entries.shape == (n_combine, 4)
    hpc = lib.pkv_decode_heads_per_item(hkv)
    groups = hkv // hpc
    pages = (lens.astype(np.int64) + 15) // 16
    assert 4 <= pps <= 32 and np.all(-(-pages // pps) <= 64)
    seen = {}
    slots = set()
    for b, sh, ns, slot0 in items.tolist():
        split, hg = sh >> 8, sh & 0xFF
        assert 0 <= b < n and 0 <= hg < groups
        assert ns == -(-pages[b] // pps) and 0 <= split < ns
        assert (b, hg, split) not in seen
        seen[(b, hg, split)] = min(pps, pages[b] - split * pps)
        assert slot0 + split not in slots
        slots.add(slot0 + split)
    assert slots == set(range(len(items)))
    for b in range(n):
        for hg in range(groups):
            assert sum(v for (bb, gg, _), v in seen.items() if bb == b and gg == hg) == pages[b]
    # items by decreasing page count (the grid's tail holds the smallest); the full-size items follow
    # their sequences' decreasing length
    sizes = [min(pps, int(pages[b]) - (y >> 8) * pps) for b, y, _, _ in items.tolist()]
    assert all(a >= c for a, c in zip(sizes, sizes[1:]))
    full = [b for (b, _, _, _), sz in zip(items.tolist(), sizes) if sz == pps]
    firsts = [full[i] for i in range(len(full)) if i == 0 or full[i] != full[i - 1]]
    assert len(set(firsts)) == len(firsts)
    assert [int(pages[b]) for b in firsts] == sorted((int(pages[b]) for b in firsts), reverse=True)
    # one combine entry per (sequence, head group) cut into several items, naming its slots
    want = {(b, hg) for (b, hg, s) in seen if -(-pages[b] // pps) > 1}
    got = set()
    for b, hg, ns, slot0 in entries.tolist():
        assert ns == -(-pages[b] // pps) > 1
        assert {slot0 + s for s in range(ns)} <= slots
        for s in range(ns):
            assert (b, hg, s) in seen
        got.add((b, hg))
    assert got == want and len(got) == n_combine


def test_plan_rejects_empty_sequences():
    from randomrepo_b200.device import plan_decode

    with pytest.raises(Exception, match="at least one token"):
        plan_decode(np.array([3, 0], dtype=np.int32), 2, 148)
