"""The host plan of a prefill / verify launch (pkv_prefill_plan), on CPU.

Records are {table row, first query position, query index, kv_head << 16 |
positions, first KV tile, end KV tile (0 = all), partial slot, 0}; the kernel
trusts them, so the plan must cover every query of every sequence and KV
head exactly once, and a key-split item's ranges must tile its keys.
"""

from __future__ import annotations

import numpy as np
import pytest

from randomrepo_b200.device import plan_prefill


@pytest.mark.parametrize("hq,hkv", [(12, 2), (28, 4), (14, 2), (8, 8)])
def test_every_query_row_once(hq, hkv):
    rng = np.random.default_rng(hq)
    past = rng.integers(0, 3000, size=9)
    qlens = rng.integers(1, 600, size=9)
    plan = plan_prefill(np.arange(9), past, qlens, hq, hkv, num_sms=148, split_waves=0)
    assert plan.n_combine == 0 and plan.n_slots == 0
    items = plan.records
    seen = np.zeros((int(qlens.sum()), hkv), dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(qlens)])
    for row, pos0, qrow0, hw, lo, hi, slot, _ in items.tolist():
        h, nt = hw >> 16, hw & 0xFFFF
        assert (lo, hi, slot) == (0, 0, -1)
        assert 1 <= nt <= 2 * (128 // (hq // hkv))
        i = row
        assert starts[i] <= qrow0 and qrow0 + nt <= starts[i + 1]
        assert pos0 == past[i] + (qrow0 - starts[i])
        seen[qrow0:qrow0 + nt, h] += 1
    assert (seen == 1).all()
    works = [-(-(r[1] + (r[3] & 0xFFFF)) // 128) for r in items.tolist()]
    assert works == sorted(works, reverse=True)  # longest key range first


def test_key_split_plan_covers_every_key_once():
    """Host plan: each split item's key ranges tile [0, n_tiles) exactly and its slots are distinct."""
    from randomrepo_b200.device import plan_prefill

    rng = np.random.default_rng(1)
    pre = rng.integers(128, 1281, size=64)
    plan = plan_prefill(np.arange(64), pre - 1, np.full(64, 5), 12, 2, num_sms=148, split_waves=2)
    items = plan.records[:plan.n_items]
    combine = plan.records[plan.n_items:]
    assert plan.n_combine == len(combine) > 0
    slots = items[:, 6][items[:, 6] >= 0]
    assert len(set(slots.tolist())) == len(slots) == plan.n_slots
    for slot0, ns, qrow0, hw, *_ in combine.tolist():
        parts = items[(items[:, 6] >= slot0) & (items[:, 6] < slot0 + ns)]
        assert len(parts) == ns and (parts[:, 2] == qrow0).all() and (parts[:, 3] == hw).all()
        kv_len = int(parts[0, 1]) + (hw & 0xFFFF)
        ranges = sorted((int(lo), int(hi)) for lo, hi in parts[:, 4:6])
        assert ranges[0][0] == 0 and ranges[-1][1] == -(-kv_len // 128)
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
