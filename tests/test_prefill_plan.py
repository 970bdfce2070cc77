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


def _verify_lists(plan):
    """Each CTA's items: its first record c, then the contiguous followers its last field names."""
    items = plan.records[:plan.n_items]
    lists = []
    for c in range(plan.n_ctas):
        f, m = int(items[c, 7]) >> 8, int(items[c, 7]) & 0xFF
        assert m <= 127 and (m == 0 or plan.n_ctas <= f and f + m <= plan.n_items)
        lists.append([c] + list(range(f, f + m)))
    return lists


@pytest.mark.parametrize("hq,hkv", [(12, 2), (28, 4), (8, 8), (32, 1)])
@pytest.mark.parametrize("num_sms", [0, 148, 7])
def test_verify_plan_covers_every_query_and_key_once(hq, hkv, num_sms):
    """pkv_verify_plan: items of at most 32 / G positions reached exactly once from the CTAs' lists;
    every (query, KV head) in exactly one item or one combine entry, whose ranges tile the item's
    keys with at least two KV tiles each."""
    from randomrepo_b200.device import plan_verify

    rng = np.random.default_rng(hq + num_sms)
    past = np.concatenate([rng.integers(0, 3000, size=20), [0, 127, 128, 8191]])
    qlens = np.concatenate([rng.integers(1, 9, size=20), [1, 5, 3, 2]])
    n = past.size
    ppv = 32 // (hq // hkv)
    plan = plan_verify(np.arange(n), past, qlens, hq, hkv, num_sms=num_sms)
    assert plan.kind == "verify"
    items = plan.records[:plan.n_items]
    combine = plan.records[plan.n_items:]
    if num_sms == 0:
        assert plan.n_combine == 0 and plan.n_slots == 0 and plan.n_ctas == plan.n_items
        assert (items[:, 7] == 0).all()
    else:
        assert plan.n_ctas == min(num_sms, plan.n_items)
    reached = sorted(k for chain in _verify_lists(plan) for k in chain)
    assert reached == list(range(plan.n_items))
    starts = np.concatenate([[0], np.cumsum(qlens)])
    seen = np.zeros((int(qlens.sum()), hkv), dtype=np.int32)
    for row, pos0, qrow0, hw, rng_, entry, slot, _ in items.tolist():
        h, nt = hw >> 16, hw & 0xFFFF
        lo, hi = rng_ & 0xFFFF, rng_ >> 16
        assert 1 <= nt <= ppv
        assert starts[row] <= qrow0 and qrow0 + nt <= starts[row + 1]
        assert pos0 == past[row] + (qrow0 - starts[row])
        if slot < 0:
            assert (lo, hi, entry) == (0, 0, -1)
            seen[qrow0:qrow0 + nt, h] += 1
        else:
            assert hi - lo >= 2
            c0, cn = combine[entry][:2]
            assert c0 <= slot < c0 + cn  # the item names the combine entry of its slot
    for slot0, ns, qrow0, hw, *_ in combine.tolist():
        parts = items[(items[:, 6] >= slot0) & (items[:, 6] < slot0 + ns)]
        assert len(parts) == ns >= 2 and (parts[:, 2] == qrow0).all() and (parts[:, 3] == hw).all()
        kv_len = int(parts[0, 1]) + (hw & 0xFFFF)
        ranges = sorted((int(r) & 0xFFFF, int(r) >> 16) for r in parts[:, 4])
        assert ranges[0][0] == 0 and ranges[-1][1] == -(-kv_len // 128)
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        seen[qrow0:qrow0 + (hw & 0xFFFF), hw >> 16] += 1
    assert (seen == 1).all()
    slots = items[:, 6][items[:, 6] >= 0]
    assert len(set(slots.tolist())) == len(slots) == plan.n_slots


def _work(rec):
    _, pos0, _, hw, rng_, _, slot, _ = rec
    return ((rng_ >> 16) - (rng_ & 0xFFFF)) if slot >= 0 else -(-(pos0 + (hw & 0xFFFF)) // 128)


def _costs(plan):
    items = plan.records[:plan.n_items].tolist()
    return items, [sum(_work(items[k]) + 2 for k in chain) for chain in _verify_lists(plan)]


def test_verify_plan_keeps_short_items_whole():
    """64 sequences, prefix U[128, 1280], k = 4 at 12/2 heads on 148 SMs: 128 items already balance
    better than cut ranges would with their combine launch, so each item gets a CTA of its own."""
    from randomrepo_b200.device import plan_verify

    rng = np.random.default_rng(0)
    pre = rng.integers(128, 1281, size=64)
    plan = plan_verify(np.arange(64), pre - 1, np.full(64, 5), 12, 2, num_sms=148)
    assert plan.n_combine == 0 and plan.n_slots == 0 and plan.n_items == plan.n_ctas == 128


@pytest.mark.parametrize("lo,hi,n", [(2048, 8192, 64), (4096, 16384, 32), (128, 1280, 16)])
def test_verify_plan_cuts_long_or_few_items(lo, hi, n):
    """Long prefixes (or few sequences): key ranges are cut, one CTA per SM (or per item), and no
    CTA's cost (its KV tiles plus 2 per item) is more than one item above the average."""
    from randomrepo_b200.device import plan_verify

    pre = np.random.default_rng(3).integers(lo, hi + 1, size=n)
    plan = plan_verify(np.arange(n), pre - 1, np.full(n, 5), 12, 2, num_sms=148)
    assert plan.n_combine > 0 and plan.n_ctas == min(148, plan.n_items)
    items, loads = _costs(plan)
    total = sum(_work(r) + 2 for r in items)
    assert total == sum(loads)
    assert max(loads) <= -(-total // plan.n_ctas) + max(_work(r) + 2 for r in items)
    for chain in _verify_lists(plan):  # each CTA's list runs longest item first
        works = [_work(items[k]) for k in chain]
        assert works == sorted(works, reverse=True)


def test_verify_plan_spills_past_128_items_per_cta():
    """More items than 128 per SM: more CTAs, none holding more than 128 items."""
    from randomrepo_b200.device import plan_verify

    n = 700
    plan = plan_verify(np.arange(n), np.full(n, 50), np.full(n, 5), 12, 2, num_sms=4)
    assert plan.n_items == 2 * n and plan.n_ctas == -(-2 * n // 128)
    lists = _verify_lists(plan)
    assert sorted(k for chain in lists for k in chain) == list(range(plan.n_items))
    assert max(len(chain) for chain in lists) <= 128


def test_verify_plan_rejects_wide_groups():
    from randomrepo_b200._lib import PKVError
    from randomrepo_b200.device import plan_verify

    with pytest.raises(PKVError):
        plan_verify(np.arange(1), np.array([10]), np.array([1]), 66, 2)
