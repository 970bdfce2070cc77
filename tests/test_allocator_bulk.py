"""Bulk allocator queries the store's hot paths use, against per-sequence views (host only, no GPU).

``pkv_allocator_token_counts``, ``pkv_allocator_chunk_slots`` and
``pkv_allocator_truncate_fill`` replace loops of ``PagedKVAllocator.view``
calls in the store (the prefill / verify layout and the speculative
truncation); each must give exactly what the per-sequence computation gives.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from randomrepo_b200 import PagedKVAllocator
from randomrepo_b200._lib import lib, raise_for_status

BS = 16


def _allocators(seed: int):
    """Two allocators driven through the same random reserve / append / fork / release trace."""
    rng = np.random.default_rng(seed)
    pair = [PagedKVAllocator(2048, BS), PagedKVAllocator(2048, BS)]
    live = []
    for sid in range(40):
        op = rng.integers(0, 10)
        if op < 6 or not live:
            n = int(rng.integers(0, 200))
            for a in pair:
                a.reserve(sid, n)
            live.append(sid)
        elif op < 8:
            parent = live[int(rng.integers(0, len(live)))]
            for a in pair:
                a.fork(parent, sid)
            live.append(sid)
        else:
            victim = live.pop(int(rng.integers(0, len(live))))
            for a in pair:
                a.release(victim)
        if live and rng.integers(0, 2):
            s = live[int(rng.integers(0, len(live)))]
            k = int(rng.integers(1, 40))
            for a in pair:
                a.append_tokens(s, k)
    return pair, live, rng


@pytest.mark.parametrize("seed", range(4))
def test_token_counts_and_chunk_slots(seed):
    (a, _), live, rng = _allocators(seed)
    ids = np.array(live, dtype=np.int64)
    assert a.token_counts(ids).tolist() == [a.view(s).token_count for s in live]
    q_lens = np.array([int(rng.integers(0, a.view(s).token_count + 1)) for s in live], dtype=np.int64)
    fill = np.full(a.total_blocks, -1, dtype=np.int32)
    fill[rng.integers(0, a.total_blocks, 50)] = rng.integers(0, BS, 50)
    want_fill = fill.copy()
    rows, past = np.empty(ids.size, np.int32), np.empty(ids.size, np.int32)
    slots = np.empty(int(q_lens.sum()), np.int64)
    raise_for_status(lib.pkv_allocator_chunk_slots(a._handle, ids.ctypes.data, q_lens.ctypes.data, ids.size,
                                                   rows.ctypes.data, past.ctypes.data, slots.ctypes.data, slots.size,
                                                   fill.ctypes.data, fill.size))
    want_slots = []
    for i, s in enumerate(live):
        v = a.view(s)
        assert rows[i] == a.row(s) and past[i] == v.token_count - q_lens[i]
        pos = np.arange(past[i], v.token_count)
        blocks = np.asarray(v.physical_blocks, dtype=np.int64)[pos // BS] if pos.size else np.empty(0, np.int64)
        want_slots.append(blocks * BS + pos % BS)
        np.maximum.at(want_fill, blocks, (pos % BS + 1).astype(np.int32))
    assert np.array_equal(slots, np.concatenate(want_slots))
    assert np.array_equal(fill, want_fill)
    with pytest.raises(ValueError, match="fewer than its chunk"):
        bad = np.array([a.view(live[0]).token_count + 1], dtype=np.int64)
        raise_for_status(lib.pkv_allocator_chunk_slots(a._handle, ids.ctypes.data, bad.ctypes.data, 1,
                                                       rows.ctypes.data, past.ctypes.data, slots.ctypes.data,
                                                       slots.size, None, 0))
    with pytest.raises(KeyError):
        a.token_counts([10**9])


@pytest.mark.parametrize("seed", range(4))
def test_truncate_fill_equals_view_based_truncation(seed):
    (a, b), live, rng = _allocators(seed)
    ids = np.array(live, dtype=np.int64)
    counts = np.array([int(rng.integers(0, a.view(s).token_count + 1)) for s in live], dtype=np.int64)
    fill_a = np.full(a.total_blocks, -1, dtype=np.int32)
    for s in live:  # every stored token recorded
        v = a.view(s)
        for j, blk in enumerate(v.physical_blocks):
            fill_a[blk] = max(fill_a[blk], min(BS, v.token_count - j * BS))
    fill_b = fill_a.copy()
    # The store's former per-sequence algorithm, on allocator a.
    tails = []
    for s, n in zip(live, counts.tolist()):
        v = a.view(s)
        keep = -(-n // BS)
        tails.append((v.physical_blocks[:keep], v.physical_blocks[keep:], n))
    a.truncate(ids, counts)
    for kept, dropped, n in tails:
        for blk in dropped:
            if a.refcount(blk) == 0:
                fill_a[blk] = -1
        if kept and n % BS and fill_a[kept[-1]] > n % BS:
            fill_a[kept[-1]] = n % BS
    # The native pass, on allocator b.
    raise_for_status(lib.pkv_allocator_truncate_fill(b._handle, ids.ctypes.data, counts.ctypes.data, ids.size,
                                                     fill_b.ctypes.data, fill_b.size))
    assert np.array_equal(fill_a, fill_b)
    for s in live:
        assert a.view(s) == b.view(s)
    assert a.metrics() == b.metrics()
