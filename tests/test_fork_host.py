"""Copy-on-write fork semantics of the product allocator against the oracle (host only).

The reference has no fork (each GRPO group member is prefilled on its own,
agentrl/generation/continuous.py:88-99), so parity here is against the oracle's
restatement of the extension: shared blocks carry refcounts, a block returns
to the free set when its last owner releases it, and the first append into a
shared partial tail block moves the appender to a private copy.
"""

from __future__ import annotations

import random

import pytest

from oracle.allocator import OracleAllocator


def _product(total, bs):
    from randomrepo_b200 import PagedKVAllocator

    return PagedKVAllocator(total, bs)


def test_group_fork_shares_prompt_blocks():
    for alloc in (OracleAllocator(64, 16), _product(64, 16)):
        alloc.reserve(0, 40)  # prompt: 3 blocks, last one partial (8 tokens)
        for child in range(1, 8):
            view = alloc.fork(0, child)
            assert view.physical_blocks == (0, 1, 2) and view.token_count == 40
        assert alloc.used_block_count == 3
        assert [alloc.refcount(b) for b in (0, 1, 2)] == [8, 8, 8]
        # members 0..6 get private tails on their first append; member 7 keeps block 2
        tails = [alloc.append_tokens(m, 1).physical_blocks[-1] for m in range(8)]
        assert tails == [3, 4, 5, 6, 7, 8, 9, 2]
        assert [alloc.refcount(b) for b in range(10)] == [8, 8, 1, 1, 1, 1, 1, 1, 1, 1]
        for m in range(8):
            alloc.release(m)
        assert alloc.free_block_count == 64 and alloc.used_block_count == 0


def test_full_tail_needs_no_copy():
    for alloc in (OracleAllocator(16, 16), _product(16, 16)):
        alloc.reserve(0, 32)
        alloc.fork(0, 1)
        assert alloc.append_tokens(1, 1).physical_blocks == (0, 1, 2)
        assert alloc.append_tokens(0, 1).physical_blocks == (0, 1, 3)
        assert alloc.refcount(0) == 2 and alloc.refcount(2) == 1


def test_fork_errors():
    for alloc in (OracleAllocator(8, 2), _product(8, 2)):
        alloc.reserve(0, 3)
        with pytest.raises(KeyError):
            alloc.fork(5, 6)
        with pytest.raises(ValueError, match="sequence_id 0 is already allocated."):
            alloc.fork(0, 0)


@pytest.mark.parametrize("seed", range(8))
def test_random_fork_traces_match_oracle(seed):
    rng = random.Random(seed)
    total, bs = rng.choice([(32, 2), (64, 16), (48, 3)])
    ora, prod = OracleAllocator(total, bs), _product(total, bs)
    live: list[int] = []
    next_id = 0
    for _ in range(300):
        r = rng.random()
        if r < 0.2 or not live:
            op = ("reserve", next_id, rng.randint(0, 3 * bs))
            next_id += 1
        elif r < 0.35:
            op = ("fork", rng.choice(live), next_id)
            next_id += 1
        elif r < 0.72:
            op = ("append_tokens", rng.choice(live), rng.choice([1, 1, 1, bs, rng.randint(0, 2 * bs)]))
        elif r < 0.8:
            sid = rng.choice(live)
            op = ("truncate", [sid], [max(0, ora.view(sid).token_count - rng.randint(0, 2 * bs))])
        else:
            op = ("release", rng.choice(live))
        results = []
        for alloc in (ora, prod):
            try:
                res = getattr(alloc, op[0])(*op[1:])
                if op[0] == "truncate":
                    res = alloc.view(op[1][0])
                results.append(("ok", None if res is None else (res.token_count, tuple(res.physical_blocks))))
            except Exception as exc:  # noqa: BLE001
                results.append((type(exc).__name__, str(exc)))
        assert results[0] == results[1], op
        if results[0][0] == "ok":
            if op[0] in ("reserve", "fork"):
                live.append(op[-1] if op[0] == "fork" else op[1])
            elif op[0] == "release":
                live.remove(op[1])
        assert ora.metrics() == prod.metrics()
    for b in range(total):
        assert ora.refcount(b) == prod.refcount(b)
    assert prod.shared_block_count == sum(1 for b in range(total) if ora.refcount(b) > 1)
