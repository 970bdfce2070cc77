"""Oracle restatement of AgentRL's ``PagedKVAllocator`` (test infrastructure).

Follows agentrl/generation/paged_kv.py:11-175 statement by statement, in plain
Python with ``heapq`` exactly as the reference does, so that every block id,
counter and exception it produces is the reference's.  Reference quirks are
kept on purpose (see the method docstrings): a ``reserve`` that runs out of
blocks part-way leaks the ids it already popped, and an ``append_tokens`` that
runs out keeps the blocks it already appended.

The copy-on-write extension (``fork``, per-block refcounts, the tail copy on
the first append to a shared partial block) has no reference counterpart.
With ``fork`` never called every refcount stays 1 and every result is the
reference's.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass


@dataclass(frozen=True, slots=True)
class SequenceView:
    """paged_kv.py:11-22 ``PagedKVSequenceView``."""

    sequence_id: int
    token_count: int
    block_size_tokens: int
    physical_blocks: tuple[int, ...]

    @property
    def logical_block_count(self) -> int:
        return len(self.physical_blocks)


class OracleAllocator:
    """paged_kv.py:25-175, plus refcounts for copy-on-write forks."""

    def __init__(self, total_blocks: int, block_size_tokens: int) -> None:
        # paged_kv.py:34-48
        if total_blocks <= 0:
            raise ValueError("total_blocks must be > 0.")
        if block_size_tokens <= 0:
            raise ValueError("block_size_tokens must be > 0.")
        self.total_blocks = total_blocks
        self.block_size_tokens = block_size_tokens
        self._free = list(range(total_blocks))
        heapq.heapify(self._free)
        self._tables: dict[int, list[int]] = {}
        self._counts: dict[int, int] = {}
        self._touched: set[int] = set()
        self._reuse = 0
        self._high = 0
        # extension: refcount per block and the log of copy-on-write copies
        self._refcount = [0] * total_blocks
        self.cow_log: list[tuple[int, int, int]] = []  # (sequence_id, src, dst)

    # paged_kv.py:50-76
    @property
    def free_block_count(self) -> int:
        return len(self._free)

    @property
    def used_block_count(self) -> int:
        return self.total_blocks - self.free_block_count

    @property
    def block_reuse_count(self) -> int:
        return self._reuse

    @property
    def max_blocks_in_use(self) -> int:
        return self._high

    @property
    def resident_sequence_count(self) -> int:
        return len(self._tables)

    @property
    def allocator_occupancy(self) -> float:
        return self.used_block_count / self.total_blocks

    @property
    def allocator_pressure(self) -> float:
        return self.allocator_occupancy

    def reserve(self, sequence_id: int, token_count: int) -> SequenceView:
        """paged_kv.py:78-91.  Running out part-way leaks the popped ids."""
        if sequence_id in self._tables:
            raise ValueError(f"sequence_id {sequence_id} is already allocated.")
        if token_count < 0:
            raise ValueError("token_count must be >= 0.")
        blocks = [self._allocate() for _ in range(self._required(token_count))]
        for b in blocks:
            self._refcount[b] = 1
        self._tables[sequence_id] = blocks
        self._counts[sequence_id] = token_count
        self._update_high()
        return self.view(sequence_id)

    def append_tokens(self, sequence_id: int, token_count: int) -> SequenceView:
        """paged_kv.py:93-110, with a copy-on-write of a shared partial tail."""
        if token_count < 0:
            raise ValueError("token_count must be >= 0.")
        if sequence_id not in self._tables:
            raise KeyError(f"Unknown sequence_id {sequence_id}.")
        if token_count == 0:
            return self.view(sequence_id)
        table = self._tables[sequence_id]
        old_total = self._counts[sequence_id]
        if table and old_total % self.block_size_tokens != 0 and self._refcount[table[-1]] > 1:
            src = table[-1]
            dst = self._allocate()
            self._refcount[src] -= 1
            self._refcount[dst] = 1
            table[-1] = dst
            self.cow_log.append((sequence_id, src, dst))
        new_total = old_total + token_count
        for _ in range(self._required(new_total) - len(table)):
            b = self._allocate()
            self._refcount[b] = 1
            table.append(b)
        self._counts[sequence_id] = new_total
        self._update_high()
        return self.view(sequence_id)

    def release(self, sequence_id: int) -> None:
        """paged_kv.py:112-120; a block returns to the heap when its refcount hits 0."""
        blocks = self._tables.pop(sequence_id, None)
        self._counts.pop(sequence_id, None)
        if blocks is None:
            raise KeyError(f"Unknown sequence_id {sequence_id}.")
        for b in blocks:
            self._refcount[b] -= 1
            if self._refcount[b] == 0:
                heapq.heappush(self._free, b)

    def fork(self, parent_id: int, child_id: int) -> SequenceView:
        """Extension: the child shares every block of the parent (refcount + 1)."""
        if child_id in self._tables:
            raise ValueError(f"sequence_id {child_id} is already allocated.")
        if parent_id not in self._tables:
            raise KeyError(f"Unknown sequence_id {parent_id}.")
        table = list(self._tables[parent_id])
        for b in table:
            self._refcount[b] += 1
        self._tables[child_id] = table
        self._counts[child_id] = self._counts[parent_id]
        return self.view(child_id)

    def truncate(self, sequence_ids, token_counts) -> None:
        """Extension: shrink sequences, releasing blocks past the new end (rollback of drafts)."""
        for sid, n in zip(sequence_ids, token_counts):
            if n < 0:
                raise ValueError("token_count must be >= 0.")
            if sid not in self._tables:
                raise KeyError(f"Unknown sequence_id {sid}.")
            if n > self._counts[sid]:
                raise ValueError("truncate cannot grow a sequence")
            table = self._tables[sid]
            while len(table) > self._required(n):
                b = table.pop()
                self._refcount[b] -= 1
                if self._refcount[b] == 0:
                    heapq.heappush(self._free, b)
            self._counts[sid] = n

    def logical_to_physical(self, sequence_id: int, logical_block_index: int) -> int:
        """paged_kv.py:122-127."""
        if logical_block_index < 0:
            raise ValueError("logical_block_index must be >= 0.")
        return self._tables[sequence_id][logical_block_index]

    def view(self, sequence_id: int) -> SequenceView:
        """paged_kv.py:129-139."""
        if sequence_id not in self._tables:
            raise KeyError(f"Unknown sequence_id {sequence_id}.")
        return SequenceView(
            sequence_id=sequence_id,
            token_count=self._counts[sequence_id],
            block_size_tokens=self.block_size_tokens,
            physical_blocks=tuple(self._tables[sequence_id]),
        )

    def metrics(self) -> dict[str, float]:
        """paged_kv.py:141-152."""
        return {
            "paged_kv_free_block_count": float(self.free_block_count),
            "paged_kv_used_block_count": float(self.used_block_count),
            "paged_kv_allocator_occupancy": float(self.allocator_occupancy),
            "paged_kv_block_reuse_count": float(self.block_reuse_count),
            "paged_kv_allocator_pressure": float(self.allocator_pressure),
            "paged_kv_max_blocks_in_use": float(self.max_blocks_in_use),
            "paged_kv_resident_sequences": float(self.resident_sequence_count),
        }

    def has_sequence(self, sequence_id: int) -> bool:
        """paged_kv.py:154-157."""
        return sequence_id in self._tables

    def refcount(self, block_id: int) -> int:
        """Extension: owners of a block (0 = free)."""
        return self._refcount[block_id]

    def _allocate(self) -> int:
        """paged_kv.py:159-167: lowest free id; a re-touched id counts as reuse."""
        if not self._free:
            raise RuntimeError("PagedKVAllocator ran out of free blocks.")
        b = heapq.heappop(self._free)
        if b in self._touched:
            self._reuse += 1
        else:
            self._touched.add(b)
        return b

    def _required(self, token_count: int) -> int:
        """paged_kv.py:169-172."""
        if token_count == 0:
            return 0
        return (token_count + self.block_size_tokens - 1) // self.block_size_tokens

    def _update_high(self) -> None:
        """paged_kv.py:174-175."""
        self._high = max(self._high, self.used_block_count)
