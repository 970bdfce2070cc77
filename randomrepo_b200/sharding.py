"""Multi-GPU partitioning of the paged-KV path: GRPO groups per rank, one gather per step.

AgentRL normalises advantages inside a group (agentrl/core/rollout.py:474-491)
and a group's members share their prompt pages, so a group never needs
another GPU's KV: each rank owns whole groups, keeps its own KV pool and
allocator, and runs its own decode steps.  The only data that crosses GPUs is
what the trainer needs from every rank: per step, the sampled token id and its
log-probability for each of the rank's sequences.

* ``assign_groups`` maps groups to ranks, either round robin (group g on rank
  g mod world) or balanced by the KV tokens a group will hold (prompt length x
  group size, largest first onto the least loaded rank), which evens out the
  decode work when prompt lengths vary widely.
* ``StepGather`` gathers the (sequence id, token id, log-probability) rows of
  every rank to every rank with one ``all_gather_into_tensor`` per call (NCCL
  over NVLink on GPUs, gloo on CPU), on fixed-size buffers so every rank makes
  the same collective call whatever its own row count.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np
import torch


def assign_groups(prompt_lens, group_size: int, world: int, policy: str = "balanced") -> list[int]:
    """Rank of each group.

    ``prompt_lens[g]`` is group g's prompt length in tokens; every member of a
    group holds that prompt (shared pages after a fork) plus its own decode.
    ``policy`` is ``"modulo"`` (g mod world) or ``"balanced"`` (greedy
    longest-first by prompt_len x group_size onto the least loaded rank; ties
    go to the lower rank, so the result is deterministic).
    """
    if world <= 0:
        raise ValueError("world must be positive")
    if group_size <= 0:
        raise ValueError("group_size must be positive")
    lens = [int(n) for n in prompt_lens]
    if any(n < 0 for n in lens):
        raise ValueError("prompt lengths must be non-negative")
    if policy == "modulo":
        return [g % world for g in range(len(lens))]
    if policy != "balanced":
        raise ValueError(f"unknown policy {policy!r}")
    order = sorted(range(len(lens)), key=lambda g: (-lens[g], g))
    heap = [(0, r) for r in range(world)]
    out = [0] * len(lens)
    for g in order:
        load, r = heapq.heappop(heap)
        out[g] = r
        heapq.heappush(heap, (load + lens[g] * group_size, r))
    return out


def groups_of_rank(assignment: list[int], rank: int) -> list[int]:
    """The groups ``assign_groups`` gave to ``rank``, in increasing order."""
    return [g for g, r in enumerate(assignment) if r == rank]


@dataclass
class GatheredStep:
    """Rows of every rank for one step, rank 0's rows first."""

    sequence_ids: torch.Tensor  # int64 [n]
    tokens: torch.Tensor        # int64 [n]
    logprobs: torch.Tensor      # float32 [n]
    counts: list[int]           # rows per rank


class StepGather:
    """One collective per step: every rank's (sequence id, token, log-probability) rows to all ranks.

    Each rank packs its rows into an int64 buffer of ``1 + 3 * max_rows``
    entries (row count, then the rows; the float32 log-probability travels as
    its bit pattern), and one ``all_gather_into_tensor`` exchanges the
    buffers.  ``max_rows`` bounds the sequences a rank contributes per call.
    """

    def __init__(self, max_rows: int, device: torch.device | str, group=None) -> None:
        import torch.distributed as dist

        if max_rows <= 0:
            raise ValueError("max_rows must be positive")
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.max_rows = int(max_rows)
        self.device = torch.device(device)
        width = 1 + 3 * self.max_rows
        self._send = torch.zeros(width, dtype=torch.int64, device=self.device)
        self._recv = torch.zeros(self.world * width, dtype=torch.int64, device=self.device)
        self._bufs: list[tuple[torch.Tensor, torch.Tensor]] = []   # per started step (reused after finish)
        self._pending: list = []

    def _pack(self, send: torch.Tensor, sequence_ids, tokens, logprobs) -> None:
        ids = torch.as_tensor(sequence_ids, dtype=torch.int64).reshape(-1)
        tok = torch.as_tensor(tokens, dtype=torch.int64).reshape(-1)
        lp = torch.as_tensor(logprobs, dtype=torch.float32).reshape(-1)
        n = ids.numel()
        if tok.numel() != n or lp.numel() != n:
            raise ValueError("sequence_ids, tokens and logprobs must have one entry per row")
        if n > self.max_rows:
            raise ValueError(f"{n} rows exceed max_rows {self.max_rows}")
        send.zero_()
        send[0] = n
        rows = send[1:1 + 3 * n].view(n, 3)
        rows[:, 0] = ids.to(self.device)
        rows[:, 1] = tok.to(self.device)
        rows[:, 2] = lp.to(self.device).view(torch.int32).to(torch.int64)

    def _unpack(self, recv: torch.Tensor) -> GatheredStep:
        width = 1 + 3 * self.max_rows
        recv = recv.view(self.world, width).cpu()
        counts = [int(c) for c in recv[:, 0].tolist()]
        parts = [recv[r, 1:1 + 3 * counts[r]].view(counts[r], 3) for r in range(self.world)]
        allrows = torch.cat(parts) if parts else recv.new_zeros((0, 3))
        return GatheredStep(sequence_ids=allrows[:, 0].clone(), tokens=allrows[:, 1].clone(),
                            logprobs=allrows[:, 2].to(torch.int32).view(torch.float32).clone(), counts=counts)

    def start(self, sequence_ids, tokens, logprobs) -> None:
        """``gather`` without waiting: the collective runs behind the caller's next work (it starts
        after the work already on the current stream, which does not wait for it); ``finish``
        returns the steps started so far, in order."""
        width = 1 + 3 * self.max_rows
        k = len(self._pending)
        if k >= len(self._bufs):
            self._bufs.append((torch.zeros(width, dtype=torch.int64, device=self.device),
                               torch.zeros(self.world * width, dtype=torch.int64, device=self.device)))
        send, recv = self._bufs[k]
        self._pack(send, sequence_ids, tokens, logprobs)
        work = self.dist.all_gather_into_tensor(recv, send, group=self.group, async_op=True)
        self._pending.append((work, recv))

    def finish(self) -> list[GatheredStep]:
        out = []
        for work, recv in self._pending:
            work.wait()
            out.append(self._unpack(recv))
        self._pending.clear()
        return out

    def gather(self, sequence_ids, tokens, logprobs) -> GatheredStep:
        ids = torch.as_tensor(sequence_ids, dtype=torch.int64).reshape(-1)
        tok = torch.as_tensor(tokens, dtype=torch.int64).reshape(-1)
        lp = torch.as_tensor(logprobs, dtype=torch.float32).reshape(-1)
        n = ids.numel()
        if tok.numel() != n or lp.numel() != n:
            raise ValueError("sequence_ids, tokens and logprobs must have one entry per row")
        if n > self.max_rows:
            raise ValueError(f"{n} rows exceed max_rows {self.max_rows}")
        send = self._send
        send.zero_()
        send[0] = n
        rows = send[1:1 + 3 * n].view(n, 3)
        rows[:, 0] = ids.to(self.device)
        rows[:, 1] = tok.to(self.device)
        rows[:, 2] = lp.to(self.device).view(torch.int32).to(torch.int64)
        self.dist.all_gather_into_tensor(self._recv, send, group=self.group)
        width = 1 + 3 * self.max_rows
        recv = self._recv.view(self.world, width)
        counts = [int(c) for c in recv[:, 0].tolist()]
        parts = [recv[r, 1:1 + 3 * counts[r]].view(counts[r], 3) for r in range(self.world)]
        allrows = torch.cat(parts) if parts else recv.new_zeros((0, 3))
        return GatheredStep(
            sequence_ids=allrows[:, 0].clone(),
            tokens=allrows[:, 1].clone(),
            logprobs=allrows[:, 2].to(torch.int32).view(torch.float32).clone(),
            counts=counts,
        )


def balance_ratio(prompt_lens, group_size: int, assignment: list[int], world: int) -> float:
    """Most loaded rank's KV tokens over the mean (1.0 = perfect balance)."""
    load = np.zeros(world)
    for g, r in enumerate(assignment):
        load[r] += int(prompt_lens[g]) * group_size
    mean = load.mean()
    return float(load.max() / mean) if mean > 0 else 1.0
