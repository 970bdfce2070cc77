"""Multi-rank host logic of the paged-KV path, on CPU with gloo (world size 2).

GRPO groups are assigned to ranks (``assign_groups``), and the only per-step
exchange is the gather of every rank's (sequence id, token, log-probability)
rows (``StepGather``).  Failure detection is tested on the host: a rank that
leaves before the step's gather makes the surviving rank's collective fail
within the process group's timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from randomrepo_b200.sharding import StepGather, assign_groups, balance_ratio, groups_of_rank


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_assign_groups_modulo_and_balanced():
    lens = [4096, 256, 300, 3900, 1024, 512, 2048, 260]
    assert assign_groups(lens, 8, 4, "modulo") == [0, 1, 2, 3, 0, 1, 2, 3]
    bal = assign_groups(lens, 8, 4, "balanced")
    assert sorted(set(bal)) == [0, 1, 2, 3]
    assert assign_groups(lens, 8, 4, "balanced") == bal  # deterministic
    assert balance_ratio(lens, 8, bal, 4) <= balance_ratio(lens, 8, assign_groups(lens, 8, 4, "modulo"), 4)
    # every group exactly once
    assert sorted(g for r in range(4) for g in groups_of_rank(bal, r)) == list(range(len(lens)))


def test_assign_groups_balanced_on_the_7b_rollout_shape():
    rng = np.random.default_rng(0)
    lens = rng.integers(256, 4097, size=512 // 8 * 8)  # 64 groups of 8 per GPU on 8 GPUs
    bal = assign_groups(lens, 8, 8)
    assert balance_ratio(lens, 8, bal, 8) < 1.02
    assert balance_ratio(lens, 8, assign_groups(lens, 8, 8, "modulo"), 8) > balance_ratio(lens, 8, bal, 8)


def test_assign_groups_rejects_bad_arguments():
    with pytest.raises(ValueError):
        assign_groups([1, 2], 8, 0)
    with pytest.raises(ValueError):
        assign_groups([1, -2], 8, 2)
    with pytest.raises(ValueError):
        assign_groups([1, 2], 8, 2, "random")


def _gather_worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        g = StepGather(max_rows=8, device="cpu")
        out = []
        for step in range(3):
            n = 3 if rank == 0 else 5 - step  # unequal and changing row counts
            ids = torch.arange(n) + 100 * rank
            tok = torch.arange(n) * 7 + step
            lp = -torch.arange(n, dtype=torch.float32) / (rank + 1) - step
            if rank == 1 and step == 2:
                lp[0] = float("-inf")
                lp[1] = float("nan")
            got = g.gather(ids, tok, lp)
            out.append((got.counts, got.sequence_ids.tolist(), got.tokens.tolist(),
                        got.logprobs.view(torch.int32).tolist()))
            g.start(ids, tok, lp)  # the same rows through the non-blocking form
        for a, b in zip(g.finish(), out):
            assert (a.counts, a.sequence_ids.tolist(), a.tokens.tolist(), a.logprobs.view(torch.int32).tolist()) == b
        dist.destroy_process_group()
        results[rank] = out
    except Exception:  # noqa: BLE001 - reported to the parent
        results[rank] = traceback.format_exc()


def test_step_gather_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        res = dict(results)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    assert res[0] == res[1]  # every rank sees the same rows
    for step, (counts, ids, tok, lpbits) in enumerate(res[0]):
        assert counts == [3, 5 - step]
        want_ids = list(range(3)) + [100 + i for i in range(5 - step)]
        assert ids == want_ids
        assert tok == [i * 7 + step for i in range(3)] + [i * 7 + step for i in range(5 - step)]
        lp0 = (-torch.arange(3, dtype=torch.float32) - step)
        lp1 = (-torch.arange(5 - step, dtype=torch.float32) / 2 - step)
        if step == 2:
            lp1[0] = float("-inf")
            lp1[1] = float("nan")
        want = torch.cat([lp0, lp1]).view(torch.int32).tolist()
        assert lpbits == want  # bit-exact, -inf and NaN included


def _dropout_worker(rank: int, world: int, port: int, results) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    g = StepGather(max_rows=4, device="cpu")
    g.gather([rank], [1], [0.5])  # step 0: both ranks
    if rank == 1:
        results[rank] = "left"
        os._exit(0)  # the rank leaves between steps, with nothing in flight
    try:
        g.gather([rank], [2], [0.25])  # step 1: the peer is gone
        results[rank] = "no error"
    except Exception as e:  # noqa: BLE001
        results[rank] = f"error: {type(e).__name__}"
    os._exit(0)


def test_step_gather_detects_a_rank_that_left():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=90)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        res = dict(results)
    assert not alive, "a rank hung instead of failing"
    assert res.get(1) == "left"
    assert str(res.get(0, "")).startswith("error"), res
