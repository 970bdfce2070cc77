"""Allocator parity on op traces recorded from the reference itself.

``allocator_traces.json`` holds seeded random reserve / append_tokens /
release / logical_to_physical traces run through the reference's
``PagedKVAllocator`` (agentrl/generation/paged_kv.py:25-175) with every
result, exception and metric; ``continuous_c1_trace.json`` holds the allocator
calls the reference's continuous loop made at the CPU-smoke shape.  Both the
oracle and the product allocator must reproduce them exactly.
"""

from __future__ import annotations

import pytest

from oracle.allocator import OracleAllocator
from tests.conftest import load_json

TRACES = load_json("allocator_traces.json")


def _product(total, bs):
    from randomrepo_b200 import PagedKVAllocator

    return PagedKVAllocator(total, bs)


IMPLS = {"oracle": OracleAllocator, "product": _product}


def _replay(alloc, trace):
    keys = trace["metric_keys"]
    for step, entry in enumerate(trace["ops"]):
        op = entry["op"]
        try:
            res = getattr(alloc, op[0])(*op[1:])
            if op[0] in ("reserve", "append_tokens"):
                got = {"ok": [res.sequence_id, res.token_count, res.block_size_tokens, list(res.physical_blocks)]}
            elif op[0] == "release":
                got = {"ok": None}
            else:
                got = {"ok": res}
        except Exception as exc:  # noqa: BLE001 - compared with the recorded exception
            got = {"error": type(exc).__name__, "message": str(exc)}
        assert got == entry["result"], f"step {step} {op}"
        metrics = alloc.metrics()
        assert [metrics[k] for k in keys] == entry["metrics"], f"step {step} {op}"


@pytest.mark.parametrize("impl", sorted(IMPLS))
@pytest.mark.parametrize("index", range(len(TRACES)))
def test_reference_trace(impl, index):
    trace = TRACES[index]
    _replay(IMPLS[impl](trace["total_blocks"], trace["block_size_tokens"]), trace)


def test_traces_cover_error_paths():
    kinds = {e["result"].get("error") for t in TRACES for e in t["ops"]}
    assert {"ValueError", "KeyError", "RuntimeError"} <= kinds


@pytest.mark.parametrize("impl", sorted(IMPLS))
def test_continuous_loop_trace(impl):
    """Replay the continuous loop's allocator calls (continuous.py:380-504, 821-857)."""
    trace = load_json("continuous_c1_trace.json")
    alloc = IMPLS[impl](64, 16)
    high = 0
    for call in trace["calls"]:
        if call[0] == "sample":
            continue
        getattr(alloc, call[0])(*call[1:])
        high = max(high, alloc.metrics()["paged_kv_max_blocks_in_use"])
    stats = trace["paged_kv_stats"]
    m = alloc.metrics()
    assert high == stats["paged_kv_max_blocks_in_use"]
    for key in ("paged_kv_free_block_count", "paged_kv_used_block_count", "paged_kv_block_reuse_count",
                "paged_kv_resident_sequences", "paged_kv_allocator_occupancy"):
        assert m[key] == stats[key], key
