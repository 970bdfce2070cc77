"""The reference's own continuous-batching tests, run unchanged with the native allocator swapped in.

AgentRL's ``ContinuousBatchingOrchestrator`` imports ``PagedKVAllocator`` at
agentrl/generation/continuous.py:16 and drives it from its paged-KV loop: pool
sizing (continuous.py:821-857), prompt reservations, per-token
``append_tokens``, releases, the occupancy / reuse metrics it mirrors into its
runtime stats, growth admission against ``free_block_count``
(continuous.py:900-937) and the soft-preemption counters (continuous.py:875-898).
This module loads the reference's tests/test_continuous.py from a checkout of
the reference (``PKV_REFERENCE_ROOT``, or a ``reference`` directory beside
this repository), swaps that import for ``randomrepo_b200.PagedKVAllocator``
(the one-line swap of the integration guide) and runs every paged-KV test of
that file unchanged.  The loop's model math stays HF's on the CPU; what the
swap changes is every allocator call, so these tests check that the drop-in
gives the loop the block tables, counts and exceptions the reference's own
assertions expect.  Skipped when no reference checkout is found.
"""

from __future__ import annotations

import importlib.util
import inspect
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("PKV_REFERENCE_ROOT", ROOT.parent / "reference"))
REF_TESTS = REF / "tests" / "test_continuous.py"
pytestmark = pytest.mark.skipif(not ((REF / "agentrl").is_dir() and REF_TESTS.is_file()),
                                reason="no reference checkout beside the repository (set PKV_REFERENCE_ROOT)")

# The paged-KV tests of the reference's tests/test_continuous.py (use_paged_kv_continuous=True).
PAGED_TESTS = [
    "test_paged_kv_continuous_collects_block_metrics",
    "test_paged_kv_prefill_seeds_resident_caches",
    "test_continuous_scheduler_defers_sequences_under_safe_policy",
    "test_scheduler_costing_is_mode_aware",
    "test_paged_kv_continuous_collects_with_dynamic_cache_model",
    "test_paged_kv_continuous_decode_uses_resident_caches",
    "test_paged_kv_continuous_decode_keeps_legacy_materialization_available",
    "test_paged_kv_continuous_constructor_cache_keeps_legacy_materialization_available",
    "test_paged_kv_continuous_dynamic_cache_handles_block_growth",
    "test_paged_kv_releases_finished_sequences_and_keeps_resident_state",
]


def _reference_module():
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    spec = importlib.util.spec_from_file_location("agentrl_reference_test_continuous", REF_TESTS)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _outcome(fn, monkeypatch) -> str:
    kwargs = {"monkeypatch": monkeypatch} if "monkeypatch" in inspect.signature(fn).parameters else {}
    try:
        fn(**kwargs)
    except Exception as e:  # noqa: BLE001 - the outcome is compared, not judged here
        return f"{type(e).__name__}: {e}"
    return "passed"


@pytest.mark.parametrize("name", PAGED_TESTS)
def test_reference_continuous_test_ends_alike_with_the_native_allocator(name, monkeypatch):
    """Each test ends the same way with either allocator: it passes with both, or (where this image's
    transformers no longer has an API the reference's fake model calls) fails with the same error."""
    mod = _reference_module()
    import agentrl.generation.continuous as continuous

    from randomrepo_b200 import PagedKVAllocator

    made = []

    class CountingAllocator(PagedKVAllocator):
        def __init__(self, *args, **kwargs):
            super().__init__(*args, **kwargs)
            made.append(self)

    fn = getattr(mod, name)
    with monkeypatch.context() as m:
        want = _outcome(fn, m)
    with monkeypatch.context() as m:
        m.setattr(continuous, "PagedKVAllocator", CountingAllocator)
        got = _outcome(fn, m)
    assert got == want
    if want == "passed" and name != "test_scheduler_costing_is_mode_aware":  # that one never builds a pool
        assert made, "the loop did not build its pool through the swapped allocator"


def test_most_reference_paged_tests_run_to_completion():
    """The comparison above is only as strong as the tests that pass: at least half of them must."""
    mod = _reference_module()
    passed = 0
    for name in PAGED_TESTS:
        mp = pytest.MonkeyPatch()
        try:
            passed += _outcome(getattr(mod, name), mp) == "passed"
        finally:
            mp.undo()
    assert passed >= len(PAGED_TESTS) // 2, passed
