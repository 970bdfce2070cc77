"""Systems-benchmark summaries on CPU: the reference's schema, aggregation and verdict rules.

``randomrepo_b200.systems`` reduces per-step telemetry rows the way AgentRL's
examples/benchmark_systems.py:113-350 does; the rows here are synthetic, and
the runs themselves are exercised in tests/test_gpu_systems.py.
"""

from __future__ import annotations

from collections import Counter

from randomrepo_b200.systems import (comparison_verdict, diagnose_run, render_comparison_table,
                                     single_run_verdict, summarize_run)

SUMMARY_KEYS = {
    "model_name", "task_name", "split", "hardware", "config_hash", "steps", "mode_name", "use_continuous_batching",
    "use_paged_kv_continuous", "mean_reward", "mean_reward_std", "mean_step_time_ms", "mean_generation_fraction",
    "mean_training_fraction", "mean_tokens_per_second", "mean_prefill_tokens_per_second",
    "mean_decode_tokens_per_second", "mean_padding_ratio", "mean_generation_padding_ratio",
    "mean_sequence_padding_ratio", "mean_cache_reuse_effectiveness", "mean_scheduler_prefill_passes",
    "mean_scheduler_decode_passes", "mean_scheduler_prefill_kv_budget_mb", "mean_scheduler_decode_kv_budget_mb",
    "mean_scheduler_prefill_admitted_kv_mb", "mean_scheduler_decode_admitted_kv_mb",
    "mean_scheduler_length_sort_passes", "mean_scheduler_length_sorted_sequences", "mean_scheduler_kv_pressure",
    "mean_scheduler_deferred_sequences", "mean_scheduler_max_concurrent_sequences", "peak_vram_mb",
    "rollout_peak_vram_mb", "min_rollout_runtime_headroom_mb", "mean_runtime_adjustments",
    "steps_with_runtime_adjustment", "steps_with_low_headroom", "dominant_runtime_bottleneck",
    "bottleneck_step_counts", "runtime_adjustment_reason_counts", "top_runtime_recommendation",
    "efficiency_diagnosis", "benchmark_verdict",
}


def _rows():
    return [
        {"total_step_time_ms": 100.0, "generation_time_ms": 80.0, "training_time_ms": 0.0, "tokens_per_second": 500.0,
         "dominant_runtime_bottleneck": "decode", "paged_kv_allocator_pressure": 0.25, "peak_vram_mb": 900.0,
         "rollout_runtime_headroom_mb": 1000.0, "runtime_adjustments": 0.0},
        {"total_step_time_ms": 120.0, "generation_time_ms": 90.0, "training_time_ms": 0.0, "tokens_per_second": 700.0,
         "dominant_runtime_bottleneck": "decode", "paged_kv_allocator_pressure": 0.5, "peak_vram_mb": 1100.0,
         "rollout_runtime_headroom_mb": 800.0, "runtime_adjustments": 1.0,
         "last_runtime_adjustment_reason": "oom_retry", "runtime_recommendation": "Lower the batch."},
    ]


def test_summary_keys_and_aggregation():
    s = summarize_run(_rows(), mode_name="paged-kv continuous batching", model_name="m", task_name="t", split="s",
                      config_fields={"a": 1}, use_continuous_batching=True, use_paged_kv_continuous=True)
    assert set(s) == SUMMARY_KEYS
    assert s["steps"] == 2 and s["mean_step_time_ms"] == 110.0 and s["mean_tokens_per_second"] == 600.0
    assert abs(s["mean_generation_fraction"] - (0.8 + 0.75) / 2) < 1e-12
    assert s["mean_scheduler_kv_pressure"] == 0.375
    assert s["peak_vram_mb"] == 1100.0 and s["min_rollout_runtime_headroom_mb"] == 800.0
    assert s["steps_with_runtime_adjustment"] == 1
    assert s["runtime_adjustment_reason_counts"] == {"oom_retry": 1}
    assert s["efficiency_diagnosis"] == "memory-constrained but recoverable"
    assert s["benchmark_verdict"] == ("paged-kv continuous batching was memory-constrained but recoverable, "
                                      "dominated by decode, and needed 1 runtime adjustment. Lower the batch.")
    assert len(s["config_hash"]) == 12


def test_diagnosis_labels_and_verdicts():
    assert diagnose_run([], "padding", Counter()) == "padding-limited"
    assert diagnose_run([], "decode_without_cache_reuse", Counter()) == "decode-limited"
    assert diagnose_run([{"runtime_adjustments": 2}], "unknown", Counter()) == "runtime-adjusted"
    assert diagnose_run([], "unknown", Counter()) == "balanced"
    assert single_run_verdict(mode_name="x", efficiency_diagnosis="balanced", dominant_bottleneck="balanced",
                              steps_with_runtime_adjustment=2, top_runtime_recommendation="") == (
        "x was balanced, and needed 2 runtime adjustments.")


def test_comparison_verdict_and_table():
    a = summarize_run(_rows()[:1], mode_name="standard rollout", model_name="m", task_name="t", split="s",
                      config_fields={}, use_continuous_batching=False, use_paged_kv_continuous=False)
    b = summarize_run([dict(_rows()[0], total_step_time_ms=40.0)], mode_name="paged-kv continuous batching",
                      model_name="m", task_name="t", split="s", config_fields={}, use_continuous_batching=True,
                      use_paged_kv_continuous=True)
    v = comparison_verdict([a, b])
    assert v.startswith("Fastest overall: paged-kv continuous batching (40.00 ms")
    assert "60.00 ms faster than standard rollout" in v and v.endswith("without runtime adjustment.")
    assert comparison_verdict([a]) == "Comparison verdict unavailable."
    table = render_comparison_table([a, b]).splitlines()
    assert table[0].startswith("| Mode | Mean reward | Mean step ms | Tokens/s")
    assert len(table) == 4 and table[3].startswith("| paged-kv continuous batching | 0.0000 | 40.00 |")
