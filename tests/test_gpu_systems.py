"""The rollout systems benchmark runs every mode on the GPU and writes the reference's summaries."""

from __future__ import annotations

import json

import pytest

pytestmark = pytest.mark.gpu


def test_compare_runtime_modes_with_speculative(cuda_device, tmp_path):
    from randomrepo_b200 import systems

    comparison = systems.main(["--arch", "tiny", "--draft-arch", "tiny", "--steps", "2", "--batch-size", "3",
                               "--group-size", "2", "--max-new-tokens", "8", "--prompt-len", "8", "24",
                               "--compare-runtime-modes", "--include-speculative", "--output-dir", str(tmp_path)])
    runs = {r["mode_name"]: r for r in comparison["runs"]}
    assert list(runs) == list(systems.MODES)
    on_disk = json.loads((tmp_path / "comparison.json").read_text())
    assert on_disk["comparison_verdict"] == comparison["comparison_verdict"]
    for name, run in runs.items():
        assert run["steps"] == 2 and run["mean_step_time_ms"] > 0 and run["mean_tokens_per_second"] > 0
        sub = tmp_path / name.replace(" ", "_").replace("-", "_")
        history = json.loads((sub / "history.json").read_text())
        assert len(history) == 2 and all(h["total_step_time_ms"] >= h["generation_time_ms"] for h in history)
    assert runs["standard rollout"]["mean_padding_ratio"] > 0  # left padding of unequal prompts
    assert runs["paged-kv continuous batching"]["mean_padding_ratio"] == 0
    assert runs["paged-kv continuous batching"]["mean_cache_reuse_effectiveness"] > 0  # forked group prompts
    assert runs["paged-kv continuous batching"]["mean_decode_tokens_per_second"] > 0
