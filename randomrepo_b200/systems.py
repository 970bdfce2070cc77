"""Rollout systems benchmark: AgentRL's runtime-mode summaries for the paged modes.

AgentRL's harness (examples/benchmark_systems.py:113-329) trains a model with
``GRPOTrainer`` on a task for a few steps in each runtime mode and reduces the
per-step telemetry rows to one summary per mode, a diagnosis, a verdict, a
head-to-head comparison and a markdown table.  The trainer, tasks and
verifiers are outside the paged-KV path, so here a step is what the path
runs: one GRPO rollout (prompts x group, sampled) plus its old-policy
log-probability pass, on seeded synthetic prompts (random token ids of a
given length range) with random-init Qwen2 weights of a named architecture.
Each mode records per-step rows under the telemetry keys the reference's
summary reads; ``summarize_run``, ``diagnose_run``, ``single_run_verdict``,
``comparison_verdict`` and ``render_comparison_table`` produce the
reference's summary keys and strings from them.  Keys with no counterpart
here (reward, runtime-controller adjustments, scheduler budgets) read 0.

Modes:
* ``standard rollout`` -- stock HF ``generate`` over the left-padded batch,
  then the reference's old-policy pass (one padded forward, log_softmax over
  [B, L-1, vocab], gather);
* ``paged-kv continuous batching`` -- ``PagedGenerator`` (packed prefill,
  copy-on-write group forks, CUDA-graph decode steps) and
  ``PagedGenerator.score``;
* ``speculative decoding`` -- ``PagedSpeculativeGenerator`` with a draft
  model, then ``score`` on the target.

Usage::

    python -m randomrepo_b200.systems --arch qwen2.5-1.5b --steps 3 --compare-runtime-modes \\
        [--include-speculative --draft-arch qwen2.5-0.5b] --output-dir ./systems_benchmark
"""

from __future__ import annotations

import argparse
import hashlib
import json
import platform
from collections import Counter
from pathlib import Path
from statistics import mean

import numpy as np
import torch

ARCHS = {
    "qwen2.5-0.5b": dict(vocab_size=151936, hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                         num_attention_heads=14, num_key_value_heads=2, tie_word_embeddings=True),
    "qwen2.5-1.5b": dict(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=28,
                         num_attention_heads=12, num_key_value_heads=2, tie_word_embeddings=True),
    "qwen2.5-7b": dict(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                       num_attention_heads=28, num_key_value_heads=4, tie_word_embeddings=False),
    # A few-layer shape for smoke runs and tests.
    "tiny": dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=False),
}

MODES = ("standard rollout", "paged-kv continuous batching", "speculative decoding")


# ---------------------------------------------------------------------------
# Summaries (the reference's schema and rules).

def _mean(rows, key: str) -> float:
    return mean(float(r.get(key, 0.0)) for r in rows) if rows else 0.0


def diagnose_run(history: list[dict], dominant_bottleneck: str, adjustment_reason_counts: Counter) -> str:
    """Run-level diagnosis from per-step signals (benchmark_systems.py:209-233)."""
    if any("oom_" in reason for reason in adjustment_reason_counts):
        return "memory-constrained but recoverable"
    labels = {"padding": "padding-limited", "kv_budget": "kv-budget-limited", "paged_kv": "paged-kv-limited",
              "decode": "decode-limited", "decode_without_cache_reuse": "decode-limited", "prefill": "prefill-limited"}
    if dominant_bottleneck in labels:
        return labels[dominant_bottleneck]
    if any(float(r.get("runtime_adjustments", 0.0)) > 0.0 for r in history):
        return "runtime-adjusted"
    return "balanced"


def single_run_verdict(*, mode_name: str, efficiency_diagnosis: str, dominant_bottleneck: str,
                       steps_with_runtime_adjustment: int, top_runtime_recommendation: str) -> str:
    """One-line verdict of a run (benchmark_systems.py:236-256)."""
    parts = [f"{mode_name} was {efficiency_diagnosis}"]
    if dominant_bottleneck != "balanced":
        parts.append(f", dominated by {dominant_bottleneck.replace('_', ' ')}")
    if steps_with_runtime_adjustment > 0:
        plural = "" if steps_with_runtime_adjustment == 1 else "s"
        parts.append(f", and needed {steps_with_runtime_adjustment} runtime adjustment{plural}")
    text = "".join(parts) + "."
    return f"{text} {top_runtime_recommendation}" if top_runtime_recommendation else text


def config_hash(fields: dict) -> str:
    """Short hash of the run's configuration (benchmark_systems.py:82-100)."""
    return hashlib.sha256(json.dumps(fields, sort_keys=True).encode("utf-8")).hexdigest()[:12]


def hardware_string() -> str:
    if torch.cuda.is_available():
        return torch.cuda.get_device_name(0)
    return f"cpu:{platform.processor() or platform.machine()}"


def summarize_run(history: list[dict], *, mode_name: str, model_name: str, task_name: str, split: str,
                  config_fields: dict, use_continuous_batching: bool, use_paged_kv_continuous: bool) -> dict:
    """Aggregate per-step rows into the reference's run summary (benchmark_systems.py:113-206)."""
    def frac(key):
        return [float(r.get(key, 0.0)) / max(float(r.get("total_step_time_ms", 1e-6)), 1e-6) for r in history]

    bottlenecks = Counter(str(r.get("dominant_runtime_bottleneck", "unknown")) for r in history)
    reasons = Counter(str(r.get("last_runtime_adjustment_reason", "none")) for r in history
                      if str(r.get("last_runtime_adjustment_reason", "none")) != "none")
    recommendations = Counter(str(r.get("runtime_recommendation", "")) for r in history
                              if r.get("runtime_recommendation"))
    dominant = bottlenecks.most_common(1)[0][0] if bottlenecks else "unknown"
    top_rec = recommendations.most_common(1)[0][0] if recommendations else ""
    adjusted = sum(1 for r in history if float(r.get("runtime_adjustments", 0.0)) > 0.0)
    diagnosis = diagnose_run(history, dominant, reasons)
    summary = {
        "model_name": model_name,
        "task_name": task_name,
        "split": split,
        "hardware": hardware_string(),
        "config_hash": config_hash(config_fields),
        "steps": len(history),
        "mode_name": mode_name,
        "use_continuous_batching": use_continuous_batching,
        "use_paged_kv_continuous": use_paged_kv_continuous,
        "mean_reward": _mean(history, "mean_reward"),
        "mean_reward_std": _mean(history, "reward_std"),
        "mean_step_time_ms": _mean(history, "total_step_time_ms"),
        "mean_generation_fraction": mean(frac("generation_time_ms")) if history else 0.0,
        "mean_training_fraction": mean(frac("training_time_ms")) if history else 0.0,
    }
    for key in ("tokens_per_second", "prefill_tokens_per_second", "decode_tokens_per_second", "padding_ratio",
                "generation_padding_ratio", "sequence_padding_ratio", "cache_reuse_effectiveness",
                "scheduler_prefill_passes", "scheduler_decode_passes", "scheduler_prefill_kv_budget_mb",
                "scheduler_decode_kv_budget_mb", "scheduler_prefill_admitted_kv_mb",
                "scheduler_decode_admitted_kv_mb", "scheduler_length_sort_passes",
                "scheduler_length_sorted_sequences"):
        summary[f"mean_{key}"] = _mean(history, key)
    summary["mean_scheduler_kv_pressure"] = mean(
        max(float(r.get("scheduler_prefill_kv_pressure", 0.0)), float(r.get("scheduler_decode_kv_pressure", 0.0)),
            float(r.get("paged_kv_allocator_pressure", 0.0))) for r in history) if history else 0.0
    summary["mean_scheduler_deferred_sequences"] = _mean(history, "scheduler_deferred_sequences")
    summary["mean_scheduler_max_concurrent_sequences"] = _mean(history, "scheduler_max_concurrent_sequences")
    summary["peak_vram_mb"] = max((float(r.get("peak_vram_mb", 0.0)) for r in history), default=0.0)
    summary["rollout_peak_vram_mb"] = max((float(r.get("rollout_peak_vram_mb", 0.0)) for r in history), default=0.0)
    summary["min_rollout_runtime_headroom_mb"] = min(
        (float(r.get("rollout_runtime_headroom_mb", 0.0)) for r in history), default=0.0)
    summary["mean_runtime_adjustments"] = _mean(history, "runtime_adjustments")
    summary["steps_with_runtime_adjustment"] = adjusted
    summary["steps_with_low_headroom"] = sum(1 for r in history if float(r.get("runtime_low_headroom", 0.0)) > 0.0)
    summary["dominant_runtime_bottleneck"] = dominant
    summary["bottleneck_step_counts"] = dict(sorted(bottlenecks.items()))
    summary["runtime_adjustment_reason_counts"] = dict(sorted(reasons.items()))
    summary["top_runtime_recommendation"] = top_rec
    summary["efficiency_diagnosis"] = diagnosis
    summary["benchmark_verdict"] = single_run_verdict(
        mode_name=mode_name, efficiency_diagnosis=diagnosis, dominant_bottleneck=dominant,
        steps_with_runtime_adjustment=adjusted, top_runtime_recommendation=top_rec)
    return summary


def comparison_verdict(summaries: list[dict]) -> str:
    """Head-to-head conclusion (benchmark_systems.py:259-291)."""
    if len(summaries) < 2:
        return "Comparison verdict unavailable."
    ordered = sorted(summaries, key=lambda s: float(s["mean_step_time_ms"]))
    fastest, slowest = ordered[0], ordered[-1]
    text = (f"Fastest overall: {fastest['mode_name']} ({float(fastest['mean_step_time_ms']):.2f} ms mean step "
            f"time, {fastest['efficiency_diagnosis']}). Slowest overall: {slowest['mode_name']} "
            f"({float(slowest['mean_step_time_ms']):.2f} ms).")
    by_mode = {str(s["mode_name"]): s for s in summaries}
    legacy = by_mode.get("continuous batching") or by_mode.get("standard rollout")
    paged = by_mode.get("paged-kv continuous batching")
    if legacy is not None and paged is not None:
        delta = float(legacy["mean_step_time_ms"]) - float(paged["mean_step_time_ms"])
        text += (f" Paged-KV continuous batching was {abs(delta):.2f} ms {'faster' if delta > 0 else 'slower'} "
                 f"than {legacy['mode_name']} ({float(paged['mean_step_time_ms']):.2f} ms vs "
                 f"{float(legacy['mean_step_time_ms']):.2f} ms).")
    adjusted = int(fastest["steps_with_runtime_adjustment"])
    if adjusted > 0:
        text += f" Fastest mode needed {adjusted} runtime adjustment{'' if adjusted == 1 else 's'}."
    elif all(int(s["steps_with_runtime_adjustment"]) == 0 for s in summaries):
        text += " All modes stayed stable without runtime adjustment."
    return text


def render_comparison_table(summaries: list[dict]) -> str:
    """Markdown table of the summaries (benchmark_systems.py:330-350 columns)."""
    lines = [
        "| Mode | Mean reward | Mean step ms | Tokens/s | Padding ratio | KV pressure | Deferred seqs | Max concurrent "
        "| Runtime diagnosis | Bottleneck | Adjusted steps | Peak VRAM MB |",
        "|---|---:|---:|---:|---:|---:|---:|---:|---|---|---:|---:|",
    ]
    for s in summaries:
        lines.append(
            f"| {s['mode_name']} | {s['mean_reward']:.4f} | {s['mean_step_time_ms']:.2f} | "
            f"{s['mean_tokens_per_second']:.2f} | {s['mean_padding_ratio']:.4f} | "
            f"{s['mean_scheduler_kv_pressure']:.2f} | {s['mean_scheduler_deferred_sequences']:.2f} | "
            f"{s['mean_scheduler_max_concurrent_sequences']:.2f} | {s['efficiency_diagnosis']} | "
            f"{s['dominant_runtime_bottleneck']} | {s['steps_with_runtime_adjustment']} | {s['peak_vram_mb']:.2f} |")
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# Running the modes.

def build_model(arch: str, device: torch.device, seed: int):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    with torch.device(device):
        return Qwen2ForCausalLM(Qwen2Config(**ARCHS[arch], max_position_embeddings=32768, rope_theta=1000000.0,
                                            attn_implementation="sdpa")).to(torch.bfloat16).eval()


def set_attention(model, name: str) -> None:
    model.config._attn_implementation = name
    for sub in model.modules():
        cfg = getattr(sub, "config", None)
        if cfg is not None:
            cfg._attn_implementation = name


def synthetic_prompts(n: int, lo: int, hi: int, vocab: int, seed: int) -> list[torch.Tensor]:
    rng = np.random.default_rng(seed)
    return [torch.from_numpy(rng.integers(0, vocab, size=int(m))) for m in rng.integers(lo, hi + 1, size=n)]


def _score_inputs(prompts, tokens, group: int):
    rows = [torch.cat([prompts[i // group], torch.tensor(t, dtype=torch.long)]) for i, t in enumerate(tokens)]
    width = max(r.numel() for r in rows)
    ids = torch.zeros(len(rows), width, dtype=torch.long)
    am = torch.zeros_like(ids)
    cm = torch.zeros(len(rows), width, dtype=torch.bool)
    for i, r in enumerate(rows):
        ids[i, :r.numel()] = r
        am[i, :r.numel()] = 1
        cm[i, prompts[i // group].numel():r.numel()] = True
    return ids, am, cm


class _Clock:
    def __init__(self):
        self.e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def mark(self, i: int) -> None:
        self.e[i].record()

    def ms(self, a: int, b: int) -> float:
        self.e[b].synchronize()
        return self.e[a].elapsed_time(self.e[b])


def run_mode(mode: str, model, prompts, *, group: int, new_tokens: int, steps: int, temperature: float,
             draft=None, k: int = 4, total_blocks: int = 16384, seed: int = 0) -> list[dict]:
    """Per-step telemetry rows of one mode (one warm-up step first, not recorded)."""
    from .hf import PagedGenerator, SamplingConfig, make_store
    from .speculative import PagedSpeculativeGenerator

    device = next(model.parameters()).device
    total_mb = torch.cuda.get_device_properties(device).total_memory / 2**20
    prompt_tokens = sum(int(p.numel()) for p in prompts)
    rows = []
    gen = spec = None
    if mode == "paged-kv continuous batching":
        gen = PagedGenerator(model, make_store(model, total_blocks), cuda_graphs=True)
    elif mode == "speculative decoding":
        if draft is None:
            raise ValueError("speculative decoding needs a draft model")
        gen = PagedGenerator(model, make_store(model, total_blocks), cuda_graphs=True)
        dgen = PagedGenerator(draft, make_store(draft, total_blocks), cuda_graphs=True, sampler=gen.sampler)
        spec = PagedSpeculativeGenerator(gen, dgen, k=k)
    elif mode == "standard rollout":
        set_attention(model, "sdpa")
    else:
        raise ValueError(f"unknown mode {mode!r}")

    for step in range(steps + 1):
        cfg = SamplingConfig(do_sample=True, temperature=temperature, seed=seed + step)
        torch.cuda.synchronize(device)
        torch.cuda.reset_peak_memory_stats(device)
        base_mb = torch.cuda.memory_allocated(device) / 2**20
        clock = _Clock()
        clock.mark(0)
        row = {"mean_reward": 0.0, "reward_std": 0.0, "training_time_ms": 0.0, "runtime_adjustments": 0.0,
               "last_runtime_adjustment_reason": "none"}
        if mode == "standard rollout":
            width = max(int(p.numel()) for p in prompts)
            ids = torch.zeros((len(prompts) * group, width), dtype=torch.long)
            mask = torch.zeros_like(ids)
            for g, p in enumerate(prompts):
                ids[g * group:(g + 1) * group, -p.numel():] = p
                mask[g * group:(g + 1) * group, -p.numel():] = 1
            with torch.inference_mode():
                out = model.generate(ids.to(device), attention_mask=mask.to(device), max_new_tokens=new_tokens,
                                     do_sample=True, temperature=temperature, top_p=1.0, top_k=0, pad_token_id=0)
            tokens = out[:, width:].tolist()
            clock.mark(1)
            sids, sam, scm = _score_inputs(prompts, tokens, group)
            with torch.inference_mode():
                d = sids.to(device)
                logits = model(input_ids=d, attention_mask=sam.to(device)).logits
                lp = torch.log_softmax(logits[:, :-1, :], dim=-1).gather(-1, d[:, 1:].unsqueeze(-1)).squeeze(-1)
                _ = lp * scm[:, 1:].to(device=device, dtype=lp.dtype)
            clock.mark(2)
            pad = 1.0 - float(mask.sum()) / mask.numel()
            gen_ms = clock.ms(0, 1)
            row.update(padding_ratio=pad, generation_padding_ratio=pad, sequence_padding_ratio=pad,
                       prefill_tokens_per_second=0.0, decode_tokens_per_second=0.0, cache_reuse_effectiveness=0.0,
                       dominant_runtime_bottleneck="padding" if pad > 0.3 else "decode")
            decode_tokens = len(tokens) * new_tokens
        else:
            if spec is not None:
                res = spec.generate(prompts, group_size=group, max_new_tokens=new_tokens, sampling=cfg,
                                    first_id=step * 100000)
                timings = {}
            else:
                res = gen.generate(prompts, group_size=group, max_new_tokens=new_tokens, sampling=cfg,
                                   first_id=step * 100000)
                timings = dict(gen.last_timings)
            tokens = res["tokens"]
            clock.mark(1)
            alloc = gen.store.allocator
            pressure = alloc.max_blocks_in_use / alloc.total_blocks  # the pool's high watermark
            sids, sam, scm = _score_inputs(prompts, tokens, group)
            gen.score(sids, sam, scm, group_size=group)
            clock.mark(2)
            gen_ms = clock.ms(0, 1)
            decode_tokens = sum(len(t) for t in tokens)
            shared, used = timings.get("shared_blocks_after_prefill", (0, 0))
            pre_ms, dec_ms = timings.get("prefill_ms", 0.0), timings.get("decode_ms", gen_ms)
            kvp = res.get("kv_pressure", {})
            preempted = float(kvp.get("paged_kv_preempted_sequences", 0.0))
            # The runtime controller's rule (agentrl/runtime/controller.py:175-181): a full pool
            # that preempted sequences makes the step paged-KV bound.
            if pressure >= 0.9 and preempted > 0:
                bottleneck = "paged_kv"
            else:
                bottleneck = "prefill" if pre_ms > dec_ms else "decode"
            row.update(padding_ratio=0.0, generation_padding_ratio=0.0, sequence_padding_ratio=0.0,
                       prefill_tokens_per_second=prompt_tokens / max(pre_ms, 1e-6) * 1e3 if pre_ms else 0.0,
                       decode_tokens_per_second=decode_tokens / max(dec_ms, 1e-6) * 1e3,
                       cache_reuse_effectiveness=shared / used if used else 0.0,
                       paged_kv_allocator_pressure=pressure,
                       paged_kv_preempted_sequences=preempted,
                       paged_kv_max_preempted_sequences=float(kvp.get("paged_kv_max_preempted_sequences", 0.0)),
                       dominant_runtime_bottleneck=bottleneck)
            if spec is not None:
                row["speculative_acceptance_rate"] = res["accepted"] / max(res["proposed"], 1)
        total_ms = clock.ms(0, 2)
        peak_mb = torch.cuda.max_memory_allocated(device) / 2**20
        row.update(generation_time_ms=gen_ms, total_step_time_ms=total_ms,
                   old_policy_time_ms=total_ms - gen_ms,
                   tokens_per_second=decode_tokens / max(gen_ms, 1e-6) * 1e3,
                   peak_vram_mb=peak_mb, rollout_peak_vram_mb=peak_mb - base_mb,
                   rollout_runtime_headroom_mb=total_mb - peak_mb, runtime_low_headroom=0.0,
                   scheduler_max_concurrent_sequences=float(len(prompts) * group))
        if step > 0:
            rows.append(row)
    return rows


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="Run GRPO rollouts in each runtime mode and summarize them.")
    ap.add_argument("--arch", default="qwen2.5-1.5b", choices=sorted(ARCHS))
    ap.add_argument("--draft-arch", default="qwen2.5-0.5b", choices=sorted(ARCHS))
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--batch-size", type=int, default=4, help="prompts per step")
    ap.add_argument("--group-size", type=int, default=8)
    ap.add_argument("--max-new-tokens", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, nargs=2, default=(64, 256))
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--speculative-k", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--output-dir", default="./systems_benchmark")
    ap.add_argument("--compare-runtime-modes", action="store_true")
    ap.add_argument("--include-speculative", action="store_true")
    return ap


def main(argv=None) -> dict:
    args = build_parser().parse_args(argv)
    device = torch.device("cuda", torch.cuda.current_device())
    out_dir = Path(args.output_dir).expanduser()
    out_dir.mkdir(parents=True, exist_ok=True)
    model = build_model(args.arch, device, args.seed)
    prompts = synthetic_prompts(args.batch_size, args.prompt_len[0], args.prompt_len[1],
                                ARCHS[args.arch]["vocab_size"], args.seed)
    modes = list(MODES[:2]) if args.compare_runtime_modes else ["paged-kv continuous batching"]
    draft = None
    if args.include_speculative:
        modes.append("speculative decoding")
        draft = build_model(args.draft_arch, device, args.seed + 1)
    fields = {"model_name": args.arch, "steps": args.steps, "batch_size": args.batch_size,
              "group_size": args.group_size, "max_new_tokens": args.max_new_tokens, "task_name": "synthetic",
              "split": "seeded"}
    summaries = []
    for mode in modes:
        history = run_mode(mode, model, prompts, group=args.group_size, new_tokens=args.max_new_tokens,
                           steps=args.steps, temperature=args.temperature, draft=draft, k=args.speculative_k,
                           seed=args.seed)
        summary = summarize_run(history, mode_name=mode, model_name=args.arch, task_name="synthetic",
                                split="seeded", config_fields=dict(fields, mode=mode),
                                use_continuous_batching=mode != "standard rollout",
                                use_paged_kv_continuous=mode != "standard rollout")
        sub = out_dir / mode.replace(" ", "_").replace("-", "_")
        sub.mkdir(parents=True, exist_ok=True)
        (sub / "summary.json").write_text(json.dumps(summary, indent=2) + "\n", encoding="utf-8")
        (sub / "history.json").write_text(json.dumps(history, indent=2) + "\n", encoding="utf-8")
        summaries.append(summary)
    comparison = {"hardware": hardware_string(), "task_name": "synthetic", "split": "seeded",
                  "model_name": args.arch, "runs": summaries, "comparison_verdict": comparison_verdict(summaries)}
    (out_dir / "comparison.json").write_text(json.dumps(comparison, indent=2) + "\n", encoding="utf-8")
    print(render_comparison_table(summaries))
    print()
    print(comparison["comparison_verdict"])
    return comparison


if __name__ == "__main__":
    main()
