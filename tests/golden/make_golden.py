"""Generate the golden fixtures of the paged-KV path by running the reference itself.

Run from the repository root, in a container where the AgentRL reference tree
is readable::

    python tests/golden/make_golden.py /path/to/agentrl/checkout

It imports ``agentrl.generation.paged_kv`` and ``agentrl.generation.continuous``
unchanged from that tree, and HF transformers' ``sdpa_attention_forward``
(the reference's attention, transformers 5.5.0), and writes:

* ``allocator_traces.json`` -- seeded random reserve/append/release/lookup op
  traces over ``PagedKVAllocator`` with every result, exception and metric;
* ``continuous_c1_trace.json`` -- the allocator calls, in order, made by
  ``ContinuousBatchingOrchestrator._generate_active_batch_with_cache`` on a
  random-init (seed 0) 2-layer Qwen2 at the CPU-smoke shape (hidden 64, 4/2
  heads, head_dim 16, vocab 512, fp32, 64-block pool of 16 tokens, 2 prompts x
  group 4, prompt lengths U[8,32], greedy, 16 new tokens), with the greedy
  tokens and the ``paged_kv_*`` runtime stats;
* ``store_roundtrip.npz`` -- ``PagedKVCacheStore.write_sequence_cache`` /
  ``read_sequence_legacy_cache`` round trips (fp32 and bf16 bit patterns,
  block sizes 2 and 16, ragged lengths);
* ``attention_sdpa.npz`` -- fp32 ``sdpa_attention_forward`` outputs for GQA
  decode, chunked prefill after a cached past, and the k+1-query verify rows
  of a full causal forward, on bf16-representable inputs;
* ``speculative_c1_trace.json`` -- ``SpeculativeRolloutOrchestrator.
  _generate_speculative_tokens`` (agentrl/generation/speculative.py) on CPU
  with the C1 target above and a draft (an unrelated 1-layer model, seed 1,
  or a copy of the target), k = 4, greedy, 16 new tokens, eos 3: every
  prompt's tokens and target log-probabilities, and the acceptance draws
  ``torch.rand`` returned in each verify round (recorded, in order).

``--only NAME`` (a fixture file's stem) rewrites just that fixture.

The fixtures are small (about 1 MB together) and are committed; tests never run
this script.
"""

from __future__ import annotations

import json
import random
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
METRIC_KEYS = [
    "paged_kv_free_block_count", "paged_kv_used_block_count", "paged_kv_allocator_occupancy",
    "paged_kv_block_reuse_count", "paged_kv_allocator_pressure", "paged_kv_max_blocks_in_use",
    "paged_kv_resident_sequences",
]


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def allocator_traces(PagedKVAllocator) -> list[dict]:
    traces = []
    for seed in range(12):
        rng = random.Random(seed)
        total = rng.choice([4, 8, 16, 40, 64])
        bs = rng.choice([1, 2, 3, 16])
        alloc = PagedKVAllocator(total_blocks=total, block_size_tokens=bs)
        ops = []
        live: list[int] = []
        next_id = 0
        for _ in range(120):
            r = rng.random()
            if r < 0.30 or not live:
                sid = next_id if rng.random() > 0.05 or not live else rng.choice(live)
                count = rng.choice([0, 1, bs, bs + 1, rng.randint(0, 3 * bs + 2)])
                if rng.random() < 0.03:
                    count = -1
                op = ["reserve", sid, count]
                if sid == next_id:
                    next_id += 1
            elif r < 0.70:
                sid = rng.choice(live) if rng.random() > 0.05 else 10_000 + next_id
                count = rng.choice([0, 1, 1, 1, bs, rng.randint(0, 2 * bs)])
                if rng.random() < 0.03:
                    count = -2
                op = ["append_tokens", sid, count]
            elif r < 0.88:
                sid = rng.choice(live) if rng.random() > 0.05 else 20_000 + next_id
                op = ["release", sid]
            else:
                sid = rng.choice(live)
                op = ["logical_to_physical", sid, rng.randint(-1, 4)]
            try:
                res = getattr(alloc, op[0])(*op[1:])
                if op[0] in ("reserve", "append_tokens"):
                    result = {"ok": [res.sequence_id, res.token_count, res.block_size_tokens, list(res.physical_blocks)]}
                    if op[0] == "reserve":
                        live.append(op[1])
                elif op[0] == "release":
                    result = {"ok": None}
                    live.remove(op[1])
                else:
                    result = {"ok": res}
            except Exception as exc:  # noqa: BLE001 - the exception is the recorded result
                result = {"error": type(exc).__name__, "message": str(exc)}
            ops.append({"op": op, "result": result, "metrics": [alloc.metrics()[k] for k in METRIC_KEYS]})
        traces.append({"total_blocks": total, "block_size_tokens": bs, "metric_keys": METRIC_KEYS, "ops": ops})
    return traces


class _IdTokenizer:
    pad_token_id = 0
    eos_token_id = 3

    def decode(self, token_ids, skip_special_tokens: bool = True) -> str:
        del skip_special_tokens
        return " ".join(str(int(v)) for v in token_ids.tolist())


def continuous_c1_trace(ref_root: Path) -> dict:
    from agentrl.core.config import GRPOConfig
    from agentrl.generation.continuous import ContinuousBatchingOrchestrator, _ScheduledSequence
    from agentrl.generation.paged_kv import PagedKVAllocator, PagedKVCacheStore
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen2Config(
        vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, rope_theta=1e4,
        max_position_embeddings=256, tie_word_embeddings=False,
    )
    model = Qwen2ForCausalLM(cfg).eval()

    class Layout:
        def __init__(self) -> None:
            self.model = model

        def policy_forward(self, input_ids, attention_mask):
            return model(input_ids=input_ids, attention_mask=attention_mask).logits

        reference_forward = policy_forward

    config = GRPOConfig(
        model_name="fake/model", batch_size=2, group_size=4, max_new_tokens=16,
        use_paged_kv_continuous=True, do_sample=False, dtype="float32",
    )
    orch = ContinuousBatchingOrchestrator(
        config=config, environment=SimpleNamespace(), verifier=SimpleNamespace(),
        tokenizer=_IdTokenizer(), layout=Layout(), device=torch.device("cpu"),
    )
    gen = torch.Generator().manual_seed(0)
    prompts = []
    for _ in range(2):
        n = int(torch.randint(8, 33, (1,), generator=gen))
        ids = torch.randint(4, 512, (n,), generator=gen)
        prompts.extend([ids.clone() for _ in range(4)])
    seqs = [
        _ScheduledSequence(original_index=i, prompt_ids=p, prompt_mask=torch.ones_like(p))
        for i, p in enumerate(prompts)
    ]
    calls: list[list] = []
    tokens: dict[int, list[int]] = {i: [] for i in range(len(seqs))}

    def build(scheduler, sequence_lengths):
        store = PagedKVCacheStore(PagedKVAllocator(total_blocks=64, block_size_tokens=16))
        for name in ("reserve", "append_tokens", "release"):
            fn = getattr(store.allocator, name)

            def wrapped(*args, _fn=fn, _name=name):
                calls.append([_name, *[int(a) for a in args]])
                return _fn(*args)

            setattr(store.allocator, name, wrapped)
        for i, n in enumerate(sequence_lengths):
            store.reserve(i, n)
        return store

    orch._build_paged_kv_allocator = build
    orig_sample = orch._sample_next_token

    def sample(logits):
        out = orig_sample(logits)
        calls.append(["sample", [int(t) for t in out.view(-1).tolist()]])
        return out

    orch._sample_next_token = sample
    scheduler = orch._build_scheduler_state(active_count=len(seqs))
    texts, _ = orch._generate_active_batch_with_cache(seqs, scheduler)
    for i, text in enumerate(texts):
        tokens[i] = [int(t) for t in text.split()] if text else []
    stats = {k: v for k, v in orch._runtime_stats.items() if k.startswith("paged_kv_")}
    return {
        "model": {"vocab": 512, "hidden": 64, "layers": 2, "heads": 4, "kv_heads": 2, "head_dim": 16},
        "prompts": [p.tolist() for p in prompts],
        "calls": calls,
        "generated": [tokens[i] for i in range(len(seqs))],
        "paged_kv_stats": stats,
    }


def speculative_c1_trace(ref_root: Path) -> dict:
    import copy

    from agentrl.core.config import GRPOConfig
    from agentrl.generation.speculative import SpeculativeRolloutOrchestrator
    from transformers import Qwen2Config, Qwen2ForCausalLM

    def model(layers: int, seed: int):
        torch.manual_seed(seed)
        cfg = Qwen2Config(
            vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=layers,
            num_attention_heads=4, num_key_value_heads=2, head_dim=16, rope_theta=1e4,
            max_position_embeddings=256, tie_word_embeddings=False,
        )
        return Qwen2ForCausalLM(cfg).eval()

    class Tokenizer(_IdTokenizer):
        def __call__(self, text, return_tensors=None, add_special_tokens=False):
            ids = torch.tensor([[int(t) for t in text.split()]], dtype=torch.long)
            return {"input_ids": ids, "attention_mask": torch.ones_like(ids)}

    target = model(2, 0)
    gen = torch.Generator().manual_seed(2)
    prompts = [torch.randint(4, 512, (int(torch.randint(8, 33, (1,), generator=gen)),), generator=gen).tolist()
               for _ in range(3)]
    cases = {}
    for name, draft in (("unrelated_draft", model(1, 1)), ("draft_equals_target", copy.deepcopy(target))):

        class Layout:
            def policy_forward(self, input_ids, attention_mask):
                return target(input_ids=input_ids, attention_mask=attention_mask).logits

        config = GRPOConfig(
            model_name="fake/model", use_speculative_decoding=True, draft_model_name="fake/draft",
            speculative_k=4, max_new_tokens=16, do_sample=False, dtype="float32",
        )
        orch = SpeculativeRolloutOrchestrator(
            config=config, environment=SimpleNamespace(), verifier=SimpleNamespace(), tokenizer=Tokenizer(),
            layout=Layout(), device=torch.device("cpu"), rng=torch.Generator().manual_seed(7), draft_model=draft,
        )
        rounds: list[list[float]] = []
        orig_verify, orig_rand = orch._verify_draft, torch.rand

        def verify(*args, **kwargs):
            rounds.append([])
            return orig_verify(*args, **kwargs)

        def rand(*args, **kwargs):
            out = orig_rand(*args, **kwargs)
            rounds[-1].append(float(out.item()))
            return out

        orch._verify_draft = verify
        runs = []
        torch.rand = rand
        try:
            with torch.no_grad():
                for p in prompts:
                    rounds.clear()
                    toks, lps = orch._generate_speculative_tokens(" ".join(str(t) for t in p))
                    runs.append({"tokens": toks.tolist(), "logprobs": lps.tolist(), "round_draws": [list(r) for r in rounds]})
        finally:
            torch.rand = orig_rand
        cases[name] = runs
    return {
        "target": {"layers": 2, "seed": 0}, "drafts": {"unrelated_draft": {"layers": 1, "seed": 1},
                                                       "draft_equals_target": "copy of the target"},
        "model": {"vocab": 512, "hidden": 64, "intermediate": 128, "heads": 4, "kv_heads": 2, "head_dim": 16},
        "k": 4, "max_new_tokens": 16, "eos_token_id": 3, "prompts": prompts, "cases": cases,
    }


def store_roundtrips(PagedKVAllocator, PagedKVCacheStore) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(1)
    cases = [("f32_bs2", torch.float32, 2, [3, 1, 4]), ("bf16_bs16", torch.bfloat16, 16, [1, 16, 17, 40]),
             ("bf16_bs2", torch.bfloat16, 2, [5, 2])]
    for name, dtype, bs, lengths in cases:
        layers, hkv, d = 2, 2, 8
        alloc = PagedKVAllocator(total_blocks=64, block_size_tokens=bs)
        store = PagedKVCacheStore(alloc)
        for sid, n in enumerate(lengths):
            store.reserve(sid, n)
        for sid, n in enumerate(lengths):
            legacy = tuple(
                tuple(torch.randn((1, hkv, n, d), generator=g).to(dtype) for _ in range(2)) for _ in range(layers)
            )
            store.write_sequence_cache(sid, legacy, legacy)
            restored = store.read_sequence_legacy_cache(sid)
            for li in range(layers):
                for si in range(2):
                    src, dst = legacy[li][si], restored[li][si]
                    assert torch.equal(src, dst)
                    if dtype == torch.bfloat16:
                        out[f"{name}/{sid}/{li}/{si}"] = _bf16_bits(dst)
                    else:
                        out[f"{name}/{sid}/{li}/{si}"] = dst.numpy()
            out[f"{name}/{sid}/blocks"] = np.array(alloc.view(sid).physical_blocks, dtype=np.int32)
    return out


def attention_fixtures() -> dict[str, np.ndarray]:
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(2)
    hq, hkv, d = 12, 2, 128
    module = SimpleNamespace(num_key_value_groups=hq // hkv, is_causal=True)
    scale = d ** -0.5

    def rnd(*shape):
        return torch.randn(shape, generator=g).to(torch.bfloat16)

    # decode: one query over T keys (HF passes no mask for a single query)
    for i, t in enumerate([1, 16, 17, 95, 160]):
        q, k, v = rnd(1, hq, 1, d), rnd(1, hkv, t, d), rnd(1, hkv, t, d)
        o, _ = sdpa_attention_forward(module, q.float(), k.float(), v.float(), None, scaling=scale)
        out[f"decode/{i}/q"] = _bf16_bits(q[0, :, 0])
        out[f"decode/{i}/k"] = _bf16_bits(k[0].transpose(0, 1))
        out[f"decode/{i}/v"] = _bf16_bits(v[0].transpose(0, 1))
        out[f"decode/{i}/o"] = o[0, 0].numpy()  # [Hq, D] (HF returns [B, T, H, D])
    # chunked prefill: tq queries after `past` cached tokens, explicit causal mask
    for i, (past, tq) in enumerate([(0, 7), (16, 9), (33, 17), (100, 5)]):
        tk = past + tq
        q, k, v = rnd(1, hq, tq, d), rnd(1, hkv, tk, d), rnd(1, hkv, tk, d)
        mask = torch.arange(tk)[None, :] <= (past + torch.arange(tq))[:, None]
        o, _ = sdpa_attention_forward(module, q.float(), k.float(), v.float(), mask[None, None], scaling=scale)
        out[f"prefill/{i}/past"] = np.array(past)
        out[f"prefill/{i}/q"] = _bf16_bits(q[0].transpose(0, 1))
        out[f"prefill/{i}/k"] = _bf16_bits(k[0].transpose(0, 1))
        out[f"prefill/{i}/v"] = _bf16_bits(v[0].transpose(0, 1))
        out[f"prefill/{i}/o"] = o[0].numpy()
    # verify: full causal forward over prefix + k drafts, rows prefix-1 .. prefix-1+k
    for i, (prefix, kdraft) in enumerate([(1, 4), (20, 4), (70, 4), (37, 2)]):
        tk = prefix + kdraft
        q, k, v = rnd(1, hq, tk, d), rnd(1, hkv, tk, d), rnd(1, hkv, tk, d)
        o, _ = sdpa_attention_forward(module, q.float(), k.float(), v.float(), None, scaling=scale, is_causal=True)
        rows = slice(prefix - 1, prefix + kdraft)
        out[f"verify/{i}/prefix"] = np.array(prefix)
        out[f"verify/{i}/q"] = _bf16_bits(q[0, :, rows].transpose(0, 1))
        out[f"verify/{i}/k"] = _bf16_bits(k[0].transpose(0, 1))
        out[f"verify/{i}/v"] = _bf16_bits(v[0].transpose(0, 1))
        out[f"verify/{i}/o"] = o[0, rows].numpy()
    return out


def main() -> None:
    args = sys.argv[1:]
    only = None
    if "--only" in args:
        i = args.index("--only")
        only = args[i + 1]
        del args[i:i + 2]
    if not args:
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_ROOT [--only NAME]\n"
                 "REFERENCE_ROOT is a checkout of the reference project (the directory holding agentrl/)")
    ref_root = Path(args[0]).resolve()
    sys.path.insert(0, str(ref_root))
    from agentrl.generation.paged_kv import PagedKVAllocator, PagedKVCacheStore

    def want(name: str) -> bool:
        return only is None or only == name

    if want("allocator_traces"):
        (HERE / "allocator_traces.json").write_text(json.dumps(allocator_traces(PagedKVAllocator)))
    if want("continuous_c1_trace"):
        (HERE / "continuous_c1_trace.json").write_text(json.dumps(continuous_c1_trace(ref_root), indent=0))
    if want("store_roundtrip"):
        np.savez_compressed(HERE / "store_roundtrip.npz", **store_roundtrips(PagedKVAllocator, PagedKVCacheStore))
    if want("attention_sdpa"):
        np.savez_compressed(HERE / "attention_sdpa.npz", **attention_fixtures())
    if want("speculative_c1_trace"):
        (HERE / "speculative_c1_trace.json").write_text(json.dumps(speculative_c1_trace(ref_root), indent=0))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
