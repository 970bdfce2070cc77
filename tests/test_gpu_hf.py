"""Greedy-token parity of the paged path inside a real model, on the GPU.

A random-init bf16 Qwen2 (seeded) decodes greedily twice: through HF's own
path -- SDPA attention with a DynamicCache, which is what AgentRL's
continuous loop runs (agentrl/generation/continuous.py:363-504) -- and through
``PagedGenerator`` on the device KV pool (packed / chunked prefill kernel,
fused append + paged decode kernel, copy-on-write group forks).

Both paths take logits in fp32 from the model's bf16 final hidden state (a
bf16 LM head leaves exact ties in the argmax of random-init logits).

Positions are compared teacher-forced: our model is fed HF's tokens and its
argmax at every step is compared with HF's token, so one early near-tie does
not cascade into the rest of a sequence.  What a bf16 model can promise is
bounded by bf16 itself: HF's own two attention backends (eager and SDPA) on
the same weights disagree on up to a few % of these positions, always at
near-ties.  The north star's ">= 99 % of greedy positions" is asserted on the
positions bf16 can decide: those whose HF top-2 logit gap exceeds the largest
gap at which HF's eager and SDPA backends disagree on the same positions
("decidable").  The bars, per configuration:
* at least 99 % agreement with HF-SDPA on the decidable positions;
* every position that differs is a near-tie (HF top-2 gap below 0.02, or
  below HF's own disagreement gap where that is larger);
* overall agreement of at least 99 % or of HF's own eager-vs-SDPA agreement
  minus 0.01, whichever is lower (measured 97.9-99.6 % overall at these
  random-init bf16 models, against 96.5-99.2 % for HF's two backends: the
  undecidable near-ties make up the rest);
* free-running agreement (each path feeds its own tokens) of at least 50 %:
  after a near-tie flips one token the two continuations differ, so this only
  guards against gross errors -- a wrong page, position or fork gives
  near-random tokens (~0.2 % at vocabulary 512).
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(device, head_dim: int, layers: int = 2, hq: int = 4, hkv: int = 2, vocab: int = 512):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=hq * head_dim, intermediate_size=2 * hq * head_dim,
                      num_hidden_layers=layers, num_attention_heads=hq, num_key_value_heads=hkv,
                      max_position_embeddings=4096, rope_theta=10000.0, attn_implementation="sdpa")
    return Qwen2ForCausalLM(cfg).to(device=device, dtype=torch.bfloat16).eval()


def _hf_greedy(model, prompts, new: int):
    """HF's path: forward with a DynamicCache per sequence, fp32 logits from the final hidden state.

    Returns the greedy tokens and, per step, the gap between HF's two largest logits.
    """
    from transformers import DynamicCache

    w = model.get_output_embeddings().weight.detach().float()
    toks, gaps = [], []
    with torch.inference_mode():
        for p in prompts:
            cache = DynamicCache()
            h = model.model(input_ids=p.unsqueeze(0).to(model.device), past_key_values=cache,
                            use_cache=True).last_hidden_state[:, -1]
            seq, gap = [], []
            for _ in range(new):
                logits = torch.nn.functional.linear(h.float(), w)[0]
                top2 = logits.topk(2).values
                gap.append(float(top2[0] - top2[1]))
                t = int(torch.argmax(logits))
                seq.append(t)
                h = model.model(input_ids=torch.tensor([[t]], device=model.device), past_key_values=cache,
                                use_cache=True).last_hidden_state[:, -1]
            toks.append(seq)
            gaps.append(gap)
    return toks, gaps


def _teacher_forced_argmax(model, prompts, tokens, new: int):
    """Argmax of fp32 logits of ``model`` (HF forward over prompt + tokens) at each generated position."""
    w = model.get_output_embeddings().weight.detach().float()
    out = []
    with torch.inference_mode():
        for p, ts in zip(prompts, tokens):
            full = torch.cat([p, torch.tensor(ts)]).to(model.device).unsqueeze(0)
            h = model.model(input_ids=full).last_hidden_state[0, p.numel() - 1:p.numel() - 1 + new]
            out.append(torch.nn.functional.linear(h.float(), w).argmax(-1).tolist())
    return out


def _agreement(a, b) -> float:
    return float(np.mean([x == y for u, v in zip(a, b) for x, y in zip(u, v)]))


def _parity(pairs, want, gaps, eager_am):
    """Agreement overall and on decidable positions, the HF noise gap and the mismatch gaps."""
    agree = float(np.mean([ok for ok, _ in pairs]))
    noise = [gp for ea, ws, gs in zip(eager_am, want, gaps) for e, w, gp in zip(ea, ws, gs) if e != w]
    noise_gap = max(noise, default=0.0)
    clear = [ok for ok, gp in pairs if gp > noise_gap]
    return agree, float(np.mean(clear)), noise_gap, [gp for ok, gp in pairs if not ok]


# 2-layer models at the head geometry of each configuration (CPU smoke 4/2 D64, Qwen2.5-1.5B 12/2 D128,
# Qwen2.5-0.5B draft 14/2 D64, Qwen2.5-7B 28/4 D128) and a 3-layer 1.5B-geometry model.
@pytest.mark.parametrize("head_dim,hq,hkv,layers", [(64, 4, 2, 2), (128, 12, 2, 2), (64, 14, 2, 2), (128, 28, 4, 2),
                                                    (128, 12, 2, 3)])
def test_greedy_tokens_match_hf_sdpa(cuda_device, head_dim, hq, hkv, layers):
    from randomrepo_b200.hf import PagedGenerator, make_store

    ref = _model(cuda_device, head_dim, layers, hq, hkv)
    ours = copy.deepcopy(ref)
    eager = copy.deepcopy(ref)
    for mod in eager.modules():
        if hasattr(mod, "config"):
            mod.config._attn_implementation = "eager"
    gen = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 512, (int(n),), generator=gen) for n in torch.randint(8, 41, (16,), generator=gen)]
    new = 32
    want, gaps = _hf_greedy(ref, prompts, new)
    store = make_store(ours, total_blocks=2048)
    g = PagedGenerator(ours, store, prefill_chunk_size=16)
    forced = g.generate(prompts, max_new_tokens=new, force_tokens=want)
    pairs = [(a == w, gp) for am, ws, gs in zip(forced["argmax"], want, gaps) for a, w, gp in zip(am, ws, gs)]
    eager_am = _teacher_forced_argmax(eager, prompts, want, new)
    floor = _agreement(eager_am, _teacher_forced_argmax(ref, prompts, want, new))
    agree, clear, noise_gap, miss = _parity(pairs, want, gaps, eager_am)
    detail = f"agreement {agree:.4f}, decidable {clear:.4f}, HF eager vs SDPA {floor:.4f} (noise gap {noise_gap:.4f})"
    assert clear >= 0.99, detail
    assert all(gp < max(0.02, noise_gap) for gp in miss), (detail, sorted(miss))
    assert agree >= min(0.99, floor - 0.01), detail
    free = g.generate(prompts, max_new_tokens=new, first_id=1000)
    free_agree = _agreement(free["tokens"], want)
    assert free_agree >= 0.5, f"free-running agreement {free_agree:.4f}"
    assert store.pool.decode_error_flag() == 0 and store.pool.prefill_error_flag() == 0
    assert store.allocator.used_block_count == 0  # every sequence released


def test_group_fork_rollout_members_share_prompt(cuda_device):
    """GRPO groups: one prefill per prompt, members forked copy-on-write; greedy members agree."""
    from randomrepo_b200.hf import PagedGenerator, make_store

    model = _model(cuda_device, 64)
    gen = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 512, (n,), generator=gen) for n in (20, 37)]
    store = make_store(model, total_blocks=512)
    g = PagedGenerator(model, store, prefill_chunk_size=512)
    solo = g.generate(prompts, group_size=1, max_new_tokens=24)
    grp = g.generate(prompts, group_size=4, max_new_tokens=24, first_id=100)
    for gi in range(2):
        for m in range(4):
            assert grp["tokens"][4 * gi + m] == solo["tokens"][gi]
    assert store.allocator.used_block_count == 0


def test_cuda_graph_decode_matches_eager(cuda_device):
    """Decode steps replayed from CUDA graphs (fixed-step mode) give the eager path's tokens and logprobs."""
    from randomrepo_b200.hf import PagedGenerator, make_store

    model = _model(cuda_device, 128, 2, 12, 2)
    gen = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 512, (n,), generator=gen) for n in (30, 77, 12)]
    eager = PagedGenerator(model, make_store(model, total_blocks=1024), prefill_chunk_size=64)
    graphs = PagedGenerator(model, make_store(model, total_blocks=1024), prefill_chunk_size=64, cuda_graphs=True)
    for group in (1, 2):  # two batch sizes: a graph each
        a = eager.generate(prompts, group_size=group, max_new_tokens=40)
        b = graphs.generate(prompts, group_size=group, max_new_tokens=40)
        assert a["tokens"] == b["tokens"]
        np.testing.assert_allclose(np.concatenate(b["logprobs"]), np.concatenate(a["logprobs"]), atol=1e-4)
    # Batches 3 and 6 run padded to the recorded sizes 4 and 8; batch 8 outgrew the
    # fixed-step capacity set for 4, so capacity grew and the graphs were re-recorded.
    assert set(graphs._graphs) == {8}
    pool = graphs.store.pool
    assert pool.decode_error_flag() == 0 and graphs.store.allocator.used_block_count == 0


def test_cuda_graphs_shrinking_batch_reuses_padded_graphs(cuda_device):
    """Sequences that stop at eos shrink the batch step by step: the graphed path pads each step to a
    recorded size (placeholder sequences) instead of recording a graph per size, with the eager tokens."""
    from randomrepo_b200.hf import PagedGenerator, graph_batch, make_store

    model = _model(cuda_device, 64, 2)
    gen = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 512, (int(n),), generator=gen) for n in torch.randint(5, 60, (12,), generator=gen)]
    probe = PagedGenerator(model, make_store(model, total_blocks=2048), prefill_chunk_size=64)
    free = probe.generate(prompts, group_size=2, max_new_tokens=48)["tokens"]
    # As eos the token found in the most sequences: several stop early, at different steps.
    eos = int(np.bincount(np.concatenate([np.unique(t) for t in free])).argmax())
    eager = PagedGenerator(model, make_store(model, total_blocks=2048), prefill_chunk_size=64, eos_token_id=eos)
    graphs = PagedGenerator(model, make_store(model, total_blocks=2048), prefill_chunk_size=64, eos_token_id=eos,
                            cuda_graphs=True)
    a = eager.generate(prompts, group_size=2, max_new_tokens=48)
    b = graphs.generate(prompts, group_size=2, max_new_tokens=48)
    assert a["tokens"] == b["tokens"]
    # Sequences still decoding at each step after the first (the first comes from prefill).
    active = {sum(len(t) > s for t in a["tokens"]) for s in range(1, 48)} - {0}
    buckets = {graph_batch(c) for c in active}
    assert len(active) >= 3 and len(buckets) < len(active)  # the batch shrank, sizes shared a graph
    assert set(graphs._graphs) == buckets
    assert graphs.store.allocator.used_block_count == 0 and graphs.store.resident_sequence_count == 0


def test_score_matches_the_reference_old_policy_pass(cuda_device):
    """PagedGenerator.score vs agentrl/core/rollout.py:456-472 run on HF (SDPA, padded batch, fp32 head).

    The rows are a sampled GRPO rollout of 3 prompts x 4 members, so the
    groups share their prompt pages; bf16 attention in the two
    implementations bounds the agreement (same scale as the greedy near-ties).
    The rollout's own recorded log-probabilities are the same quantity and
    must agree as well.
    """
    from randomrepo_b200.hf import PagedGenerator, SamplingConfig, make_store

    model = _model(cuda_device, 64, 2)
    store = make_store(model, total_blocks=1024)
    g = PagedGenerator(copy.deepcopy(model), store, prefill_chunk_size=16)
    gen = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 512, (int(n),), generator=gen) for n in (9, 21, 34)]
    roll = g.generate(prompts, group_size=4, max_new_tokens=24,
                      sampling=SamplingConfig(do_sample=True, temperature=1.0, seed=3))
    rows = [torch.cat([prompts[i // 4], torch.tensor(t)]) for i, t in enumerate(roll["tokens"])]
    width = max(r.numel() for r in rows)
    ids = torch.zeros(len(rows), width, dtype=torch.long)
    am = torch.zeros_like(ids)
    cm = torch.zeros(len(rows), width, dtype=torch.bool)
    for i, r in enumerate(rows):
        ids[i, :r.numel()] = r
        am[i, :r.numel()] = 1
        cm[i, prompts[i // 4].numel():r.numel()] = True
    got = g.score(ids, am, cm, group_size=4, max_logit_rows=37).cpu()
    w = model.get_output_embeddings().weight.detach().float()
    with torch.inference_mode():
        h = model.model(input_ids=ids.to(cuda_device), attention_mask=am.to(cuda_device)).last_hidden_state
        logits = torch.nn.functional.linear(h.float(), w)
    want = torch.zeros_like(got)
    want[:, 1:] = (torch.log_softmax(logits[:, :-1], -1).gather(-1, ids[:, 1:].to(cuda_device).unsqueeze(-1))
                   .squeeze(-1).cpu() * cm[:, 1:])
    diff = (got - want)[cm].abs()
    assert float(diff.max()) < 0.1 and float(diff.mean()) < 0.02, (float(diff.max()), float(diff.mean()))
    assert (got[~cm] == 0).all()
    rolled = torch.tensor([lp for seq in roll["logprobs"] for lp in seq])
    scored = torch.cat([got[i, prompts[i // 4].numel():rows[i].numel()] for i in range(len(rows))])
    d2 = (rolled - scored).abs()
    assert float(d2.max()) < 0.1 and float(d2.mean()) < 0.02, (float(d2.max()), float(d2.mean()))
    assert store.allocator.used_block_count == 0


def test_greedy_tokens_at_the_qwen2p5_1p5b_architecture(cuda_device):
    """The same teacher-forced check at the full Qwen2.5-1.5B architecture (28 layers, 12/2 heads,
    head_dim 128, vocab 151 936, random-init bf16; prompts of 64-256 tokens in one 512-token prefill
    chunk).  Random-init logits this deep are flat (median top-2 gap ~0.13), so bf16 near-ties are
    frequent.  Bars: >= 99 % agreement on the decidable positions (HF top-2 gap above the largest gap
    at which HF's own eager and SDPA backends disagree), every mismatch a near-tie (gap below
    max(0.05, twice that gap)), and overall agreement at least HF's eager-vs-SDPA agreement minus 0.01."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from randomrepo_b200.hf import PagedGenerator, make_store

    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=28,
                      num_attention_heads=12, num_key_value_heads=2, max_position_embeddings=32768,
                      rope_theta=1e6, tie_word_embeddings=True, attn_implementation="sdpa")
    with torch.device(cuda_device):
        ref = Qwen2ForCausalLM(cfg).to(torch.bfloat16).eval()
    ours = copy.deepcopy(ref)
    eager = copy.deepcopy(ref)
    for mod in eager.modules():
        if hasattr(mod, "config"):
            mod.config._attn_implementation = "eager"
    gen = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 151936, (int(n),), generator=gen) for n in torch.randint(64, 257, (8,), generator=gen)]
    new = 32
    want, gaps = _hf_greedy(ref, prompts, new)
    store = make_store(ours, total_blocks=4096)
    g = PagedGenerator(ours, store, prefill_chunk_size=512)
    forced = g.generate(prompts, max_new_tokens=new, force_tokens=want)
    pairs = [(a == w, gp) for am, ws, gs in zip(forced["argmax"], want, gaps) for a, w, gp in zip(am, ws, gs)]
    eager_am = _teacher_forced_argmax(eager, prompts, want, new)
    floor = _agreement(eager_am, _teacher_forced_argmax(ref, prompts, want, new))
    agree, clear, noise_gap, miss = _parity(pairs, want, gaps, eager_am)
    detail = f"agreement {agree:.4f}, decidable {clear:.4f}, HF eager vs SDPA {floor:.4f} (noise gap {noise_gap:.4f})"
    assert clear >= 0.99, detail
    assert all(gp < max(0.05, 2 * noise_gap) for gp in miss), (detail, sorted(miss)[-5:])
    assert agree >= floor - 0.01, detail
    assert store.pool.decode_error_flag() == 0 and store.pool.prefill_error_flag() == 0
    assert store.allocator.used_block_count == 0


def test_fused_layers_match_hf_modules(cuda_device):
    """Fused norm / rotary / SiLU launches (installed by PagedGenerator) against the same generator running HF's
    own module code: teacher-forced on the same tokens, greedy selections agree on >= 99 % of positions (every
    disagreement a near-tie under 0.02) and the chosen tokens' log-probabilities within 0.05."""
    from randomrepo_b200.hf import PagedGenerator, make_store

    base = _model(cuda_device, 128, 3, 12, 2)
    fused_m, plain_m = copy.deepcopy(base), copy.deepcopy(base)
    gen = torch.Generator().manual_seed(19)
    prompts = [torch.randint(0, 512, (int(n),), generator=gen) for n in torch.randint(8, 60, (6,), generator=gen)]
    new = 24
    want, gaps = _hf_greedy(base, prompts, new)
    fused = PagedGenerator(fused_m, make_store(fused_m, total_blocks=1024), prefill_chunk_size=32)
    plain = PagedGenerator(plain_m, make_store(plain_m, total_blocks=1024), prefill_chunk_size=32,
                           fused_layers=False)
    assert fused.fused_layers and not plain.fused_layers
    a = fused.generate(prompts, max_new_tokens=new, force_tokens=want)
    b = plain.generate(prompts, max_new_tokens=new, force_tokens=want)
    pairs = [(x == y, gp) for u, v, gs in zip(a["argmax"], b["argmax"], gaps) for x, y, gp in zip(u, v, gs)]
    assert float(np.mean([ok for ok, _ in pairs])) >= 0.99
    assert all(gp < 0.02 for ok, gp in pairs if not ok)
    np.testing.assert_allclose(np.concatenate(a["logprobs"]), np.concatenate(b["logprobs"]), atol=0.05)
    # Outside a generator forward the model runs HF's own code again (here with SDPA attention).
    for m in (fused_m, plain_m):
        for mod in m.modules():
            if hasattr(mod, "config"):
                mod.config._attn_implementation = "sdpa"
    with torch.inference_mode():
        ids = prompts[0].unsqueeze(0).to(cuda_device)
        assert torch.equal(fused_m(input_ids=ids).logits, plain_m(input_ids=ids).logits)


@pytest.mark.parametrize("cuda_graphs", [False, True])
def test_rollout_under_kv_pressure_matches_the_unpressured_run(cuda_device, cuda_graphs):
    """GRPO groups in a pool far too small for them: sequences are deferred (soft preemption) and evicted
    and re-prefilled, as the admission needs.  Teacher-forced on the unpressured run's tokens, greedy
    choices agree on >= 99 % of positions (every disagreement a near-tie: the batch composition changes the
    split-K plan and GEMM shapes, hence bf16 rounding) and log-probabilities within 0.05."""
    from randomrepo_b200.hf import PagedGenerator, make_store

    model = _model(cuda_device, 64, 2)
    gen = torch.Generator().manual_seed(31)
    prompts = [torch.randint(0, 512, (n,), generator=gen) for n in (20, 37, 9)]
    new = 48
    free_gen = PagedGenerator(model, make_store(model, total_blocks=1024), prefill_chunk_size=64,
                              cuda_graphs=cuda_graphs)
    want = free_gen.generate(prompts, group_size=4, max_new_tokens=new)
    assert want["kv_pressure"]["paged_kv_preempted_sequences"] == 0
    store = make_store(model, total_blocks=20)
    tight = PagedGenerator(model, store, prefill_chunk_size=64, cuda_graphs=cuda_graphs)
    got = tight.generate(prompts, group_size=4, max_new_tokens=new, force_tokens=want["tokens"])
    kv = got["kv_pressure"]
    assert kv["paged_kv_preempted_sequences"] > 0 and kv["paged_kv_evicted_sequences"] > 0
    assert got["tokens"] == want["tokens"]
    pairs = [(a == b, lp) for u, v, lps in zip(got["argmax"], want["argmax"], want["logprobs"])
             for a, b, lp in zip(u, v, lps)]
    assert float(np.mean([ok for ok, _ in pairs])) >= 0.99
    np.testing.assert_allclose(np.concatenate(got["logprobs"]), np.concatenate(want["logprobs"]), atol=0.05)
    assert store.pool.decode_error_flag() == 0 and store.pool.prefill_error_flag() == 0
    assert store.allocator.used_block_count == 0


def test_hf_generate_with_a_paged_cache_equals_a_dynamic_cache(cuda_device):
    """HF's own ``generate`` (unchanged model code, SDPA attention) with its K/V in the store's pages
    through ``PagedCache`` gives the same greedy tokens as with HF's ``DynamicCache``, and the pages then
    hold bit for bit the K/V the DynamicCache holds."""
    from randomrepo_b200.hf import PagedCache, make_store

    model = _model(cuda_device, 64, 2)
    gen = torch.Generator().manual_seed(41)
    ids = torch.randint(0, 512, (3, 21), generator=gen).to(cuda_device)
    mask = torch.ones_like(ids)
    with torch.inference_mode():
        want = model.generate(ids, attention_mask=mask, max_new_tokens=24, do_sample=False, pad_token_id=0,
                              return_dict_in_generate=True)
        store = make_store(model, total_blocks=256)
        sids = [100, 101, 102]
        for s in sids:
            store.reserve(s, 0)
        cache = PagedCache(store, sids, num_layers=model.config.num_hidden_layers)
        got = model.generate(ids, attention_mask=mask, past_key_values=cache, max_new_tokens=24, do_sample=False,
                             pad_token_id=0, return_dict_in_generate=True)
    assert torch.equal(got.sequences, want.sequences)
    dyn = want.past_key_values
    n = cache.get_seq_length()
    assert n == dyn.get_seq_length() == ids.shape[1] + 24 - 1
    for b, s in enumerate(sids):
        pages = store.read_sequence_legacy_cache(s)
        for layer in range(model.config.num_hidden_layers):
            assert torch.equal(pages[layer][0][0], dyn.layers[layer].keys[b])
            assert torch.equal(pages[layer][1][0], dyn.layers[layer].values[b])


def test_paged_cache_with_the_paged_kernels_matches_a_dynamic_cache(cuda_device):
    """The same model switched to the ``paged_b200`` attention, its HF forwards over a
    ``PagedCache(kernels=True)``: a batched prefill forward and then decode forwards run on the store's
    kernels (chunked-prefill kernel, fused append + paged decode) and give the logits of the same
    forwards over a ``DynamicCache`` with SDPA within bf16 (greedy choices equal where not near-ties),
    and HF ``generate`` runs on them end to end."""
    from transformers import DynamicCache

    from randomrepo_b200.hf import PagedCache, make_store, use_paged_attention

    ref = _model(cuda_device, 128, 2, 12, 2)
    ours = copy.deepcopy(ref)
    use_paged_attention(ours)
    gen = torch.Generator().manual_seed(43)
    ids = torch.randint(0, 512, (4, 37), generator=gen).to(cuda_device)
    store = make_store(ours, total_blocks=256)
    sids = [7, 8, 9, 10]
    for s in sids:
        store.reserve(s, 0)
    cache = PagedCache(store, sids, num_layers=2, kernels=True)
    dyn = DynamicCache(config=ref.config)
    agree, total = 0, 0
    with torch.inference_mode():
        x = ids
        for _ in range(6):
            a = ref(input_ids=x, past_key_values=dyn, use_cache=True).logits[:, -1].float()
            b = ours(input_ids=x, past_key_values=cache, use_cache=True).logits[:, -1].float()
            np.testing.assert_allclose(b.cpu().numpy(), a.cpu().numpy(), atol=0.05, rtol=0.02)
            top2 = a.topk(2, dim=-1).values
            decidable = (top2[:, 0] - top2[:, 1]) > 0.02
            agree += int(((a.argmax(-1) == b.argmax(-1)) | ~decidable).sum())
            total += a.shape[0]
            x = a.argmax(-1, keepdim=True)
    assert agree == total
    assert cache.get_seq_length() == dyn.get_seq_length() == 37 + 5
    assert store.pool.decode_error_flag() == 0 and store.pool.prefill_error_flag() == 0
    # HF generate end to end on the kernels (free-running, so after a bf16 near-tie the continuations may
    # differ: the per-forward logits above are the numerical check; here the run, its first choices and
    # its cache length).
    store2 = make_store(ours, total_blocks=256)
    for s in sids:
        store2.reserve(s, 0)
    cache2 = PagedCache(store2, sids, 2, kernels=True)
    with torch.inference_mode():
        out = ours.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=16, do_sample=False,
                            pad_token_id=0, past_key_values=cache2)
        want = ref.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=16, do_sample=False,
                            pad_token_id=0)
    assert out.shape == want.shape and torch.equal(out[:, :38], want[:, :38])
    assert cache2.get_seq_length() == 37 + 15
    assert store2.pool.decode_error_flag() == 0 and store2.pool.prefill_error_flag() == 0
