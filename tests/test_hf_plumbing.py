"""HF integration plumbing on CPU: PagedGenerator over a fake store equals HF's own greedy generate.

The fake store (tests/fakes.py) is test infrastructure: it keeps every sequence's K/V
per layer in plain fp32 tensors (with copy-on-write forks, releases and the
decode-step descriptor the real store returns) and attends with the oracle's
arithmetic (oracle/attention.py).  Running a tiny fp32 Qwen2 through
``PagedGenerator`` with it checks, without a GPU, everything the integration
adds around the kernels: the attention-interface layouts, packed and chunked
prefill positions, decode positions, group forks and sampling bookkeeping.
The result must equal HF ``generate`` (SDPA, DynamicCache, greedy) token for
token.  Token selection goes through the oracle's sampler (the reference's
torch ops); the device store and the device sampler run the same generator
in tests/test_gpu_hf.py.
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle.sampling import OracleSampler
from tests.fakes import FakeStore


def _tiny_model():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                      rope_theta=10000.0, attn_implementation="sdpa")
    return Qwen2ForCausalLM(cfg).eval()


def test_paged_generator_equals_hf_greedy_generate_on_cpu():
    import copy

    from randomrepo_b200.hf import PagedGenerator

    ref = _tiny_model()
    ours = copy.deepcopy(ref)
    gen = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 128, (n,), generator=gen) for n in (9, 23, 40)]
    new = 12
    want = []
    for p in prompts:
        out = ref.generate(p.unsqueeze(0), attention_mask=torch.ones(1, p.numel(), dtype=torch.long),
                           max_new_tokens=new, do_sample=False, pad_token_id=0)
        want.append(out[0, p.numel():].tolist())
    g = PagedGenerator(ours, FakeStore(2), prefill_chunk_size=16, sampler=OracleSampler())  # prompts of 23 / 40 tokens take 2-3 chunks
    res = g.generate(prompts, group_size=2, max_new_tokens=new)
    assert res["sequence_ids"] == [0, 1, 2, 3, 4, 5]
    for gi in range(3):
        for m in range(2):
            assert res["tokens"][2 * gi + m] == want[gi]
    assert ours.config._attn_implementation == "paged_b200"
    assert not g.store.count  # every sequence released


def test_teacher_forcing_and_sampling_bookkeeping():
    from randomrepo_b200.hf import PagedGenerator, SamplingConfig

    model = _tiny_model()
    g = PagedGenerator(model, FakeStore(2), prefill_chunk_size=64, eos_token_id=None, sampler=OracleSampler())
    prompts = [torch.arange(5), torch.arange(7)]
    forced = [[3, 4, 5, 6], [7, 8, 9, 10]]
    res = g.generate(prompts, max_new_tokens=4, force_tokens=forced)
    assert res["tokens"] == forced
    assert all(len(a) == 4 for a in res["argmax"])
    assert all(np.isfinite(res["logprobs"][i]).all() for i in range(2))
    s1 = g.generate(prompts, max_new_tokens=6, sampling=SamplingConfig(do_sample=True, temperature=1.0, seed=5),
                    first_id=100)
    s2 = g.generate(prompts, max_new_tokens=6, sampling=SamplingConfig(do_sample=True, temperature=1.0, seed=5),
                    first_id=200)
    assert s1["tokens"] == s2["tokens"]  # seeded sampling is reproducible


def test_eos_stops_and_releases():
    from randomrepo_b200.hf import PagedGenerator

    model = _tiny_model()
    store = FakeStore(2)
    g = PagedGenerator(model, store, eos_token_id=None, sampler=OracleSampler())
    first = g.generate([torch.arange(6)], max_new_tokens=3)["tokens"][0]
    g2 = PagedGenerator(model, store, eos_token_id=first[1], sampler=OracleSampler())
    res = g2.generate([torch.arange(6)], max_new_tokens=8, first_id=10)
    assert res["tokens"][0] == first[:2]  # stops right after emitting eos
    assert not store.count


def test_paged_attention_outside_a_generator_raises():
    from randomrepo_b200.hf import paged_attention_forward

    class M:
        layer_idx = 0

    with pytest.raises(RuntimeError):
        paged_attention_forward(M(), torch.zeros(1, 4, 1, 16), torch.zeros(1, 2, 1, 16), torch.zeros(1, 2, 1, 16))


def test_kv_geometry_follows_the_reference_rule():
    from types import SimpleNamespace

    from randomrepo_b200.hf import kv_geometry

    # agentrl/generation/scheduler.py:16-29
    assert kv_geometry(SimpleNamespace(num_hidden_layers=28, num_key_value_heads=2, num_attention_heads=12,
                                       hidden_size=1536)) == (28, 2, 128)
    assert kv_geometry(SimpleNamespace(num_hidden_layers=2, num_key_value_heads=None, num_attention_heads=4,
                                       hidden_size=64, head_dim=None)) == (2, 4, 16)
    assert kv_geometry(SimpleNamespace(num_hidden_layers=24, num_key_value_heads=2, num_attention_heads=14,
                                       hidden_size=896, head_dim=64)) == (24, 2, 64)


def _reference_compute_logprobs(model, input_ids, attention_mask, completion_mask):
    """agentrl/core/rollout.py:456-472 on an HF model (full padded forward, log_softmax, gather, mask)."""
    with torch.no_grad():
        logits = model(input_ids=input_ids, attention_mask=attention_mask).logits.float()
    token_logprobs = torch.log_softmax(logits[:, :-1, :], dim=-1)
    gathered = token_logprobs.gather(dim=-1, index=input_ids[:, 1:].unsqueeze(-1)).squeeze(-1)
    aligned = torch.zeros_like(input_ids, dtype=logits.dtype)
    aligned[:, 1:] = gathered * completion_mask[:, 1:].to(dtype=logits.dtype)
    return aligned


@pytest.mark.parametrize("group_size", [1, 2])
def test_score_equals_reference_compute_logprobs(group_size):
    from randomrepo_b200.hf import PagedGenerator

    model = _tiny_model()
    gen = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 128, (n,), generator=gen) for n in (6, 13)]
    rows, comp = [], []
    for gi, p in enumerate(prompts):
        for m in range(group_size):
            c = torch.randint(0, 128, (5 + 7 * m + 3 * gi,), generator=gen)
            rows.append(torch.cat([p, c]))
            mask = torch.cat([torch.zeros(p.numel(), dtype=torch.bool), torch.ones(c.numel(), dtype=torch.bool)])
            mask[p.numel() + 2] = False  # a masked hole inside the completion
            comp.append(mask)
    width = max(r.numel() for r in rows)
    ids = torch.zeros(len(rows), width, dtype=torch.long)
    am = torch.zeros_like(ids)
    cm = torch.zeros(len(rows), width, dtype=torch.bool)
    for i, (r, c) in enumerate(zip(rows, comp)):
        ids[i, :r.numel()] = r
        am[i, :r.numel()] = 1
        cm[i, :r.numel()] = c
    want = _reference_compute_logprobs(model, ids, am, cm)
    store = FakeStore(2)
    g = PagedGenerator(copy.deepcopy(model), store, prefill_chunk_size=8, sampler=OracleSampler())
    got = g.score(ids, am, cm, group_size=group_size, max_logit_rows=5)
    torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
    assert (got[~cm] == 0).all()
    assert not store.count  # temporary sequences released
    with pytest.raises(ValueError):
        g.score(ids, 1 - am, cm)


def test_paged_generator_reproduces_the_reference_orchestrator_c1():
    """Greedy tokens of the reference's own continuous-batching loop, pinned.

    tests/golden/continuous_c1_trace.json holds what AgentRL's
    ``ContinuousBatchingOrchestrator._generate_active_batch_with_cache``
    (agentrl/generation/continuous.py:363-504, paged-KV mode) generated on
    CPU for a random-init fp32 Qwen2 (2 layers, 4/2 heads, head_dim 16, vocab
    512, seed 0): two prompts x group 4, greedy, 16 new tokens.  The same
    model and prompts through ``PagedGenerator`` (the paged attention
    interface over the fake store, one prefill per group plus forks) must give
    the same tokens (bar: >= 99 % of positions; here every one).
    """
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from randomrepo_b200.hf import PagedGenerator
    from tests.conftest import load_json

    trace = load_json("continuous_c1_trace.json")
    m = trace["model"]
    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=m["vocab"], hidden_size=m["hidden"], intermediate_size=128,
                      num_hidden_layers=m["layers"], num_attention_heads=m["heads"],
                      num_key_value_heads=m["kv_heads"], head_dim=m["head_dim"], rope_theta=1e4,
                      max_position_embeddings=256, tie_word_embeddings=False)
    model = Qwen2ForCausalLM(cfg).eval()
    prompts = [torch.tensor(p) for p in trace["prompts"]]
    group = 4
    heads = prompts[::group]
    assert all(torch.equal(prompts[i], heads[i // group]) for i in range(len(prompts)))
    g = PagedGenerator(model, FakeStore(m["layers"]), prefill_chunk_size=512, eos_token_id=3,
                       sampler=OracleSampler())
    res = g.generate(heads, group_size=group, max_new_tokens=16)
    want = trace["generated"]
    got = res["tokens"]
    total = sum(len(w) for w in want)
    same = sum(a == b for w, t in zip(want, got) for a, b in zip(w, t))
    assert [len(t) for t in got] == [len(w) for w in want]
    assert same / total >= 0.99, (same, total)
    assert got == want


def test_packed_projection_weights_keep_the_model_unchanged():
    """The fused layers pack q / k / v and gate / up weights into one tensor each; the modules' parameters
    become views into them, so HF's own forward gives bit-identical logits, and no extra copy stays alive."""
    from randomrepo_b200.hf import _pack_weights, install_fused_layers

    model = _tiny_model()
    ids = torch.randint(0, 128, (1, 17), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        before = model(input_ids=ids).logits
        for layer in model.model.layers:
            _pack_weights(layer)
        after = model(input_ids=ids).logits
    assert torch.equal(before, after)
    for layer in model.model.layers:
        w, b, hq, hkv = layer.self_attn._pkv_qkv
        attn = layer.self_attn
        assert attn.q_proj.weight.data_ptr() == w.data_ptr()
        assert attn.k_proj.weight.data_ptr() == w[hq * 16:].data_ptr()
        assert attn.v_proj.bias.data_ptr() == b[(hq + hkv) * 16:].data_ptr()
        assert layer.mlp.up_proj.weight.data_ptr() == layer.mlp._pkv_gate_up[128:].data_ptr()
    # Re-allocated parameters (a move or cast) are packed again on next use.
    from randomrepo_b200.hf import _gate_up

    mlp = model.model.layers[0].mlp
    old = mlp._pkv_gate_up
    mlp.gate_proj.weight.data = mlp.gate_proj.weight.data.clone()
    assert _gate_up(mlp) is not old and mlp._pkv_gate_up.data_ptr() == mlp.gate_proj.weight.data_ptr()
    # A CPU / fp32 model keeps HF's forwards: the fused kernels are for bf16 / f16 on the GPU.
    assert install_fused_layers(_tiny_model()) is False


def test_packed_weights_follow_a_projection_replaced_on_its_own():
    """A weight sync or adapter merge may set ``.data`` of one projection only (v_proj, up_proj, a bias):
    the packed tensors must then be rebuilt from the current parameters, not keep the old values."""
    from randomrepo_b200.hf import _gate_up, _pack_qkv, _pack_weights, _qkv_packed

    model = _tiny_model()
    layer = model.model.layers[0]
    with torch.no_grad():
        _pack_weights(layer)
    attn, mlp = layer.self_attn, layer.mlp
    assert _qkv_packed(attn)
    gen = torch.Generator().manual_seed(9)
    for name in ("v_proj", "k_proj"):
        proj = getattr(attn, name)
        proj.weight.data = torch.randn(proj.weight.shape, generator=gen)
        assert not _qkv_packed(attn)
        with torch.no_grad():
            _pack_qkv(attn)
        assert _qkv_packed(attn)
        w, b, _, _ = attn._pkv_qkv
        assert torch.equal(w, torch.cat([attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight], 0))
    attn.q_proj.bias.data = torch.randn(attn.q_proj.bias.shape, generator=gen)
    assert not _qkv_packed(attn)
    with torch.no_grad():
        _pack_qkv(attn)
    assert torch.equal(attn._pkv_qkv[1], torch.cat([attn.q_proj.bias, attn.k_proj.bias, attn.v_proj.bias], 0))
    new_up = torch.randn(mlp.up_proj.weight.shape, generator=gen)
    mlp.up_proj.weight.data = new_up
    gu = _gate_up(mlp)
    assert torch.equal(gu[mlp.gate_proj.weight.shape[0]:], new_up)
    assert _gate_up(mlp) is gu  # packed again once, then reused


def test_rollout_under_kv_pressure_defers_evicts_and_keeps_the_tokens():
    """A pool far too small for the batch: growth admission defers sequences whose next token needs a
    block (continuous.py:900-937; soft preemptions counted as continuous.py:875-898 counts them), and
    when no sequence can grow at all one is evicted and re-prefilled later.  Teacher-forced on the tokens
    of an unpressured run, every position's greedy choice and log-probability equal that run's."""
    from oracle.sampling import OracleSampler
    from randomrepo_b200.hf import PagedGenerator

    model = _tiny_model()
    gen = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, 128, (int(n),), generator=gen) for n in (20, 9, 33)]
    new = 40
    free_run = PagedGenerator(model, FakeStore(2), prefill_chunk_size=64, sampler=OracleSampler())
    want = free_run.generate(prompts, group_size=3, max_new_tokens=new)
    assert want["kv_pressure"]["paged_kv_preempted_sequences"] == 0 and want["steps"] == new
    # 9 sequences of up to 73 tokens need ~40 blocks of 16 with the prompts shared; give them 14.
    store = FakeStore(2, total_blocks=14)
    tight = PagedGenerator(model, store, prefill_chunk_size=64, sampler=OracleSampler())
    got = tight.generate(prompts, group_size=3, max_new_tokens=new, force_tokens=want["tokens"])
    kv = got["kv_pressure"]
    assert kv["paged_kv_preempted_sequences"] > 0 and kv["paged_kv_max_preempted_sequences"] >= 1
    assert kv["paged_kv_evicted_sequences"] > 0 and kv["paged_kv_recomputed_tokens"] > 0
    assert kv["scheduler_decode_growth_blocks_admitted"] <= kv["scheduler_decode_growth_block_demand"]
    assert got["steps"] > new
    assert got["tokens"] == want["tokens"]
    assert got["argmax"] == want["argmax"]
    for a, b in zip(got["logprobs"], want["logprobs"]):
        np.testing.assert_allclose(a, b, atol=1e-4)
    assert store.refs == {}  # every block returned


def test_paged_cache_is_a_transformers_cache_class():
    """``PagedCache`` (defined on first use) is a ``transformers`` ``Cache`` subclass, so HF's loops
    and ``isinstance`` checks accept it; its behaviour runs on the GPU (tests/test_gpu_hf.py)."""
    from transformers.cache_utils import Cache

    import randomrepo_b200.hf as hf
    from randomrepo_b200.hf import PagedCache

    assert isinstance(PagedCache, type) and issubclass(PagedCache, Cache)
    assert hf.PagedCache is PagedCache and PagedCache.__qualname__ == "PagedCache"
