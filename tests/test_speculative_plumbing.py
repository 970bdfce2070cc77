"""Paged speculative decoding on CPU: the batched loop equals the reference's one-sequence loop.

``PagedSpeculativeGenerator`` runs here over two fake stores (tests/fakes.py)
with the oracle's sampler, i.e. with the reference's own torch arithmetic for
every decision, so the comparison below checks the loop's bookkeeping: which
tokens each model's cache holds after every round (pending tokens, truncation
of rejected drafts, the bonus token), group forks, eos and max_new_tokens
handling.  The reference side is ``oracle.speculative.generate``: the
algorithm of agentrl/generation/speculative.py:148-274 with full-prefix
forwards of the same HF models.  Both consume the same acceptance draws.
The device kernels run the same loop in tests/test_gpu_speculative.py.
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle import speculative as ospec
from oracle.sampling import OracleSampler
from tests.fakes import FakeStore


def _model(seed: int, layers: int = 2, vocab: int = 96):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=64, intermediate_size=128, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                      rope_theta=10000.0, attn_implementation="sdpa")
    return Qwen2ForCausalLM(cfg).eval()


def _full_logits(model):
    def fn(ids):
        with torch.no_grad():
            return model(input_ids=torch.tensor([ids]), use_cache=False).logits[0].float()
    return fn


def _last_logits(model):
    full = _full_logits(model)
    return lambda ids: full(ids)[-1]


U_TABLE = torch.rand((64, 64, 8), generator=torch.Generator().manual_seed(7))


def _uniform(seq: int, rnd: int):
    return U_TABLE[seq, rnd].tolist()


def _spec(target, draft, k, eos=None, chunk=16):
    from randomrepo_b200.hf import PagedGenerator
    from randomrepo_b200.speculative import PagedSpeculativeGenerator

    sampler = OracleSampler()
    t = PagedGenerator(target, FakeStore(target.config.num_hidden_layers), prefill_chunk_size=chunk,
                       sampler=sampler)
    d = PagedGenerator(draft, FakeStore(draft.config.num_hidden_layers), prefill_chunk_size=chunk,
                       sampler=sampler)
    return PagedSpeculativeGenerator(t, d, k=k, eos_token_id=eos)


def _reference(target, draft, prompt, k, new, eos, seq):
    return ospec.generate(prompt, _full_logits(target), _last_logits(draft), k=k, max_new_tokens=new,
                          eos_token_id=eos, uniform_fn=lambda r, i: _uniform(seq, r)[i])


@pytest.mark.parametrize("k", [1, 3, 4])
def test_batched_paged_loop_equals_reference_loop(k):
    target, draft = _model(0), _model(1, layers=1)
    gen = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 96, (n,), generator=gen) for n in (1, 7, 20, 33)]
    new = 13
    sg = _spec(copy.deepcopy(target), copy.deepcopy(draft), k)
    res = sg.generate(prompts, max_new_tokens=new, uniforms=_uniform, trace=True)
    assert res["rounds"] > 1
    assert 0 < res["accepted"] <= res["proposed"]
    for i, p in enumerate(prompts):
        want, want_lp, rounds = _reference(target, draft, p.tolist(), k, new, None, i)
        assert res["tokens"][i] == want
        np.testing.assert_allclose(res["logprobs"][i], want_lp, rtol=1e-4, atol=1e-4)
        got_rounds = [(pl, dr[:nd], na) for pl, dr, nd, na, _ in res["trace"][i]]
        assert got_rounds == [(pl, dr, na) for pl, dr, na, _ in rounds]
    assert not sg.target.store.count and not sg.draft.store.count


def test_rejections_bonuses_and_truncation_all_happen():
    target, draft = _model(0), _model(1, layers=1)
    sg = _spec(copy.deepcopy(target), copy.deepcopy(draft), 3)
    prompts = [torch.arange(5), torch.arange(9) * 3 % 96]
    res = sg.generate(prompts, max_new_tokens=24, uniforms=_uniform, trace=True)
    rounds = [r for tr in res["trace"] for r in tr]
    assert any(na < nd for _, _, nd, na, _ in rounds)               # a rejection -> correction
    assert any(na == nd and len(em) == nd + 1 for _, _, nd, na, em in rounds)  # all accepted -> bonus


def test_groups_fork_and_eos_stops():
    target, draft = _model(0), _model(1, layers=1)
    prompt = torch.arange(11) * 5 % 96
    # Pick as eos a token the reference emits mid-way, so the eos path runs.
    free, _, _ = _reference(target, draft, prompt.tolist(), 3, 16, None, 0)
    eos = free[6]
    want, want_lp, _ = _reference(target, draft, prompt.tolist(), 3, 16, eos, 0)
    assert want[-1] == eos and len(want) <= 7
    sg = _spec(copy.deepcopy(target), copy.deepcopy(draft), 3, eos=eos)
    res = sg.generate([prompt], group_size=3, max_new_tokens=16, uniforms=lambda s, r: _uniform(0, r))
    assert res["sequence_ids"] == [0, 1, 2]
    for m in range(3):  # same draws for every member -> the same completion
        assert res["tokens"][m] == want
    assert not sg.target.store.count and not sg.draft.store.count


def test_max_new_tokens_smaller_than_k():
    target, draft = _model(0), _model(1, layers=1)
    sg = _spec(copy.deepcopy(target), copy.deepcopy(draft), 4)
    res = sg.generate([torch.arange(6)], max_new_tokens=2, uniforms=_uniform)
    want, _, _ = _reference(target, draft, list(range(6)), 4, 2, None, 0)
    assert res["tokens"][0] == want and len(want) == 2


def test_sampled_rounds_are_reproducible_and_in_vocab():
    from randomrepo_b200.hf import SamplingConfig

    target, draft = _model(0), _model(1, layers=1)
    sg = _spec(target, draft, 3)
    cfg = SamplingConfig(do_sample=True, temperature=0.8, seed=11)
    a = sg.generate([torch.arange(6), torch.arange(4)], max_new_tokens=10, sampling=cfg)
    b = sg.generate([torch.arange(6), torch.arange(4)], max_new_tokens=10, sampling=cfg, first_id=50)
    assert a["tokens"] == b["tokens"]
    assert all(0 <= t < 96 for seq in a["tokens"] for t in seq)
    assert all(np.isfinite(seq).all() and max(seq) <= 0 for seq in a["logprobs"])


def test_oracle_verify_draft_known_answers():
    # Vocabulary of 4; target rows for positions prefix-1 .. prefix-1+2.
    t = torch.log(torch.tensor([[0.1, 0.6, 0.2, 0.1], [0.5, 0.1, 0.3, 0.1], [0.25, 0.25, 0.4, 0.1]]))
    q0 = torch.tensor([0.1, 0.3, 0.5, 0.1])
    q1 = torch.tensor([0.1, 0.8, 0.05, 0.05])
    dl = [float(torch.log(q0[1])), float(torch.log(q1[1]))]
    # u = 0: every draft accepted, then the bonus is the argmax of the last row.
    r = ospec.verify_draft(t, [1, 1], dl, [q0, q1], [0.0, 0.0])
    assert [s[0] for s in r.steps] == [1, 1, 2] and r.n_accepted == 2
    # Draft 0 (p_t 0.6 >= q 0.3) accepted for any u; draft 1 (0.1 vs 0.8) rejected at u = 0.5:
    # correction = argmax of max(p - q, 0) = [0.4, 0, 0.25, 0.05] -> token 0.
    r = ospec.verify_draft(t, [1, 1], dl, [q0, q1], [0.99, 0.5])
    assert [s[0] for s in r.steps] == [1, 0] and r.n_accepted == 1
    assert abs(r.steps[1][1] - float(t[1].log_softmax(-1)[0])) < 1e-6
    # An accepted eos ends the round with no draw.
    r = ospec.verify_draft(t, [1, 1], dl, [q0, q1], [0.0, 0.0], eos_token_id=1)
    assert [s[0] for s in r.steps] == [1] and r.n_accepted == 1
    # Draft equal to target everywhere: the correction is all zero -> fall back to p_target.
    p1 = t[1].softmax(-1)
    r = ospec.verify_draft(t[1:], [3], [float(torch.log(p1[3])) + 0.01], [p1 * 1.0001], [1.0])
    assert r.n_accepted == 0 and r.steps[0][0] == 0


def _c1_model(trace: dict, layers: int, seed: int):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    m = trace["model"]
    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=m["vocab"], hidden_size=m["hidden"], intermediate_size=m["intermediate"],
                      num_hidden_layers=layers, num_attention_heads=m["heads"], num_key_value_heads=m["kv_heads"],
                      head_dim=m["head_dim"], rope_theta=1e4, max_position_embeddings=256, tie_word_embeddings=False)
    return Qwen2ForCausalLM(cfg).eval()


@pytest.mark.parametrize("case", ["unrelated_draft", "draft_equals_target"])
def test_reference_orchestrator_run_is_reproduced(case):
    """The reference's own speculative loop, pinned.

    tests/golden/speculative_c1_trace.json records what AgentRL's
    ``SpeculativeRolloutOrchestrator._generate_speculative_tokens``
    (agentrl/generation/speculative.py:148-274) produced on CPU for a
    random-init fp32 Qwen2 target (2 layers, head_dim 16, vocab 512, seed 0)
    with an unrelated 1-layer draft (rejections and corrections) or a copy of
    the target (every draft accepted, bonus tokens), k = 4, greedy, 16 new
    tokens, eos 3 -- including the acceptance draws its ``torch.rand`` returned
    in every verify round.  Given those draws, the oracle's loop and the
    batched paged loop (PagedSpeculativeGenerator over fake stores, all three
    prompts at once) emit the same tokens and the same target log-probabilities.
    """
    from tests.conftest import load_json

    trace = load_json("speculative_c1_trace.json")
    target = _c1_model(trace, trace["target"]["layers"], trace["target"]["seed"])
    if case == "draft_equals_target":
        draft = copy.deepcopy(target)
    else:
        draft = _c1_model(trace, trace["drafts"][case]["layers"], trace["drafts"][case]["seed"])
    runs = trace["cases"][case]
    k, new, eos = trace["k"], trace["max_new_tokens"], trace["eos_token_id"]

    def draws(seq: int, rnd: int) -> list[float]:
        got = runs[seq]["round_draws"][rnd]
        return got + [0.5] * (k - len(got))  # draws after a rejection are never read

    for i, p in enumerate(trace["prompts"]):
        toks, lps, rounds = ospec.generate(p, _full_logits(target), _last_logits(draft), k=k, max_new_tokens=new,
                                           eos_token_id=eos, uniform_fn=lambda r, j, i=i: draws(i, r)[j])
        assert toks == runs[i]["tokens"]
        np.testing.assert_allclose(lps, runs[i]["logprobs"], rtol=1e-5, atol=1e-5)
        assert len(rounds) == len(runs[i]["round_draws"])

    sg = _spec(copy.deepcopy(target), copy.deepcopy(draft), k, eos=eos)
    res = sg.generate([torch.tensor(p) for p in trace["prompts"]], max_new_tokens=new, uniforms=draws)
    for i in range(len(trace["prompts"])):
        assert res["tokens"][i] == runs[i]["tokens"]
        np.testing.assert_allclose(res["logprobs"][i], runs[i]["logprobs"], rtol=1e-4, atol=1e-4)
    assert not sg.target.store.count and not sg.draft.store.count
