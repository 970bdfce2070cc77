"""Vocabulary-row kernels on the GPU against the oracle (reference arithmetic).

* ``token_logprobs`` / ``logsumexp`` equal float64 log_softmax + gather
  (agentrl/core/rollout.py:462-465) within 2e-5, on Qwen2's vocabulary of
  151 936 (vector loads), an odd vocabulary (scalar loads) and strided rows.
* greedy ``sample`` equals torch.argmax exactly, ties included (first index).
* sampled ``sample`` draws from softmax(logits / T) (top-p filtered): the
  empirical distribution of 400 000 draws is within a total-variation
  distance that the sample size bounds (0.02), and never leaves the nucleus.
* ``spec_accept`` equals the oracle's restatement of ``_verify_draft``
  (agentrl/generation/speculative.py:217-274) on random rounds at vocabulary
  151 936: the same accepted counts, emitted tokens and log-probabilities,
  except where the oracle itself sits on a tie (|u - acceptance| < 1e-5, or
  a top-2 gap of the argmax draw below 1e-6); sampled corrections and bonus
  tokens follow max(p - q, 0) and p.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampling as osamp
from oracle import speculative as ospec

pytestmark = pytest.mark.gpu

QWEN_VOCAB = 151936


def _sampler(dev, seed=0):
    from randomrepo_b200.sampling import DeviceSampler

    return DeviceSampler(dev, seed=seed)


@pytest.mark.parametrize("rows,vocab,pad", [(37, QWEN_VOCAB, 0), (5, 1001, 0), (3, 1001, 3), (9, 8200, 40),
                                            (1, 7, 0)])
def test_token_logprobs_match_log_softmax(cuda_device, rows, vocab, pad):
    g = torch.Generator().manual_seed(rows + vocab)
    full = torch.randn(rows, vocab + pad, generator=g) * 3.0
    logits = full.to(cuda_device)[:, :vocab]  # a row stride of vocab + pad
    tokens = torch.randint(0, vocab, (rows,), generator=g)
    s = _sampler(cuda_device)
    got = s.token_logprobs(logits, tokens.to(cuda_device)).cpu().numpy()
    want = osamp.token_logprobs(full[:, :vocab].numpy(), tokens.numpy())
    np.testing.assert_allclose(got, want, atol=2e-5, rtol=0)
    lse = s.logsumexp(logits).cpu().numpy().astype(np.float64)
    x = full[:, :vocab].double().numpy()
    np.testing.assert_allclose(lse, np.log(np.exp(x - x.max(1, keepdims=True)).sum(1)) + x.max(1), atol=2e-5)


def test_token_logprobs_batched_shape_and_out_of_range(cuda_device):
    s = _sampler(cuda_device)
    logits = torch.randn(3, 4, 300, device=cuda_device)
    tok = torch.randint(0, 300, (3, 4), device=cuda_device)
    tok[1, 2] = 300
    tok[2, 0] = -1
    got = s.token_logprobs(logits, tok)
    assert got.shape == (3, 4)
    want = torch.log_softmax(logits.double(), -1).gather(-1, tok.clamp(0, 299).unsqueeze(-1)).squeeze(-1)
    ok = torch.ones_like(got, dtype=torch.bool)
    ok[1, 2] = ok[2, 0] = False
    assert torch.isnan(got[~ok]).all()
    torch.testing.assert_close(got[ok].double(), want[ok], atol=2e-5, rtol=0)


def test_rejects_host_tensors():
    from randomrepo_b200.sampling import _rows

    with pytest.raises(ValueError):
        _rows(torch.zeros(2, 8), "test")


@pytest.mark.parametrize("vocab", [QWEN_VOCAB, 513])
def test_greedy_sample_is_torch_argmax_with_ties(cuda_device, vocab):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, vocab, generator=g)
    # Ties: equal maxima at two columns (in different chunks / threads).
    x[3, 10] = x[3, vocab - 3] = 50.0
    x[4, min(8192, vocab - 1)] = x[4, min(8191, vocab - 2)] = x[4, 100] = 60.0
    x[5, :] = 1.0
    logits = x.to(cuda_device)
    s = _sampler(cuda_device)
    tok, lp, am = s.sample(logits)
    want = torch.argmax(x, dim=-1)
    assert torch.equal(tok.cpu(), want) and torch.equal(am.cpu(), want)
    np.testing.assert_allclose(lp.cpu().numpy(), osamp.token_logprobs(x.numpy(), want.numpy()), atol=2e-5)


def _tv(counts: np.ndarray, probs: np.ndarray) -> float:
    return 0.5 * float(np.abs(counts / counts.sum() - probs).sum())


@pytest.mark.parametrize("temperature,top_p", [(1.0, 1.0), (0.7, 1.0), (1.3, 0.8)])
def test_sampled_tokens_follow_the_distribution(cuda_device, temperature, top_p):
    from randomrepo_b200.sampling import SamplingConfig

    vocab, n = 48, 400_000
    g = torch.Generator().manual_seed(9)
    row = torch.randn(vocab, generator=g) * 1.5
    logits = row.to(cuda_device).expand(n, vocab).contiguous()
    s = _sampler(cuda_device, seed=3)
    cfg = SamplingConfig(do_sample=True, temperature=temperature, top_p=top_p)
    tok, lp, am = s.sample(logits, cfg)
    counts = np.bincount(tok.cpu().numpy(), minlength=vocab).astype(np.float64)
    filt = osamp.apply_top_p((row / temperature).unsqueeze(0), top_p)[0]
    probs = torch.softmax(filt.double(), -1).numpy()
    assert counts[probs == 0].sum() == 0  # nothing outside the nucleus
    assert _tv(counts, probs) < 0.02, _tv(counts, probs)
    # The recorded log-probability is at temperature 1 (the old-policy value).
    ref = torch.log_softmax(row.double(), -1).numpy()
    np.testing.assert_allclose(lp.cpu().numpy()[:1000], ref[tok.cpu().numpy()[:1000]], atol=2e-5)
    assert torch.all(am == int(torch.argmax(row)))
    # Reseeding repeats the draws.
    s.reseed(3)
    tok2, _, _ = s.sample(logits, cfg)
    assert torch.equal(tok, tok2)


def _spec_case(seed: int, n: int, k: int, vocab: int, noise: float):
    g = torch.Generator().manual_seed(seed)
    tl = torch.randn(n, k + 1, vocab, generator=g) * 2.0
    dl = tl[:, :k] + noise * torch.randn(n, k, vocab, generator=g)
    dtok = torch.argmax(dl, dim=-1)
    # Some drafts are the draft's second choice (often rejected).
    alt = torch.topk(dl, 2, dim=-1).indices[..., 1]
    pick = torch.rand(n, k, generator=g) < 0.3
    dtok = torch.where(pick, alt, dtok)
    nd = torch.full((n,), k, dtype=torch.int32)
    nd[::7] = torch.randint(0, k + 1, nd[::7].shape, generator=g).to(torch.int32)
    u = torch.rand(n, k, generator=g)
    return tl, dl, dtok, nd, u


@pytest.mark.parametrize("vocab,temperature", [(QWEN_VOCAB, 1.0), (QWEN_VOCAB, 0.7), (1000, 1.0)])
def test_spec_accept_greedy_matches_oracle(cuda_device, vocab, temperature):
    n, k = 48, 4
    tl, dl, dtok, nd, u = _spec_case(1, n, k, vocab, 0.7)
    eos = int(dtok[5, 1])  # an eos among the drafts of some sequences
    s = _sampler(cuda_device)
    tok, lp, n_out, n_acc = s.spec_accept(tl.to(cuda_device), dl.to(cuda_device), dtok.to(cuda_device),
                                          nd.to(cuda_device), draft_temperature=temperature, do_sample=False,
                                          eos_token_id=eos, uniforms=u.to(cuda_device))
    want = ospec.accept_batch(tl, dl, dtok, nd, u, draft_temperature=temperature, eos_token_id=eos)
    tok, lp, n_out, n_acc = tok.cpu(), lp.cpu(), n_out.cpu(), n_acc.cpu()
    exact = 0
    for b in range(n):
        tied = want.u_margin[b] < 1e-5 or want.draw_gap[b] < 1e-6
        same = (int(n_acc[b]) == int(want.n_acc[b]) and int(n_out[b]) == int(want.n_out[b])
                and torch.equal(tok[b], want.tokens[b]))
        assert same or tied, (b, tok[b].tolist(), want.tokens[b].tolist(), want.u_margin[b], want.draw_gap[b])
        if same:
            exact += 1
            m = int(n_out[b])
            np.testing.assert_allclose(lp[b, :m].numpy(), want.logprobs[b, :m].numpy(), atol=1e-4)
    assert exact >= n - 2
    assert (n_acc < torch.as_tensor(nd).clamp(max=k)).any() and (n_out == n_acc + 1).any()


def test_spec_accept_sampled_corrections_and_bonus_follow_the_distribution(cuda_device):
    vocab, n, k = 16, 200_000, 2
    g = torch.Generator().manual_seed(4)
    t_row = torch.randn(k + 1, vocab, generator=g)
    d_row = torch.randn(k, vocab, generator=g)
    tl = t_row.expand(n, k + 1, vocab).contiguous()
    dl = d_row.expand(n, k, vocab).contiguous()
    p0 = torch.softmax(t_row[0].double(), -1)
    q0 = torch.softmax(d_row[0].double(), -1)
    d0 = int(torch.argmax(q0 - p0))          # a draft the target likes less than the draft does
    dtok = torch.tensor([d0, 0]).expand(n, k).contiguous()
    nd = torch.full((n,), k, dtype=torch.int32)
    s = _sampler(cuda_device, seed=21)
    dev = cuda_device
    # u = 1: draft 0 rejected (acceptance < 1) -> correction from max(p - q, 0).
    tok, _, n_out, n_acc = s.spec_accept(tl.to(dev), dl.to(dev), dtok.to(dev), nd.to(dev), do_sample=True,
                                         uniforms=torch.ones(n, k, device=dev))
    assert torch.all(n_acc == 0) and torch.all(n_out == 1)
    corr = (p0 - q0).clamp(min=0)
    corr = (corr / corr.sum()).numpy()
    counts = np.bincount(tok[:, 0].cpu().numpy(), minlength=vocab).astype(np.float64)
    assert counts[corr == 0].sum() == 0 and _tv(counts, corr) < 0.01, _tv(counts, corr)
    # u = 0: both drafts accepted -> bonus from p of row k (temperature 1).
    tok, lp, n_out, n_acc = s.spec_accept(tl.to(dev), dl.to(dev), dtok.to(dev), nd.to(dev), do_sample=True,
                                          draft_temperature=0.5, uniforms=torch.zeros(n, k, device=dev))
    assert torch.all(n_acc == 2) and torch.all(n_out == 3)
    pk = torch.softmax(t_row[k].double(), -1).numpy()
    counts = np.bincount(tok[:, 2].cpu().numpy(), minlength=vocab).astype(np.float64)
    assert _tv(counts, pk) < 0.01, _tv(counts, pk)
    np.testing.assert_allclose(lp[:100, 2].cpu().numpy(), np.log(pk)[tok[:100, 2].cpu().numpy()], atol=2e-5)


def test_spec_accept_hashed_draws_are_reproducible_and_bad_tokens_flagged(cuda_device):
    n, k, vocab = 32, 4, 4096
    tl, dl, dtok, nd, _ = _spec_case(2, n, k, vocab, 1.0)
    dev = cuda_device
    args = (tl.to(dev), dl.to(dev), dtok.to(dev), nd.to(dev))
    s = _sampler(dev, seed=5)
    a = s.spec_accept(*args, do_sample=True)
    s.reseed(5)
    b = s.spec_accept(*args, do_sample=True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    bad = dtok.clone()
    bad[3, 0] = vocab
    nd_full = torch.full((n,), k, dtype=torch.int32)
    _, _, n_out, _ = s.spec_accept(tl.to(dev), dl.to(dev), bad.to(dev), nd_full.to(dev))
    assert int(n_out[3]) == -1 and (n_out[torch.arange(n) != 3] > 0).all()
