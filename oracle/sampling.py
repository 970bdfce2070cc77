"""Oracle restatement of the reference's vocabulary-row arithmetic (test infrastructure).

* Token log-probabilities: ``RolloutOrchestrator._compute_logprobs``
  (agentrl/core/rollout.py:456-472): log_softmax over the vocabulary, then a
  gather of the next token.
* Next-token selection: ``_sample_next_token`` / ``_apply_top_p``
  (rollout.py:307-329): argmax, or ``torch.multinomial`` over
  softmax(top_p(logits / T)).
* Speculative accept / reject: ``oracle.speculative``.

``OracleSampler`` offers these behind the interface of the library's
``DeviceSampler`` (same method names, argument meaning and outputs) with the
reference's own torch CPU ops, so that the rollout loops can be exercised on
CPU in tests.  Nothing outside tests imports this module.
"""

from __future__ import annotations

import numpy as np
import torch

from . import speculative as _spec


def log_softmax64(logits: np.ndarray) -> np.ndarray:
    """float64 log_softmax over the last axis."""
    x = np.asarray(logits, dtype=np.float64)
    m = x.max(axis=-1, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(axis=-1, keepdims=True))


def token_logprobs(logits: np.ndarray, tokens: np.ndarray) -> np.ndarray:
    """rollout.py:462-465 in float64: log_softmax(logits)[row, tokens[row]]."""
    lp = log_softmax64(logits)
    tok = np.asarray(tokens, dtype=np.int64).reshape(-1)
    return np.take_along_axis(lp.reshape(tok.size, -1), tok[:, None], axis=1)[:, 0]


def apply_top_p(logits: torch.Tensor, top_p: float) -> torch.Tensor:
    """rollout.py:317-329: nucleus filter with the crossing token kept."""
    if top_p >= 1.0:
        return logits
    sorted_logits, sorted_indices = torch.sort(logits, descending=True, dim=-1)
    cumulative = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
    mask = cumulative > top_p
    mask[..., 1:] = mask[..., :-1].clone()
    mask[..., 0] = False
    filtered = sorted_logits.masked_fill(mask, float("-inf"))
    return torch.empty_like(filtered).scatter(-1, sorted_indices, filtered)


class OracleSampler:
    """CPU stand-in for ``randomrepo_b200.sampling.DeviceSampler`` built from the reference's torch ops."""

    def __init__(self, device=None, seed: int = 0) -> None:
        self.device = torch.device("cpu")
        self.reseed(seed)

    def reseed(self, seed: int) -> None:
        self.seed = int(seed)
        self.gen = torch.Generator().manual_seed(self.seed)

    def token_logprobs(self, logits: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        lp = torch.log_softmax(logits.float(), dim=-1)
        return lp.gather(-1, tokens.long().unsqueeze(-1)).squeeze(-1)

    def sample(self, logits: torch.Tensor, cfg=None, temperature: float | None = None):
        logits = logits.float()
        do_sample = bool(getattr(cfg, "do_sample", False)) if cfg is not None else bool(temperature)
        t = float(temperature if temperature is not None else getattr(cfg, "temperature", 1.0))
        top_p = float(getattr(cfg, "top_p", 1.0)) if cfg is not None else 1.0
        am = torch.argmax(logits, dim=-1)
        if do_sample and t > 0:
            probs = torch.softmax(apply_top_p(logits / t, top_p), dim=-1)
            tok = torch.multinomial(probs.reshape(-1, probs.shape[-1]), 1, generator=self.gen).reshape(am.shape)
        else:
            tok = am
        lp = torch.log_softmax(logits, dim=-1).gather(-1, tok.unsqueeze(-1)).squeeze(-1)
        return tok, lp, am

    def spec_accept(self, target_logits, draft_logits, draft_tokens, n_draft, *, draft_temperature=1.0,
                    do_sample=False, eos_token_id=None, uniforms=None):
        n, k1, _ = target_logits.shape
        if uniforms is None:
            uniforms = torch.rand((n, k1 - 1), generator=self.gen)
        sample_fn = None
        if do_sample:
            def sample_fn(probs):
                return int(torch.multinomial(probs, 1, generator=self.gen).item())
        res = _spec.accept_batch(target_logits, draft_logits, draft_tokens, n_draft, uniforms,
                                 draft_temperature=draft_temperature, eos_token_id=eos_token_id, sample_fn=sample_fn)
        return res.tokens, res.logprobs, res.n_out, res.n_acc
