"""Oracle restatement of the reference's speculative decoding (test infrastructure).

``SpeculativeRolloutOrchestrator`` (agentrl/generation/speculative.py) with the
model calls and the random draws supplied by the caller:

* ``propose`` -- ``_draft_propose`` (speculative.py:188-215): up to
  min(k, max_new_tokens) draft tokens, each from softmax(draft logits / T)
  (argmax when greedy), stopping after eos;
* ``verify_draft`` -- ``_verify_draft`` (speculative.py:217-274): accept draft
  i when u_i <= min(1, exp(lp_target - lp_draft)); on the first rejection draw
  a correction from max(p_target - p_draft, 0) (p_target if that is all zero);
  after accepting every draft draw a bonus token from p_target of the last
  row; an accepted eos ends the round;
* ``generate`` -- ``_generate_speculative_tokens`` (speculative.py:148-185):
  rounds of propose + verify over the growing prefix until max_new_tokens or
  eos, every model call a full forward over the whole prefix;
* ``accept_batch`` -- ``verify_draft`` for a batch of rounds laid out as the
  library's ``pkv_spec_accept`` takes them.

The target's probabilities are softmax(logits) at temperature 1 and the
draft's softmax(logits / T), as in the reference (speculative.py:200,236-237).
Arithmetic is the reference's float32 torch on CPU.  Nothing outside tests
imports this module.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


def _argmax(probs: torch.Tensor) -> int:
    return int(torch.argmax(probs).item())


def _gap(probs: torch.Tensor) -> float:
    """Top-1 minus top-2 of a distribution: how far an argmax draw is from a tie."""
    if probs.numel() < 2:
        return float("inf")
    top = torch.topk(probs.double(), 2).values
    return float(top[0] - top[1])


@dataclass
class VerifyResult:
    steps: list                 # [(token, target logprob)]
    n_accepted: int
    u_margin: float = float("inf")    # min |u - acceptance| over the decisions taken
    draw_gap: float = float("inf")    # top-1 minus top-2 of the argmax draw's distribution


def propose(draft_last_logits, prefix: list[int], k: int, max_new_tokens: int, *, temperature: float = 1.0,
            eos_token_id: int | None = None, sample_fn=None):
    """speculative.py:188-215.  ``draft_last_logits(ids) -> [vocab]`` logits after ``ids``."""
    eff_t = temperature if temperature > 0 else 1.0
    tokens, logprobs, probs_list = [], [], []
    current = list(prefix)
    for _ in range(min(k, max_new_tokens)):
        logits = draft_last_logits(current).float()
        probs = torch.softmax(logits / eff_t, dim=-1)
        tok = sample_fn(probs) if sample_fn is not None else _argmax(probs)
        tokens.append(tok)
        logprobs.append(float(torch.log(probs[tok] + 1e-12).item()))
        probs_list.append(probs)
        current.append(tok)
        if tok == eos_token_id:
            break
    return tokens, logprobs, probs_list


def verify_draft(target_rows: torch.Tensor, draft_tokens, draft_logprobs, draft_probs, uniforms, *,
                 eos_token_id: int | None = None, sample_fn=None) -> VerifyResult:
    """speculative.py:217-274.  ``target_rows [n_draft + 1, vocab]``: the target's logits at
    positions prefix_len - 1 .. prefix_len - 1 + n_draft of the full verify forward."""
    if not draft_tokens:
        return VerifyResult([], 0)
    rows = target_rows.float()
    logprobs = torch.log_softmax(rows, dim=-1)
    probs = torch.softmax(rows, dim=-1)
    draw = sample_fn if sample_fn is not None else _argmax
    res = VerifyResult([], 0)
    for index, (token_id, draft_logprob, draft_prob) in enumerate(zip(draft_tokens, draft_logprobs, draft_probs)):
        policy_logprob = float(logprobs[index, token_id].item())
        acceptance = min(1.0, float(torch.exp(torch.tensor(policy_logprob - draft_logprob)).item()))
        u = float(uniforms[index])
        res.u_margin = min(res.u_margin, abs(u - acceptance))
        if u <= acceptance:
            res.steps.append((int(token_id), policy_logprob))
            res.n_accepted += 1
            if token_id == eos_token_id:
                return res
            continue
        correction = (probs[index] - draft_prob.float()).clamp(min=0)
        if float(correction.sum().item()) <= 0:
            correction = probs[index]
        else:
            correction = correction / correction.sum()
        tok = draw(correction)
        if sample_fn is None:
            res.draw_gap = _gap(correction)
        res.steps.append((tok, float(logprobs[index, tok].item())))
        return res
    last = len(draft_tokens)
    tok = draw(probs[last])
    if sample_fn is None:
        res.draw_gap = _gap(probs[last])
    res.steps.append((tok, float(logprobs[last, tok].item())))
    return res


@dataclass
class AcceptResult:
    tokens: torch.Tensor        # [n, k+1] int64, -1 past n_out
    logprobs: torch.Tensor      # [n, k+1] float32, 0 past n_out
    n_out: torch.Tensor         # [n] int32
    n_acc: torch.Tensor         # [n] int32
    u_margin: list = field(default_factory=list)
    draw_gap: list = field(default_factory=list)


def accept_batch(target_logits, draft_logits, draft_tokens, n_draft, uniforms, *, draft_temperature: float = 1.0,
                 eos_token_id: int | None = None, sample_fn=None) -> AcceptResult:
    """``verify_draft`` per sequence of a batch: target_logits [n, k+1, vocab], draft_logits
    [n, k, vocab] (the draft logits that proposed each token), draft_tokens [n, k], n_draft [n],
    uniforms [n, k]."""
    tl = torch.as_tensor(target_logits).float().cpu()
    dl = torch.as_tensor(draft_logits).float().cpu()
    dt = torch.as_tensor(draft_tokens).long().cpu()
    nd = torch.as_tensor(n_draft).long().cpu()
    uu = torch.as_tensor(uniforms).float().cpu()
    n, k1, _ = tl.shape
    k = k1 - 1
    eff_t = draft_temperature if draft_temperature > 0 else 1.0
    out = AcceptResult(torch.full((n, k1), -1, dtype=torch.int64), torch.zeros((n, k1), dtype=torch.float32),
                       torch.zeros(n, dtype=torch.int32), torch.zeros(n, dtype=torch.int32))
    for b in range(n):
        m = int(min(max(int(nd[b]), 0), k))
        toks = [int(t) for t in dt[b, :m]]
        probs = [torch.softmax(dl[b, i] / eff_t, dim=-1) for i in range(m)]
        lps = [float(torch.log(probs[i][toks[i]] + 1e-12).item()) for i in range(m)]
        if m == 0:
            # speculative.py:170-171: no proposal -> one direct policy step
            # (_direct_policy_step, :276-283), a draw from the target's row 0.
            draw = sample_fn if sample_fn is not None else _argmax
            lp0 = torch.log_softmax(tl[b, 0], dim=-1)
            tok = draw(lp0.exp())
            res = VerifyResult([(tok, float(lp0[tok].item()))], 0)
            if sample_fn is None:
                res.draw_gap = _gap(lp0.exp())
        else:
            res = verify_draft(tl[b, :m + 1], toks, lps, probs, uu[b, :m], eos_token_id=eos_token_id,
                               sample_fn=sample_fn)
        for i, (tok, lp) in enumerate(res.steps):
            out.tokens[b, i] = tok
            out.logprobs[b, i] = lp
        out.n_out[b] = len(res.steps)
        out.n_acc[b] = res.n_accepted
        out.u_margin.append(res.u_margin)
        out.draw_gap.append(res.draw_gap)
    return out


def generate(prompt: list[int], target_logits, draft_last_logits, *, k: int, max_new_tokens: int,
             eos_token_id: int | None = None, temperature: float = 1.0, uniform_fn=None, sample_fn=None):
    """speculative.py:148-185 for one prompt.

    ``target_logits(ids) -> [len(ids), vocab]`` is a full forward; ``uniform_fn(round, i)`` gives
    the acceptance draw of draft i in round ``round`` (the reference calls torch.rand).  Returns
    (tokens, logprobs, rounds) with rounds a list of (prefix_len, drafts, n_accepted, emitted).
    """
    generated: list[int] = []
    logprobs: list[float] = []
    rounds = []
    r = 0
    while len(generated) < max_new_tokens:
        prefix = list(prompt) + generated
        drafts, dlps, dprobs = propose(draft_last_logits, prefix, k, max_new_tokens, temperature=temperature,
                                       eos_token_id=eos_token_id, sample_fn=sample_fn)
        rows = target_logits(prefix + drafts)[len(prefix) - 1:]
        us = [uniform_fn(r, i) for i in range(len(drafts))]
        res = verify_draft(rows, drafts, dlps, dprobs, us, eos_token_id=eos_token_id, sample_fn=sample_fn)
        steps = res.steps
        if not steps:
            lp0 = torch.log_softmax(rows[0].float(), dim=-1)
            tok = (sample_fn or _argmax)(lp0.exp())
            steps = [(tok, float(lp0[tok].item()))]
        rounds.append((len(prefix), list(drafts), res.n_accepted, [t for t, _ in steps]))
        r += 1
        for tok, lp in steps:
            generated.append(tok)
            logprobs.append(lp)
            if tok == eos_token_id:
                return generated, logprobs, rounds
            if len(generated) >= max_new_tokens:
                break
    return generated, logprobs, rounds
