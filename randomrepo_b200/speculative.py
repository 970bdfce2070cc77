"""Paged speculative decoding: draft and target both keep paged caches; accept / reject runs on the device.

AgentRL's ``SpeculativeRolloutOrchestrator`` (agentrl/generation/speculative.py:148-274)
decodes one sequence at a time and recomputes the whole prefix with a full
forward for every draft token and for every verify.  ``PagedSpeculativeGenerator``
runs the same algorithm over a whole batch with both models' K/V in paged
stores:

* each prompt is prefilled once per model (all but its last token, which
  opens the first round) and the other members of its GRPO group fork the
  prompt's pages (copy-on-write);
* a round over all active sequences is k draft forwards -- the first feeds
  the draft the one or two tokens it has not seen yet, the rest are decode
  steps; with ``cuda_graphs=True`` on the draft all of them are graphed decode
  steps (sequences two tokens behind take one extra step first) -- then
  one target forward of k + 1 tokens per sequence, the paged verify read
  (``verify`` rows = positions prefix_len - 1 .. prefix_len - 1 + k),
  replayed from a CUDA graph with ``cuda_graphs=True`` on the target;
* ``pkv_spec_accept`` decides every sequence's round in one launch group;
* rejected drafts leave both caches through ``truncate`` (blocks past the
  kept tokens return to the pool, shared prompt blocks stay shared).

Decisions follow the reference exactly, including that the target's
distributions are softmax(logits) at temperature 1 while the draft's are
softmax(logits / T) (speculative.py:200,236-237), that the draft proposes
min(k, max_new_tokens) tokens and stops after eos (:198-211), and that an
accepted eos ends the sequence without a further draw (:247-249).  The
acceptance draws u come from the sampler's counter-based hash unless a
``uniforms`` function supplies them (tests give both implementations the same
draws).
"""

from __future__ import annotations

import torch

from .sampling import SamplingConfig


class PagedSpeculativeGenerator:
    """Batched speculative rollout over two ``PagedGenerator`` s (target = policy, draft = frozen proposal model)."""

    def __init__(self, target, draft, *, k: int = 4, eos_token_id: int | None = None, sampler=None) -> None:
        if k < 1:
            raise ValueError("k must be positive")  # config.py validates speculative_k > 0
        if target.device != draft.device:
            raise ValueError("target and draft must live on one device")
        self.target = target
        self.draft = draft
        self.k = int(k)
        self.eos_token_id = eos_token_id
        self._sampler = sampler

    @property
    def sampler(self):
        return self._sampler if self._sampler is not None else self.target.sampler

    @staticmethod
    def break_even(draft_model_size_b: float, policy_model_size_b: float, k: int) -> float:
        """speculative.py:53-67: K / (1 + draft / policy size)."""
        if draft_model_size_b <= 0 or policy_model_size_b <= 0:
            raise ValueError("Model sizes must be positive.")
        if k <= 0:
            raise ValueError("K must be positive.")
        return k / (1.0 + draft_model_size_b / policy_model_size_b)

    # -- helpers ----------------------------------------------------------------
    @staticmethod
    def _prefill_prefixes(gen, ids, prefixes) -> None:
        """Reserve each sequence and write the K/V of its prefix (possibly empty) in packed chunks."""
        for sid in ids:
            gen.store.reserve(sid, 0)
        cs = gen.prefill_chunk_size
        longest = max((len(p) for p in prefixes), default=0)
        for c in range(0, longest, cs):
            members = [j for j, p in enumerate(prefixes) if len(p) > c]
            if members:
                gen.extend_hidden([ids[j] for j in members], [prefixes[j][c:c + cs] for j in members])

    def _draft_round(self, ids, pending, k: int, temperature: float | None):
        """k draft proposals per sequence: (tokens [n, k] int64, logits [n, k, vocab] float32)."""
        draft, sampler = self.draft, self.sampler
        dev = draft.device
        h2d = draft._h2d
        if draft.cuda_graphs:
            # Graphed decode steps only: sequences two tokens behind take one
            # step on their own first (its logits are not needed).
            two = [j for j, p in enumerate(pending) if len(p) == 2]
            if two:
                draft.decode_step([ids[j] for j in two], h2d.to_device([pending[j][0] for j in two], dev,
                                                                       torch.long))
            first = draft.decode_step(ids, h2d.to_device([p[-1] for p in pending], dev, torch.long))
        elif all(len(p) == 1 for p in pending):
            first = draft.decode_step(ids, h2d.to_device([p[0] for p in pending], dev, torch.long))
        else:
            first = draft.extend(ids, pending)
        n, vocab = first.shape
        logits = torch.empty((n, k, vocab), dtype=torch.float32, device=dev)
        tokens = torch.empty((n, k), dtype=torch.int64, device=dev)
        cur = first
        for j in range(k):
            if j:
                cur = draft.decode_step(ids, tokens[:, j - 1])
            logits[:, j].copy_(cur)
            tok, _, _ = sampler.sample(cur, temperature=temperature)
            tokens[:, j].copy_(tok)
        return tokens, logits

    # -- rollout ------------------------------------------------------------------
    def generate(self, prompts, *, group_size: int = 1, max_new_tokens: int = 16,
                 sampling: SamplingConfig | None = None, first_id: int = 0, release: bool = True,
                 uniforms=None, trace: bool = False) -> dict:
        """Roll out ``group_size`` completions per prompt with speculative decoding.

        Returns ``{"sequence_ids", "tokens", "logprobs" (the target's
        log-probability of each emitted token, speculative.py:168-169),
        "rounds", "proposed", "accepted"}`` and with ``trace`` a per-sequence
        list of rounds ``(prefix_len, drafts, n_draft, n_accepted, emitted)``.
        ``uniforms(seq_index, round_index) -> k floats`` (optional) supplies the
        acceptance draws.
        """
        cfg = sampling or SamplingConfig()
        self.sampler.reseed(cfg.seed)
        do_sample = bool(cfg.do_sample) and cfg.temperature > 0
        eff_t = cfg.temperature if cfg.temperature > 0 else 1.0
        draft_t = eff_t if do_sample else None
        k = min(self.k, int(max_new_tokens))
        n_groups = len(prompts)
        heads = [first_id + g * group_size for g in range(n_groups)]
        toks = [[int(t) for t in torch.as_tensor(p).reshape(-1).tolist()] for p in prompts]
        if any(len(t) == 0 for t in toks):
            raise ValueError("prompts must be non-empty")
        seq_ids = [heads[g] + m for g in range(n_groups) for m in range(group_size)]
        n = len(seq_ids)
        result = {"sequence_ids": seq_ids, "tokens": [[] for _ in range(n)], "logprobs": [[] for _ in range(n)],
                  "rounds": 0, "proposed": 0, "accepted": 0}
        if trace:
            result["trace"] = [[] for _ in range(n)]
        if max_new_tokens <= 0 or n == 0:
            return result

        try:
            return self._rounds(toks, heads, seq_ids, group_size, max_new_tokens, k, do_sample, eff_t, draft_t,
                                uniforms, trace, release, result)
        except BaseException:
            if release:
                self._release(seq_ids)
            raise

    def _rounds(self, toks, heads, seq_ids, group_size, max_new_tokens, k, do_sample, eff_t, draft_t, uniforms,
                trace, release, result) -> dict:
        """Prefill both caches, then speculative rounds until every sequence is done."""
        sampler = self.sampler
        eos = self.eos_token_id
        n_groups = len(toks)
        n = len(seq_ids)
        # Prompts minus their last token into both caches, once per group.
        for gen in (self.target, self.draft):
            self._prefill_prefixes(gen, heads, [t[:-1] for t in toks])
            for g in range(n_groups):
                for m in range(1, group_size):
                    gen.store.fork(heads[g], heads[g] + m)
        longest = max(len(t) for t in toks) + max_new_tokens + k + 1
        for gen in (self.target, self.draft):
            if gen.cuda_graphs:
                gen.reserve_tables(longest)

        prompt_of = [toks[i // group_size] for i in range(n)]
        gen_toks = result["tokens"]
        gen_lps = result["logprobs"]
        dlen = [len(p) - 1 for p in prompt_of]      # tokens in the draft's cache
        active = list(range(n))
        dev = self.target.device
        rnd = 0
        while active:
            ids = [seq_ids[i] for i in active]
            prefix = [prompt_of[i] + gen_toks[i] for i in active]
            plen = [len(p) for p in prefix]
            pending = [prefix[j][dlen[i]:] for j, i in enumerate(active)]
            dtok, dlogits = self._draft_round(ids, pending, k, draft_t)
            if eos is not None:
                is_eos = dtok == eos
                first = torch.argmax(is_eos.to(torch.int32), dim=1)
                n_draft = torch.where(is_eos.any(dim=1), first + 1, torch.full_like(first, k)).to(torch.int32)
            else:
                n_draft = torch.full((len(active),), k, dtype=torch.int32, device=dev)
            # Target verify: the last accepted token and the k drafts of every sequence.
            dtok_h = dtok.cpu()
            chunks = [[prefix[j][-1]] + dtok_h[j].tolist() for j in range(len(active))]
            tlogits = self.target.verify_logits(ids, chunks).view(len(active), k + 1, -1)
            u = None
            if uniforms is not None:
                u = torch.tensor([list(uniforms(i, rnd))[:k] for i in active], dtype=torch.float32, device=dev)
            out_tok, out_lp, n_out, n_acc = sampler.spec_accept(
                tlogits, dlogits, dtok, n_draft, draft_temperature=eff_t, do_sample=do_sample, eos_token_id=eos,
                uniforms=u)
            out_tok, out_lp = out_tok.cpu().tolist(), out_lp.cpu().tolist()
            n_out, n_acc, nd_h = n_out.cpu().tolist(), n_acc.cpu().tolist(), n_draft.cpu().tolist()
            rnd += 1
            result["rounds"] = rnd
            still, t_keep, d_keep, keep_ids = [], [], [], []
            for j, i in enumerate(active):
                if n_out[j] < 0:
                    raise ValueError(f"sequence {seq_ids[i]}: a draft token lies outside the vocabulary")
                result["proposed"] += nd_h[j]
                result["accepted"] += n_acc[j]
                emitted = out_tok[j][:n_out[j]]
                done = False
                kept = 0
                for t, lp in zip(emitted, out_lp[j][:n_out[j]]):
                    gen_toks[i].append(int(t))
                    gen_lps[i].append(float(lp))
                    kept += 1
                    if t == eos or len(gen_toks[i]) >= max_new_tokens:
                        done = True
                        break
                if trace:
                    result["trace"][i].append((plen[j], dtok_h[j].tolist(), nd_h[j], n_acc[j], emitted[:kept]))
                if done:
                    if release:
                        for gen in (self.target, self.draft):
                            if gen.store.has_sequence(seq_ids[i]):
                                gen.store.release(seq_ids[i])
                    continue
                still.append(i)
                keep_ids.append(seq_ids[i])
                # Target: holds prefix + k drafts; keep up to the token before the new last one.
                t_keep.append(plen[j] + kept - 1)
                # Draft: holds prefix + drafts 1..k-1; keep what the new prefix still agrees with.
                dlen[i] = min(plen[j] + k - 1, plen[j] + kept - 1)
                d_keep.append(dlen[i])
            if keep_ids:
                self.target.store.truncate(keep_ids, t_keep)
                self.draft.store.truncate(keep_ids, d_keep)
            active = still
        if release:
            self._release(seq_ids)
        return result

    def _release(self, seq_ids) -> None:
        for sid in seq_ids:
            for gen in (self.target, self.draft):
                if gen.store.has_sequence(sid):
                    gen.store.release(sid)
        for gen in (self.target, self.draft):
            gen.release_placeholders()
