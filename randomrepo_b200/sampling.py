"""Vocabulary-row kernels of libpkv_b200: token log-probabilities, token selection, speculative accept / reject.

Every rollout step ends in [sequences, vocab] fp32 logits (151 936 columns for
Qwen2).  AgentRL turns them into tokens with torch ops (agentrl/core/rollout.py:307-329),
recomputes the tokens' log-probabilities with a second full forward and a
[B, L, vocab] log_softmax (rollout.py:456-472), and accepts or rejects
speculative drafts one sequence and one ``.item()`` at a time
(agentrl/generation/speculative.py:217-274).  ``DeviceSampler`` does each of
these in one pass over the logits rows on the GPU:

* ``token_logprobs`` -- log_softmax + gather without materialising the
  log-softmax (``pkv_token_logprobs``);
* ``sample`` -- argmax, or a draw from softmax(logits / T) (top-p filtered
  when ``top_p < 1``), plus the token's temperature-1 log-probability and the
  row's argmax (``pkv_sample_tokens``);
* ``spec_accept`` -- the accept / reject / correction / bonus decisions of a
  whole batch of speculative rounds (``pkv_spec_accept``).

Draws come from a counter-based hash of (seed, call counter, row, column), so
a sampler reseeded with the same seed repeats its draws.  There is no CPU
path: host tensors are rejected.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import lib


@dataclass
class SamplingConfig:
    """agentrl/core/rollout.py:307-329: greedy unless do_sample with temperature > 0 (then top-p)."""

    do_sample: bool = False
    temperature: float = 1.0
    top_p: float = 1.0
    seed: int = 0

    @property
    def sampling(self) -> bool:
        return bool(self.do_sample) and self.temperature > 0


def top_p_filter(logits: torch.Tensor, top_p: float) -> torch.Tensor:
    """Nucleus filter of rollout.py:317-329: keep the smallest prefix of the sorted
    distribution whose mass reaches ``top_p`` (the token that crosses it included)."""
    if top_p >= 1.0:
        return logits
    sorted_logits, idx = torch.sort(logits, descending=True, dim=-1)
    probs = torch.softmax(sorted_logits, dim=-1)
    cum = probs.cumsum(dim=-1)
    drop = cum - probs > top_p
    sorted_logits = sorted_logits.masked_fill(drop, float("-inf"))
    return torch.full_like(logits, float("-inf")).scatter(-1, idx, sorted_logits)


def _stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def _rows(logits: torch.Tensor, what: str) -> tuple[int, int, int]:
    """(rows, vocab, row stride) of fp32 CUDA logits [..., vocab] whose rows are evenly strided."""
    if not logits.is_cuda:
        raise ValueError(f"{what}: logits must be a CUDA tensor (the vocabulary kernels have no CPU path)")
    if logits.dtype != torch.float32:
        raise ValueError(f"{what}: logits must be float32")
    if logits.dim() < 1 or logits.shape[-1] < 1 or logits.stride(-1) != 1:
        raise ValueError(f"{what}: logits must be [..., vocab] with a contiguous vocabulary dim")
    vocab = logits.shape[-1]
    try:
        flat = logits.view(-1, vocab)
    except RuntimeError:
        raise ValueError(f"{what}: logits rows must be evenly strided") from None
    rows = flat.shape[0]
    return rows, vocab, (flat.stride(0) if rows > 1 else vocab)


class DeviceSampler:
    """Sampling, log-probabilities and speculative accept / reject on the device."""

    def __init__(self, device=None, seed: int = 0) -> None:
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DeviceSampler runs on a CUDA device")
        self.seed = int(seed)
        self.offset = 0
        self.launches = 0
        self._ws = torch.empty(0, dtype=torch.uint8, device=self.device)
        self._tickets = torch.zeros(0, dtype=torch.int32, device=self.device)

    def reseed(self, seed: int) -> None:
        """Restart the draw sequence: the same seed repeats the same draws."""
        self.seed = int(seed)
        self.offset = 0

    def _workspace(self, nbytes: int, n_tickets: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Scratch of ``nbytes`` and ``n_tickets`` tickets (zero-filled once; the kernels leave them zero)."""
        if nbytes < 0 or n_tickets < 0:
            raise ValueError("invalid vocabulary-row workspace request")
        if nbytes > self._ws.numel():
            self._ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
        if n_tickets > self._tickets.numel():
            self._tickets = torch.zeros(max(n_tickets, 4096), dtype=torch.int32, device=self.device)
        return self._ws, self._tickets

    def _next_offset(self) -> int:
        self.offset += 1
        return self.offset

    # -- log-probabilities ------------------------------------------------------
    def token_logprobs(self, logits: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        """``log_softmax(logits, -1).gather(-1, tokens)`` for logits [..., vocab] and tokens [...]
        (rollout.py:462-465); NaN where a token lies outside the vocabulary."""
        rows, vocab, ld = _rows(logits, "token_logprobs")
        tok = tokens.to(device=logits.device, dtype=torch.int64).reshape(-1).contiguous()
        if tok.numel() != rows:
            raise ValueError("token_logprobs: one token per logits row")
        out = torch.empty(rows, dtype=torch.float32, device=logits.device)
        if rows:
            ws, tk = self._workspace(int(lib.pkv_sampling_workspace_bytes(rows, vocab)), rows)
            st = lib.pkv_token_logprobs(logits.data_ptr(), ld, rows, vocab, tok.data_ptr(), out.data_ptr(), None,
                                        tk.data_ptr(), ws.data_ptr(), ws.numel(), _stream_ptr())
            _lib.raise_for_status(st)
            self.launches += 1
        return out.view(tokens.shape)

    def logsumexp(self, logits: torch.Tensor) -> torch.Tensor:
        """``torch.logsumexp(logits, -1)`` in one pass per row."""
        rows, vocab, ld = _rows(logits, "logsumexp")
        out = torch.empty(rows, dtype=torch.float32, device=logits.device)
        if rows:
            ws, tk = self._workspace(int(lib.pkv_sampling_workspace_bytes(rows, vocab)), rows)
            st = lib.pkv_token_logprobs(logits.data_ptr(), ld, rows, vocab, None, None, out.data_ptr(),
                                        tk.data_ptr(), ws.data_ptr(), ws.numel(), _stream_ptr())
            _lib.raise_for_status(st)
            self.launches += 1
        return out.view(logits.shape[:-1])

    # -- token selection --------------------------------------------------------
    def sample(self, logits: torch.Tensor, cfg: SamplingConfig | None = None,
               temperature: float | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Next tokens of logits [n, vocab]: (tokens int64 [n], their temperature-1
        log-probabilities [n], the rows' argmax [n]).

        Greedy unless ``cfg`` samples (rollout.py:307-315); a sampled draw is from
        softmax(top_p_filter(logits / T)).  ``temperature`` overrides ``cfg``'s
        (and samples when > 0 and ``cfg`` is None).
        """
        _rows(logits, "sample")
        if cfg is None:
            cfg = SamplingConfig(do_sample=temperature is not None and temperature > 0,
                                 temperature=temperature if temperature is not None else 1.0)
        t = float(cfg.temperature if temperature is None else temperature)
        do_sample = bool(cfg.do_sample) and t > 0
        race = None
        if do_sample and cfg.top_p < 1.0:
            logits = logits.contiguous()
            race = top_p_filter(logits / t, cfg.top_p).contiguous()
            t = 1.0
        rows, vocab, ld = _rows(logits, "sample")
        tok = torch.empty(rows, dtype=torch.int64, device=logits.device)
        lp = torch.empty(rows, dtype=torch.float32, device=logits.device)
        am = torch.empty(rows, dtype=torch.int64, device=logits.device)
        if rows:
            ws, tk = self._workspace(int(lib.pkv_sampling_workspace_bytes(rows, vocab)), rows)
            st = lib.pkv_sample_tokens(logits.data_ptr(), race.data_ptr() if race is not None else None, ld, rows,
                                       vocab, t if do_sample else 1.0, int(do_sample), self.seed,
                                       self._next_offset(), tok.data_ptr(), lp.data_ptr(), am.data_ptr(),
                                       tk.data_ptr(), ws.data_ptr(), ws.numel(), _stream_ptr())
            _lib.raise_for_status(st)
            self.launches += 1
        shape = logits.shape[:-1]
        return tok.view(shape), lp.view(shape), am.view(shape)

    # -- speculative decoding ---------------------------------------------------
    def spec_accept(self, target_logits: torch.Tensor, draft_logits: torch.Tensor, draft_tokens: torch.Tensor,
                    n_draft: torch.Tensor, *, draft_temperature: float = 1.0, do_sample: bool = False,
                    eos_token_id: int | None = None, uniforms: torch.Tensor | None = None):
        """Accept / reject a batch of speculative rounds (speculative.py:217-274).

        ``target_logits [n, k+1, vocab]``, ``draft_logits [n, k, vocab]`` (fp32,
        contiguous), ``draft_tokens [n, k]``, ``n_draft [n]`` valid drafts per
        sequence, ``uniforms [n, k]`` the acceptance draws (None: hashed from the
        sampler's seed).  Returns (tokens [n, k+1] int64, logprobs [n, k+1]
        fp32, n_out [n] int32, n_accepted [n] int32); tokens past n_out are -1.
        """
        if target_logits.dim() != 3 or draft_logits.dim() != 3:
            raise ValueError("spec_accept: target logits [n, k+1, vocab] and draft logits [n, k, vocab]")
        n, k1, vocab = target_logits.shape
        k = k1 - 1
        if draft_logits.shape != (n, k, vocab):
            raise ValueError("spec_accept: draft logits must be [n, k, vocab] for target logits [n, k+1, vocab]")
        for t, what in ((target_logits, "target"), (draft_logits, "draft")):
            if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError(f"spec_accept: {what} logits must be contiguous float32 CUDA tensors")
        dev = target_logits.device
        dtok = draft_tokens.to(device=dev, dtype=torch.int64).contiguous()
        nd = n_draft.to(device=dev, dtype=torch.int32).contiguous()
        if dtok.shape != (n, k) or nd.shape != (n,):
            raise ValueError("spec_accept: draft_tokens [n, k] and n_draft [n]")
        u = None
        if uniforms is not None:
            u = uniforms.to(device=dev, dtype=torch.float32).contiguous()
            if u.shape != (n, k):
                raise ValueError("spec_accept: uniforms [n, k]")
        tok = torch.empty((n, k1), dtype=torch.int64, device=dev)
        lp = torch.empty((n, k1), dtype=torch.float32, device=dev)
        n_out = torch.empty(n, dtype=torch.int32, device=dev)
        n_acc = torch.empty(n, dtype=torch.int32, device=dev)
        if n:
            ws, tk = self._workspace(int(lib.pkv_spec_workspace_bytes(n, k, vocab)), int(lib.pkv_spec_tickets(n, k)))
            st = lib.pkv_spec_accept(target_logits.data_ptr(), draft_logits.data_ptr(), vocab, dtok.data_ptr(),
                                     nd.data_ptr(), u.data_ptr() if u is not None else None, n, k, vocab,
                                     float(draft_temperature), int(bool(do_sample)),
                                     -1 if eos_token_id is None else int(eos_token_id), self.seed,
                                     self._next_offset(), tok.data_ptr(), lp.data_ptr(), n_out.data_ptr(),
                                     n_acc.data_ptr(), tk.data_ptr(), ws.data_ptr(), ws.numel(), _stream_ptr())
            _lib.raise_for_status(st)
            self.launches += 3
        return tok, lp, n_out, n_acc
