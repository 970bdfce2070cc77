"""CPU stand-in for the paged store (test infrastructure).

``FakeStore`` keeps every sequence's K/V per layer in plain fp32 tensors (with
copy-on-write forks as clones, truncation, releases and the decode-step
descriptor the real store returns) and attends with the oracle's arithmetic
(oracle/attention.py), so that the HF integration and the rollout loops can
be checked without a GPU.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle.attention import gqa_attention


@dataclass
class _FakeStep:
    host_lens: np.ndarray
    ids: list


class FakeStore:
    def __init__(self, layers: int):
        self.layers = layers
        self.kv = {}    # sid -> list per layer of [k [T,Hkv,D], v]
        self.count = {}

    def reserve(self, sid, n):
        assert sid not in self.count
        self.count[sid] = n
        self.kv[sid] = [[None, None] for _ in range(self.layers)]

    def append_tokens(self, sid, n):
        self.count[sid] += n

    def fork(self, parent, child):
        self.count[child] = self.count[parent]
        self.kv[child] = [[k.clone(), v.clone()] for k, v in self.kv[parent]]

    def has_sequence(self, sid):
        return sid in self.count

    def token_count(self, sid):
        return self.count[sid]

    def truncate(self, ids, counts):
        for sid, n in zip(ids, counts):
            assert n <= self.count[sid]
            self.count[sid] = n
            for ent in self.kv[sid]:
                if ent[0] is not None:
                    ent[0], ent[1] = ent[0][:n], ent[1][:n]

    def release(self, sid):
        del self.count[sid], self.kv[sid]

    def decode_step(self, ids):
        for s in ids:
            self.count[s] += 1
        return _FakeStep(np.array([self.count[s] for s in ids]), list(ids))

    def _append(self, sid, layer, k, v):
        ent = self.kv[sid][layer]
        ent[0] = k if ent[0] is None else torch.cat([ent[0], k])
        ent[1] = v if ent[1] is None else torch.cat([ent[1], v])
        assert ent[0].shape[0] == self.count[sid]

    def decode_attention(self, step, layer, q, k, v, scale=None):
        outs = []
        for i, sid in enumerate(step.ids):
            self._append(sid, layer, k[i:i + 1], v[i:i + 1])
            kk, vv = self.kv[sid][layer]
            o = gqa_attention(q[i:i + 1].numpy(), kk.numpy(), vv.numpy(), scale, past=kk.shape[0] - 1)
            outs.append(torch.from_numpy(o))
        return torch.cat(outs).to(q.dtype)

    def prefill_attention(self, ids, q, k, v, q_lens=None, layer=0, scale=None, step=None):
        outs, off = [], 0
        for sid, n in zip(ids, q_lens):
            n = int(n)
            self._append(sid, layer, k[off:off + n], v[off:off + n])
            kk, vv = self.kv[sid][layer]
            past = kk.shape[0] - n
            o = gqa_attention(q[off:off + n].numpy(), kk.numpy(), vv.numpy(), scale, past=past)
            outs.append(torch.from_numpy(o))
            off += n
        return torch.cat(outs).to(q.dtype)
