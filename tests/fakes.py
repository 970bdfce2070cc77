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
    """With ``total_blocks`` it also keeps block accounting like the device allocator: blocks of
    ``block_size`` tokens, forks sharing them by refcount, a shared partial tail copied on the first
    append, and ``RuntimeError`` when no block is free."""

    def __init__(self, layers: int, total_blocks: int | None = None, block_size: int = 16):
        self.layers = layers
        self.kv = {}    # sid -> list per layer of [k [T,Hkv,D], v]
        self.count = {}
        self.block_size = block_size
        self.total_blocks = total_blocks
        self.blocks = {}  # sid -> list of block ids
        self.refs = {}    # block id -> refcount
        self._next_block = 0

    # -- block accounting (only with total_blocks) --
    @property
    def free_block_count(self):
        return None if self.total_blocks is None else self.total_blocks - len(self.refs)

    def _grow(self, sid):
        if self.total_blocks is None:
            return
        blocks, n, bs = self.blocks[sid], self.count[sid], self.block_size
        if n % bs != 0 and self.refs[blocks[-1]] > 1:
            self.refs[blocks[-1]] -= 1
            blocks[-1] = self._alloc()
        while len(blocks) < -(-(n + 1) // bs):
            blocks.append(self._alloc())

    def _alloc(self):
        if len(self.refs) >= self.total_blocks:
            raise RuntimeError("PagedKVAllocator ran out of free blocks.")
        b = self._next_block
        self._next_block += 1
        self.refs[b] = 1
        return b

    def _drop(self, blocks):
        for b in blocks:
            self.refs[b] -= 1
            if self.refs[b] == 0:
                del self.refs[b]

    def growth_blocks(self, ids):
        out = []
        for sid in ids:
            blocks, n, bs = self.blocks[sid], self.count[sid], self.block_size
            out.append(1 if len(blocks) < -(-(n + 1) // bs) or (n % bs != 0 and self.refs[blocks[-1]] > 1) else 0)
        return np.array(out, dtype=np.int32)

    def reserve(self, sid, n):
        assert sid not in self.count
        self.count[sid] = 0
        self.blocks[sid] = []
        for _ in range(n):
            self._grow(sid)
            self.count[sid] += 1
        self.kv[sid] = [[None, None] for _ in range(self.layers)]

    def append_tokens(self, sid, n):
        for _ in range(n):
            self._grow(sid)
            self.count[sid] += 1

    def fork(self, parent, child):
        self.count[child] = self.count[parent]
        self.kv[child] = [[k.clone(), v.clone()] for k, v in self.kv[parent]]
        self.blocks[child] = list(self.blocks[parent])
        for b in self.blocks[child]:
            self.refs[b] += 1

    def has_sequence(self, sid):
        return sid in self.count

    def token_count(self, sid):
        return self.count[sid]

    def truncate(self, ids, counts):
        for sid, n in zip(ids, counts):
            assert n <= self.count[sid]
            self.count[sid] = n
            keep = -(-n // self.block_size)
            if self.total_blocks is not None:
                self._drop(self.blocks[sid][keep:])
            del self.blocks[sid][keep:]
            for ent in self.kv[sid]:
                if ent[0] is not None:
                    ent[0], ent[1] = ent[0][:n], ent[1][:n]

    def release(self, sid):
        if self.total_blocks is not None:
            self._drop(self.blocks[sid])
        del self.count[sid], self.kv[sid], self.blocks[sid]

    def decode_step(self, ids):
        for s in ids:
            self._grow(s)
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
