"""The reference's resident-cache decode step on the CPU (test / CPU-baseline infrastructure).

Restates what one decode step of AgentRL's paged-KV continuous loop does per
admitted sequence (agentrl/generation/continuous.py:465-497):

1. bucket sequences by identical length (continuous.py:452) and stack each
   bucket's resident caches along the batch (``_stack_dynamic_cache``,
   continuous.py:1090-1104) -- with ragged lengths almost every bucket is one
   sequence, so stacking is a no-op;
2. inside the model, append the step's K/V to the cache (``DynamicLayer.update``:
   ``torch.cat([keys, new], dim=-2)``, transformers cache_utils.py:119-120);
3. GQA attention of the single query over the whole cache (HF
   ``sdpa_attention_forward``, integrations/sdpa_attention.py:40-62);
4. split the batched cache back per sequence with ``.clone()``
   (``_split_dynamic_cache``, continuous.py:1106-1121);
5. ``PagedKVAllocator.append_tokens(seq, 1)`` (continuous.py:492-493).

Caches are held as float16 arrays (two bytes per element like the
reference's bf16 caches); the attention arithmetic is float32.  Buckets run
on a thread pool (numpy releases the GIL in its kernels), so the step uses
every host core it is given.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .allocator import OracleAllocator


class ResidentDecodeBatch:
    def __init__(self, lengths, num_q_heads: int, num_kv_heads: int, head_dim: int, seed: int = 0,
                 block_size: int = 16, total_blocks: int | None = None, threads: int = 1) -> None:
        rng = np.random.default_rng(seed)
        self.hq, self.hkv, self.d = num_q_heads, num_kv_heads, head_dim
        self.keys = [rng.standard_normal((num_kv_heads, n, head_dim), dtype=np.float32).astype(np.float16)
                     for n in lengths]
        self.values = [rng.standard_normal((num_kv_heads, n, head_dim), dtype=np.float32).astype(np.float16)
                       for n in lengths]
        need = sum(-(-(n + 4096) // block_size) for n in lengths)
        self.allocator = OracleAllocator(total_blocks or need, block_size)
        for i, n in enumerate(lengths):
            self.allocator.reserve(i, n)
        self.threads = threads
        self._pool = ThreadPoolExecutor(max_workers=threads) if threads > 1 else None

    def close(self) -> None:
        if self._pool is not None:
            self._pool.shutdown()

    def _one(self, i: int, q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray) -> np.ndarray:
        keys = np.concatenate([self.keys[i], k_new[:, None, :]], axis=1)  # DynamicLayer.update
        values = np.concatenate([self.values[i], v_new[:, None, :]], axis=1)
        group = self.hq // self.hkv
        out = np.empty((self.hq, self.d), dtype=np.float32)
        scale = np.float32(self.d ** -0.5)
        for h in range(self.hkv):
            kf = keys[h].astype(np.float32)
            vf = values[h].astype(np.float32)
            qh = q[h * group : (h + 1) * group].astype(np.float32)
            s = (qh @ kf.T) * scale
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            out[h * group : (h + 1) * group] = p @ vf
        self.keys[i] = keys.copy()  # _split_dynamic_cache: .clone()
        self.values[i] = values.copy()
        return out

    def step(self, indices, q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray) -> np.ndarray:
        """One decode step for ``indices``; q [n, Hq, D], k_new/v_new [n, Hkv, D]."""
        args = [(i, q[j], k_new[j], v_new[j]) for j, i in enumerate(indices)]
        if self._pool is None:
            outs = [self._one(*a) for a in args]
        else:
            outs = list(self._pool.map(lambda a: self._one(*a), args))
        for i in indices:
            self.allocator.append_tokens(i, 1)
        return np.stack(outs)

    def rollback(self, indices) -> None:
        """Drop the token the last step appended (keeps the workload's lengths stationary)."""
        for i in indices:
            self.keys[i] = self.keys[i][:, :-1]
            self.values[i] = self.values[i][:, :-1]
            self.allocator.truncate([i], [self.allocator.view(i).token_count - 1])



class TorchResidentDecodeBatch:
    """The same resident-cache decode step in the reference's own torch operations and dtype.

    bf16 caches ``[1, Hkv, T, D]`` per sequence; per step, sequences of equal
    length form a bucket (continuous.py:452) whose caches are stacked with
    ``torch.cat(dim=0)`` (``_stack_dynamic_cache``, continuous.py:1090-1104),
    the step's K/V is appended with ``torch.cat(dim=-2)`` (``DynamicLayer.update``,
    transformers cache_utils.py:119-120), the single query attends through
    ``scaled_dot_product_attention(..., enable_gqa=True)`` (the mask-free GQA branch
    of HF ``sdpa_attention_forward``, integrations/sdpa_attention.py:40-62), the
    batched cache is split back with ``.clone()`` per sequence
    (``_split_dynamic_cache``, continuous.py:1106-1121) and
    ``PagedKVAllocator.append_tokens(seq, 1)`` runs (continuous.py:492-493).
    Torch's intra-op threads carry the work (``torch.set_num_threads``).
    """

    def __init__(self, lengths, num_q_heads: int, num_kv_heads: int, head_dim: int, seed: int = 0,
                 block_size: int = 16, dtype=None) -> None:
        import torch

        self.torch = torch
        dtype = dtype or torch.bfloat16
        g = torch.Generator().manual_seed(seed)
        self.hq, self.hkv, self.d = num_q_heads, num_kv_heads, head_dim
        self.keys = [torch.randn((1, num_kv_heads, n, head_dim), generator=g).to(dtype) for n in lengths]
        self.values = [torch.randn((1, num_kv_heads, n, head_dim), generator=g).to(dtype) for n in lengths]
        need = sum(-(-(n + 4096) // block_size) for n in lengths)
        self.allocator = OracleAllocator(need, block_size)
        for i, n in enumerate(lengths):
            self.allocator.reserve(i, n)

    def step(self, indices, q, k_new, v_new):
        """One decode step; q [n, Hq, D], k_new / v_new [n, Hkv, D] (torch, the caches' dtype)."""
        torch = self.torch
        out = torch.empty(q.shape, dtype=q.dtype)
        buckets: dict[int, list[int]] = {}
        for j, i in enumerate(indices):
            buckets.setdefault(int(self.keys[i].shape[2]), []).append(j)
        for js in buckets.values():
            ii = [indices[j] for j in js]
            keys = torch.cat([self.keys[i] for i in ii], dim=0)
            values = torch.cat([self.values[i] for i in ii], dim=0)
            keys = torch.cat([keys, k_new[js].unsqueeze(2)], dim=-2)
            values = torch.cat([values, v_new[js].unsqueeze(2)], dim=-2)
            o = torch.nn.functional.scaled_dot_product_attention(q[js].unsqueeze(2), keys, values,
                                                                 scale=self.d ** -0.5, enable_gqa=True)
            out[js] = o[:, :, 0]
            for b, i in enumerate(ii):
                self.keys[i] = keys[b:b + 1].clone()
                self.values[i] = values[b:b + 1].clone()
        for i in indices:
            self.allocator.append_tokens(i, 1)
        return out

    def rollback(self, indices) -> None:
        """Drop the token the last step appended (keeps the workload's lengths stationary)."""
        for i in indices:
            self.keys[i] = self.keys[i][:, :, :-1]
            self.values[i] = self.values[i][:, :, :-1]
            self.allocator.truncate([i], [self.allocator.view(i).token_count - 1])


class TorchBlockStoreDecodeBatch(TorchResidentDecodeBatch):
    """The reference's block-store round trip for a decode step, in torch (bf16).

    Per sequence: ``read_sequence_legacy_cache`` (paged_kv.py:283-321: a scan of
    every stored key for the sequence's blocks, then ``torch.cat`` of its chunks
    and a trim), the step's K/V appended with ``torch.cat``, GQA SDPA, then
    ``append_tokens`` and ``write_sequence_cache`` of the grown cache
    (paged_kv.py:245-269: trim, ``split(block_size, dim=2)``, ``clone`` per block).
    """

    def __init__(self, lengths, num_q_heads: int, num_kv_heads: int, head_dim: int, seed: int = 0,
                 block_size: int = 16, dtype=None) -> None:
        super().__init__(lengths, num_q_heads, num_kv_heads, head_dim, seed, block_size, dtype)
        self._storage: dict = {}
        for i in range(len(lengths)):
            self._write(i, self.keys[i], self.values[i])
        self.keys = self.values = None

    def _write(self, i: int, keys, values) -> None:
        view = self.allocator.view(i)
        for state_index, tensor in enumerate((keys, values)):
            chunks = list(tensor[:, :, :view.token_count].split(view.block_size_tokens, dim=2))
            for block_id, chunk in zip(view.physical_blocks, chunks, strict=True):
                self._storage[(block_id, 0, state_index)] = chunk.clone()

    def _read(self, i: int):
        view = self.allocator.view(i)
        keys = [key for key in self._storage if key[0] in view.physical_blocks]
        states = sorted({k[2] for k in keys})
        return [self.torch.cat([self._storage[(b, 0, s)] for b in view.physical_blocks], dim=2)[:, :, :view.token_count]
                for s in states]

    def step(self, indices, q, k_new, v_new):
        torch = self.torch
        out = torch.empty(q.shape, dtype=q.dtype)
        for j, i in enumerate(indices):
            keys, values = self._read(i)
            keys = torch.cat([keys, k_new[j:j + 1].unsqueeze(2)], dim=-2)
            values = torch.cat([values, v_new[j:j + 1].unsqueeze(2)], dim=-2)
            o = torch.nn.functional.scaled_dot_product_attention(q[j:j + 1].unsqueeze(2), keys, values,
                                                                 scale=self.d ** -0.5, enable_gqa=True)
            out[j] = o[0, :, 0]
            self.allocator.append_tokens(i, 1)
            self._write(i, keys, values)
        return out

    def rollback(self, indices) -> None:
        for i in indices:
            self.allocator.truncate([i], [self.allocator.view(i).token_count - 1])
