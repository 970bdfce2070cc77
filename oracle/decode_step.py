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

