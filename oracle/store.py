"""Oracle restatement of AgentRL's ``PagedKVCacheStore`` data path (test infrastructure).

Follows agentrl/generation/paged_kv.py:178-360.  Tensors are numpy arrays of
any dtype (bf16 travels as its uint16 bit pattern), so every comparison with
the device store is a bit comparison.  Storage is keyed ``(block, layer,
state)`` and holds the per-block chunk ``[1, Hkv, <=block_size, D]`` exactly as
paged_kv.py:259-269 stores it; the last chunk of a sequence is partial.

Extension (no reference counterpart): ``copy_block`` restates the
copy-on-write tail copy and ``append_token`` restates one decode-step append
into the paged layout (the reference appends by ``torch.cat`` into a resident
cache, transformers cache_utils.py:119-120, whose content the paged layout must
reproduce).
"""

from __future__ import annotations

import numpy as np

from .allocator import OracleAllocator


class OracleStore:
    def __init__(self, allocator: OracleAllocator) -> None:
        self.allocator = allocator
        self._storage: dict[tuple[int, int, int], np.ndarray] = {}

    def release(self, sequence_id: int) -> None:
        """paged_kv.py:205-213 (storage of blocks still shared by a fork is kept)."""
        view = self.allocator.view(sequence_id)
        self.allocator.release(sequence_id)
        for block_id in view.physical_blocks:
            if self.allocator.refcount(block_id) == 0:
                for key in [k for k in self._storage if k[0] == block_id]:
                    del self._storage[key]

    def write_sequence_cache(self, sequence_id: int, legacy_cache) -> None:
        """paged_kv.py:245-269: trim to token_count, split by block, clone per block."""
        view = self.allocator.view(sequence_id)
        token_count = view.token_count
        bs = view.block_size_tokens
        if token_count == 0:
            return
        for layer_index, layer_cache in enumerate(legacy_cache):
            for state_index, tensor in enumerate(layer_cache):
                trimmed = tensor[:, :, :token_count, ...]
                n = trimmed.shape[2]
                chunks = [trimmed[:, :, s : s + bs, ...] for s in range(0, n, bs)]
                if len(chunks) != view.logical_block_count:
                    raise ValueError(
                        "Cache chunk count does not match allocated block count "
                        f"for sequence {sequence_id}: {len(chunks)} vs {view.logical_block_count}."
                    )
                for block_id, chunk in zip(view.physical_blocks, chunks, strict=True):
                    self._storage[(block_id, layer_index, state_index)] = chunk.copy()

    def read_sequence_legacy_cache(self, sequence_id: int):
        """paged_kv.py:283-321 (block path): concatenate the chunks, trim to token_count."""
        view = self.allocator.view(sequence_id)
        keys = [k for k in self._storage if k[0] in view.physical_blocks]
        if not keys:
            raise LookupError("no stored blocks for this sequence")
        layers = []
        for layer_index in sorted({k[1] for k in keys}):
            states = []
            for state_index in sorted({k[2] for k in keys if k[1] == layer_index}):
                chunks = [self._storage[(b, layer_index, state_index)] for b in view.physical_blocks]
                states.append(np.concatenate(chunks, axis=2)[:, :, : view.token_count, ...])
            layers.append(tuple(states))
        return tuple(layers)

    def copy_block(self, src: int, dst: int) -> None:
        """Extension: the copy-on-write copy of a shared tail block."""
        for key in [k for k in self._storage if k[0] == src]:
            self._storage[(dst, key[1], key[2])] = self._storage[key].copy()

    def append_token(self, sequence_id: int, layer_index: int, k: np.ndarray, v: np.ndarray) -> None:
        """Extension: write one token ``k, v [Hkv, D]`` at position token_count - 1.

        The allocator's ``append_tokens(sequence_id, 1)`` must already have run.
        A block that receives its first token gets a chunk of one row, so the
        chunk layout stays the reference's (partial last chunk, paged_kv.py:262).
        """
        view = self.allocator.view(sequence_id)
        bs = view.block_size_tokens
        pos = view.token_count - 1
        block = view.physical_blocks[pos // bs]
        off = pos % bs
        for state_index, row in ((0, k), (1, v)):
            key = (block, layer_index, state_index)
            row4 = row[None, :, None, :]
            old = self._storage.get(key)
            if old is None or off == 0:
                self._storage[key] = row4.copy()
            else:
                self._storage[key] = np.concatenate([old[:, :, :off, :], row4], axis=2)
