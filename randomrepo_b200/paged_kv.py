"""Drop-in paged-KV allocator and store over libpkv_b200.

The classes keep the names, signatures, properties, metric keys, exceptions
and messages of AgentRL's ``agentrl/generation/paged_kv.py`` so that the
continuous-batching loop, the scheduler admission code and the telemetry
that call them run unchanged:

* ``PagedKVSequenceView`` -- paged_kv.py:11-22;
* ``PagedKVAllocator`` -- paged_kv.py:25-175, here a handle to the C++ block
  allocator (lowest free id first, so block tables equal the reference's);
* ``PagedKVCacheStore`` -- paged_kv.py:178-360, here backed by one device KV
  pool per store instead of a dict of cloned per-block tensors.

Additions that the reference does not have: ``fork`` (copy-on-write sharing of
a sequence's blocks, for the members of a GRPO group that share one prompt),
and the device decode path (``decode_step`` + ``decode_attention``) that
appends each step's K/V into the pages and runs paged GQA attention on them.
"""

from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from . import _lib
from ._lib import lib
from . import device as _device
from .device import KVPool, PrefillPlan, plan_prefill, plan_verify, verify_supported


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_stream(device: torch.device) -> int:
    """Raw cudaStream_t of the current torch stream on ``device``."""
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


class _on_device:
    """Make ``device`` current only if it is not (the common case costs one query)."""

    __slots__ = ("_device", "_prev")

    def __init__(self, device: torch.device) -> None:
        self._device = device
        self._prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self._device.index:
            self._prev = cur
            torch.cuda.set_device(self._device)
        return self

    def __exit__(self, *exc) -> None:
        if self._prev is not None:
            torch.cuda.set_device(self._prev)


def _is_i64_vector(a) -> bool:
    return type(a) is np.ndarray and a.dtype == np.int64 and a.ndim == 1 and a.flags.c_contiguous


class _PointerCache:
    """Data addresses of the int64 index arrays a decode loop hands over every step (usually the
    same array objects): ``ndarray.ctypes.data`` costs about a microsecond per call.  Entries keep
    their array alive, so an address stays valid while it is cached; at most 16 are kept."""

    __slots__ = ("_entries",)

    def __init__(self) -> None:
        self._entries: dict[int, tuple[np.ndarray, int]] = {}

    def __call__(self, a: np.ndarray) -> int:
        e = self._entries.get(id(a))
        if e is not None and e[0] is a:
            return e[1]
        if len(self._entries) >= 16:
            self._entries.clear()
        ptr = a.ctypes.data
        self._entries[id(a)] = (a, ptr)
        return ptr


@dataclass(frozen=True, slots=True)
class PagedKVSequenceView:
    """Read-only sequence mapping inside the paged-KV allocator (paged_kv.py:11-22)."""

    sequence_id: int
    token_count: int
    block_size_tokens: int
    physical_blocks: tuple[int, ...]

    @property
    def logical_block_count(self) -> int:
        return len(self.physical_blocks)


class PagedKVAllocator:
    """Fixed pool of equal blocks with a per-sequence block table (paged_kv.py:25-175).

    Allocation pops the lowest free block id; a release returns a sequence's
    blocks (a block shared by forks returns when its last owner releases it).
    """

    def __init__(self, total_blocks: int, block_size_tokens: int) -> None:
        status = ctypes.c_int32(0)
        handle = lib.pkv_allocator_create(int(total_blocks), int(block_size_tokens), ctypes.byref(status))
        if not handle:
            _lib.raise_for_status(status.value)
        self._handle = handle
        self.total_blocks = int(total_blocks)
        self.block_size_tokens = int(block_size_tokens)
        self._view_buf = np.zeros(64, dtype=np.int32)
        self._ptr = _PointerCache()
        weakref.finalize(self, lib.pkv_allocator_destroy, handle)

    def _stats(self) -> _lib.AllocatorStats:
        st = _lib.AllocatorStats()
        lib.pkv_allocator_get_stats(self._handle, ctypes.byref(st))
        return st

    # paged_kv.py:50-76
    @property
    def free_block_count(self) -> int:
        return int(self._stats().free_block_count)

    @property
    def used_block_count(self) -> int:
        return int(self._stats().used_block_count)

    @property
    def block_reuse_count(self) -> int:
        return int(self._stats().block_reuse_count)

    @property
    def max_blocks_in_use(self) -> int:
        return int(self._stats().max_blocks_in_use)

    @property
    def resident_sequence_count(self) -> int:
        return int(self._stats().resident_sequence_count)

    @property
    def allocator_occupancy(self) -> float:
        return self.used_block_count / self.total_blocks

    @property
    def allocator_pressure(self) -> float:
        return self.allocator_occupancy

    def reserve(self, sequence_id: int, token_count: int) -> PagedKVSequenceView:
        """Reserve enough blocks for a fresh sequence (paged_kv.py:78-91)."""
        _lib.raise_for_status(lib.pkv_allocator_reserve(self._handle, int(sequence_id), int(token_count)))
        return self.view(sequence_id)

    def append_tokens(self, sequence_id: int, token_count: int) -> PagedKVSequenceView:
        """Grow a sequence by the provided number of tokens (paged_kv.py:93-110)."""
        _lib.raise_for_status(lib.pkv_allocator_append_tokens(self._handle, int(sequence_id), int(token_count)))
        return self.view(sequence_id)

    def release(self, sequence_id: int) -> None:
        """Release all blocks owned by one sequence (paged_kv.py:112-120)."""
        _lib.raise_for_status(lib.pkv_allocator_release(self._handle, int(sequence_id)))

    def fork(self, parent_id: int, child_id: int) -> PagedKVSequenceView:
        """Share all of ``parent_id``'s blocks with a new sequence ``child_id``.

        No reference counterpart.  The child's first append into a shared,
        partially filled tail block gets a private copy of that block first.
        """
        _lib.raise_for_status(lib.pkv_allocator_fork(self._handle, int(parent_id), int(child_id)))
        return self.view(child_id)

    def logical_to_physical(self, sequence_id: int, logical_block_index: int) -> int:
        """Resolve one logical block index to its physical block id (paged_kv.py:122-127)."""
        out = ctypes.c_int64()
        st = lib.pkv_allocator_logical_to_physical(self._handle, int(sequence_id), int(logical_block_index),
                                                   ctypes.byref(out))
        _lib.raise_for_status(st, key=sequence_id)
        return int(out.value)

    def view(self, sequence_id: int) -> PagedKVSequenceView:
        """Return a read-only snapshot for one sequence (paged_kv.py:129-139)."""
        count = ctypes.c_int64()
        n = ctypes.c_int64()
        buf = self._view_buf
        st = lib.pkv_allocator_view(self._handle, int(sequence_id), ctypes.byref(count), buf.ctypes.data,
                                    buf.size, ctypes.byref(n))
        _lib.raise_for_status(st)
        if n.value > buf.size:
            self._view_buf = buf = np.zeros(max(n.value, 2 * buf.size), dtype=np.int32)
            lib.pkv_allocator_view(self._handle, int(sequence_id), ctypes.byref(count), buf.ctypes.data, buf.size,
                                   ctypes.byref(n))
        return PagedKVSequenceView(
            sequence_id=sequence_id,
            token_count=int(count.value),
            block_size_tokens=self.block_size_tokens,
            physical_blocks=tuple(int(b) for b in buf[: n.value]),
        )

    def metrics(self) -> dict[str, float]:
        """Allocator metrics for runtime reporting (paged_kv.py:141-152)."""
        st = self._stats()
        occupancy = st.used_block_count / self.total_blocks
        return {
            "paged_kv_free_block_count": float(st.free_block_count),
            "paged_kv_used_block_count": float(st.used_block_count),
            "paged_kv_allocator_occupancy": float(occupancy),
            "paged_kv_block_reuse_count": float(st.block_reuse_count),
            "paged_kv_allocator_pressure": float(occupancy),
            "paged_kv_max_blocks_in_use": float(st.max_blocks_in_use),
            "paged_kv_resident_sequences": float(st.resident_sequence_count),
        }

    def has_sequence(self, sequence_id: int) -> bool:
        """Whether the allocator still tracks the sequence (paged_kv.py:154-157)."""
        return bool(lib.pkv_allocator_has_sequence(self._handle, int(sequence_id)))

    # -- extension ------------------------------------------------------------
    def truncate(self, sequence_ids, token_counts) -> None:
        """Shrink each sequence to its token count, releasing blocks past the end.

        No reference counterpart: it rolls back rejected speculative drafts.
        """
        if _is_i64_vector(sequence_ids) and _is_i64_vector(token_counts):
            ids, counts = sequence_ids, token_counts
            p_ids, p_counts = self._ptr(ids), self._ptr(counts)
        else:
            ids = np.ascontiguousarray(np.atleast_1d(np.asarray(sequence_ids, dtype=np.int64)))
            counts = np.ascontiguousarray(np.atleast_1d(np.asarray(token_counts, dtype=np.int64)))
            p_ids, p_counts = ids.ctypes.data, counts.ctypes.data
        if ids.shape != counts.shape:
            raise ValueError("sequence_ids and token_counts must have the same length")
        _lib.raise_for_status(lib.pkv_allocator_truncate(self._handle, p_ids, p_counts, ids.size))

    def append_many(self, sequence_ids, token_counts) -> None:
        """``append_tokens(sid, n)`` for each pair, in order, without building the views it returns."""
        h = self._handle
        for sid, n in zip(sequence_ids, token_counts):
            _lib.raise_for_status(lib.pkv_allocator_append_tokens(h, int(sid), int(n)))

    def token_counts(self, sequence_ids) -> np.ndarray:
        """Token counts of several sequences (int64), without building their views."""
        ids = np.ascontiguousarray(np.atleast_1d(np.asarray(sequence_ids, dtype=np.int64)))
        out = np.empty(ids.size, dtype=np.int64)
        _lib.raise_for_status(lib.pkv_allocator_token_counts(self._handle, ids.ctypes.data, ids.size,
                                                             out.ctypes.data))
        return out

    def growth_blocks(self, sequence_ids) -> np.ndarray:
        """Free blocks one more token takes for each sequence (int32 0 / 1): a new block at a block
        boundary, or the copy-on-write copy of a partial tail block that forks still share.
        No reference counterpart (the reference's admission tests len % block_size == 0 only,
        agentrl/generation/continuous.py:915-919, and has no forks)."""
        ids = np.ascontiguousarray(np.atleast_1d(np.asarray(sequence_ids, dtype=np.int64)))
        out = np.empty(ids.size, dtype=np.int32)
        _lib.raise_for_status(lib.pkv_allocator_growth_blocks(self._handle, ids.ctypes.data, ids.size,
                                                              out.ctypes.data))
        return out

    def refcount(self, block_id: int) -> int:
        out = ctypes.c_int32()
        _lib.raise_for_status(lib.pkv_allocator_refcount(self._handle, int(block_id), ctypes.byref(out)))
        return int(out.value)

    def row(self, sequence_id: int) -> int:
        """Row of the sequence in the device block table."""
        out = ctypes.c_int32()
        _lib.raise_for_status(lib.pkv_allocator_row(self._handle, int(sequence_id), ctypes.byref(out)))
        return int(out.value)

    @property
    def shared_block_count(self) -> int:
        return int(self._stats().shared_block_count)


@dataclass
class DecodeStep:
    """One decode step (one token appended per sequence) as uploaded to the device.

    ``info`` is the native step descriptor (device pointers to the table rows,
    token counts, new blocks, work items and slots of the step); it is valid
    until the store's next ``decode_step``.  ``host_rows`` / ``host_lens`` are
    the same rows and token counts on the host.
    """

    sequence_ids: np.ndarray
    info: _lib.StepInfo
    serial: int
    host_rows: np.ndarray
    host_lens: np.ndarray
    committed: bool = False

    @property
    def batch(self) -> int:
        return int(self.info.batch)

    @property
    def n_items(self) -> int:
        return int(self.info.n_items)

    @property
    def pages_per_split(self) -> int:
        return int(self.info.pages_per_split)


@dataclass
class PrefillStep:
    """One prefill / verify forward's layout on the device, shared by every layer.

    Sequence i's chunk is its last ``q_lens[i]`` tokens; ``slots`` are the pool
    slots of the chunks' tokens (packed in ``sequence_ids`` order) and
    ``records`` the uploaded work items of ``plan``.
    """

    sequence_ids: np.ndarray
    q_lens: np.ndarray
    num_q_heads: int
    total_q: int
    plan: PrefillPlan | None
    slots: torch.Tensor | None
    records: torch.Tensor | None


def host_input_tensor(shape, dtype: torch.dtype, *, write_combined: bool = True) -> torch.Tensor:
    """A CPU tensor in page-locked host memory from ``pkv_host_alloc``, for the q / k / v a host
    hands to ``PagedKVCacheStore.decode``: write-combined by default, which the GPU reads over
    PCIe without snooping the host's caches (about twice the host-to-device bandwidth of
    cacheable page-locked memory on the hosts measured here).  Reading it back on the host is
    slow; keep outputs in ordinary page-locked memory.  Freed when the tensor is collected."""
    n = 1
    for x in shape:
        n *= int(x)
    itemsize = torch.empty((), dtype=dtype).element_size()
    nbytes = max(1, n * itemsize)
    ptr = ctypes.c_void_p()
    _lib.raise_for_status(lib.pkv_host_alloc(nbytes, 1 if write_combined else 0, ctypes.byref(ptr)))
    raw = (ctypes.c_char * nbytes).from_address(ptr.value)
    t = torch.frombuffer(raw, dtype=torch.uint8)[: n * itemsize].view(dtype).view(*shape)
    weakref.finalize(raw, lib.pkv_host_free, ptr.value)  # runs once no tensor over ``raw`` is left
    return t


class PagedKVCacheStore:
    """Block-backed KV store (paged_kv.py:178-360) on a device KV pool.

    The pool is created on the first write from the cache's geometry (layers,
    KV heads, head dim, dtype, device), or up front when all of
    ``num_layers``, ``num_kv_heads``, ``head_dim`` and ``dtype`` are given.
    Reads return new tensors on the device the sequence was written from.
    """

    def __init__(self, allocator: PagedKVAllocator, *, num_layers: int | None = None,
                 num_kv_heads: int | None = None, head_dim: int | None = None, dtype: torch.dtype | None = None,
                 device: torch.device | str | int | None = None) -> None:
        self.allocator = allocator
        self._cache_templates: dict[int, Any] = {}
        self._resident_caches: dict[int, Any] = {}
        self._io_device: dict[int, torch.device] = {}
        # Tokens stored in each block's chunk (-1: the block holds no stored chunk).
        self._block_fill = np.full(allocator.total_blocks, -1, dtype=np.int32)
        self._pool: KVPool | None = None
        # Host buffers of the decode fast path, reused from step to step.
        self._host3: np.ndarray | None = None
        self._host3_ptrs = (0, 0, 0)
        self._io_checked: tuple = ()
        if None not in (num_layers, num_kv_heads, head_dim, dtype):
            self._pool = self._new_pool(num_layers, num_kv_heads, head_dim, dtype, device)

    # -- reference API (paged_kv.py:192-216) ------------------------------------
    @property
    def resident_sequence_count(self) -> int:
        return self.allocator.resident_sequence_count

    @property
    def pool(self) -> KVPool | None:
        return self._pool

    def reserve(self, sequence_id: int, token_count: int) -> PagedKVSequenceView:
        return self.allocator.reserve(sequence_id, token_count)

    def append_tokens(self, sequence_id: int, token_count: int) -> PagedKVSequenceView:
        return self.allocator.append_tokens(sequence_id, token_count)

    def has_sequence(self, sequence_id: int) -> bool:
        return self.allocator.has_sequence(sequence_id)

    def token_count(self, sequence_id: int) -> int:
        """Tokens the sequence holds (KeyError if unknown)."""
        return int(self.allocator.token_counts([sequence_id])[0])

    def token_counts(self, sequence_ids) -> np.ndarray:
        """Tokens each sequence holds (KeyError for an unknown id)."""
        return self.allocator.token_counts(sequence_ids)

    def append_many(self, sequence_ids, token_counts) -> None:
        """``append_tokens`` for each (sequence, count) pair, in order, without returning views."""
        self.allocator.append_many(sequence_ids, token_counts)

    @property
    def free_block_count(self) -> int:
        return self.allocator.free_block_count

    def growth_blocks(self, sequence_ids) -> np.ndarray:
        """Free blocks each sequence's next token takes (``PagedKVAllocator.growth_blocks``)."""
        return self.allocator.growth_blocks(sequence_ids)

    def release(self, sequence_id: int) -> None:
        """paged_kv.py:205-213: drop the resident cache, the stored blocks and the table."""
        view = self.allocator.view(sequence_id)
        self._resident_caches.pop(sequence_id, None)
        self._cache_templates.pop(sequence_id, None)
        self._io_device.pop(sequence_id, None)
        self.allocator.release(sequence_id)
        for block_id in view.physical_blocks:
            if self.allocator.refcount(block_id) == 0:
                self._block_fill[block_id] = -1

    def metrics(self) -> dict[str, float]:
        return self.allocator.metrics()

    # -- resident caches (paged_kv.py:218-243) ------------------------------------
    # Restated from agentrl/generation/paged_kv.py:218-243: plain dict bookkeeping whose
    # behaviour, names and messages the drop-in contract fixes, kept statement for statement.
    def cache_template(self, sequence_id: int) -> Any:
        return self._cache_templates[sequence_id]

    def set_resident_cache(self, sequence_id: int, cache: Any, cache_template: Any | None = None) -> None:
        if not self.allocator.has_sequence(sequence_id):
            raise KeyError(f"Unknown sequence_id {sequence_id}.")
        self._resident_caches[sequence_id] = cache
        if cache_template is not None:
            self._cache_templates[sequence_id] = cache_template

    def resident_cache(self, sequence_id: int) -> Any:
        return self._resident_caches[sequence_id]

    def has_resident_cache(self, sequence_id: int) -> bool:
        return sequence_id in self._resident_caches

    def clear_resident_cache(self, sequence_id: int) -> None:
        resident_cache = self._resident_caches.get(sequence_id)
        if resident_cache is not None and self.allocator.has_sequence(sequence_id):
            cache_template = self._cache_templates.get(sequence_id, resident_cache)
            self.write_sequence_cache(
                sequence_id=sequence_id,
                legacy_cache=self._as_legacy_cache(resident_cache, sequence_id),
                cache_template=cache_template,
            )
        self._resident_caches.pop(sequence_id, None)

    # -- block storage (paged_kv.py:245-347) --------------------------------------
    # The block write and gather run on the device kernels; the resident / template branches of
    # read_sequence_legacy_cache, write_batched_legacy_cache and the _stack / _split helpers are
    # restated from agentrl/generation/paged_kv.py:271-281, 287-303 and 335-360 (tuple plumbing
    # whose results the drop-in contract fixes).
    def write_sequence_cache(self, sequence_id: int, legacy_cache: tuple[tuple[torch.Tensor, ...], ...],
                             cache_template: Any) -> None:
        """paged_kv.py:245-269: trim to token_count, split into blocks, store each block's chunk."""
        view = self.allocator.view(sequence_id)
        token_count = view.token_count
        bs = view.block_size_tokens
        self._cache_templates[sequence_id] = cache_template
        if token_count == 0:
            return
        n_written = None
        for layer_cache in legacy_cache:
            for tensor in layer_cache:
                n = int(tensor[:, :, :token_count, ...].shape[2])
                chunks = max(1, -(-n // bs))
                if chunks != view.logical_block_count:
                    raise ValueError(
                        "Cache chunk count does not match allocated block count "
                        f"for sequence {sequence_id}: {chunks} vs {view.logical_block_count}."
                    )
                if n_written is not None and n != n_written:
                    raise ValueError("every layer and state of a sequence cache must hold the same token count")
                n_written = n
        first = legacy_cache[0][0]
        if any(len(layer) != 2 for layer in legacy_cache):
            raise ValueError("the paged pool stores (key, value) pairs per layer")
        pool = self._ensure_pool(len(legacy_cache), first.shape[1], first.shape[3], first.dtype, first.device)
        self._io_device[sequence_id] = first.device
        if n_written:
            src = torch.stack([torch.stack([layer[0][0, :, :n_written], layer[1][0, :, :n_written]])
                               for layer in legacy_cache]).to(pool.device)
            slots = self._slots(view.physical_blocks, [min(bs, n_written - j * bs)
                                                       for j in range(view.logical_block_count)], bs)
            self._sync()
            pool.scatter(0, src[:, 0], src[:, 1], slots)
        for j, block_id in enumerate(view.physical_blocks):
            self._block_fill[block_id] = max(0, min(bs, (n_written or 0) - j * bs))

    def write_batched_legacy_cache(self, sequence_ids: list[int], legacy_cache: tuple[tuple[torch.Tensor, ...], ...],
                                   cache_template: Any) -> None:
        """paged_kv.py:271-281."""
        split_caches = self._split_legacy_cache(legacy_cache)
        if len(split_caches) != len(sequence_ids):
            raise ValueError("Batched legacy cache does not match the number of sequence ids.")
        for sequence_id, sequence_cache in zip(sequence_ids, split_caches, strict=True):
            self.write_sequence_cache(sequence_id, sequence_cache, cache_template)

    def read_sequence_legacy_cache(self, sequence_id: int) -> tuple[tuple[torch.Tensor, ...], ...]:
        """paged_kv.py:283-321: resident cache, else the stored blocks, else the template."""
        view = self.allocator.view(sequence_id)
        token_count = view.token_count
        resident_cache = self._resident_caches.get(sequence_id)
        if resident_cache is not None:
            legacy_cache = self._as_legacy_cache(resident_cache, sequence_id)
            return tuple(
                tuple(tensor[:, :, :token_count, ...].clone() for tensor in layer_cache)
                for layer_cache in legacy_cache
            )
        fills = self._block_fill[list(view.physical_blocks)] if view.physical_blocks else np.zeros(0, np.int32)
        if self._pool is None or not (fills >= 0).any():
            legacy_template = self._as_legacy_cache(self._cache_templates[sequence_id], sequence_id)
            return tuple(
                tuple(tensor[:, :, :token_count, ...].clone() for tensor in layer_template)
                for layer_template in legacy_template
            )
        missing = np.flatnonzero(fills < 0)
        if missing.size:
            raise KeyError((view.physical_blocks[int(missing[0])], 0, 0))
        n = min(int(fills.sum()), token_count)
        return self._gather_legacy(view.physical_blocks, fills, n, self._io_device.get(sequence_id))

    def read_batched_legacy_cache(self, sequence_ids: list[int]) -> tuple[tuple[torch.Tensor, ...], ...]:
        """paged_kv.py:331-333."""
        sequence_caches = [self.read_sequence_legacy_cache(sequence_id) for sequence_id in sequence_ids]
        return self._stack_legacy_cache(sequence_caches)

    @staticmethod
    def _as_legacy_cache(cache: Any, sequence_id: int) -> tuple[tuple[torch.Tensor, ...], ...]:
        """paged_kv.py:323-329."""
        if isinstance(cache, tuple):
            return cache
        if hasattr(cache, "to_legacy_cache"):
            return cache.to_legacy_cache()
        layers = getattr(cache, "layers", None)
        if layers is not None and all(hasattr(layer, "keys") and hasattr(layer, "values") for layer in layers):
            # transformers >= 5 caches dropped to_legacy_cache; their layers hold keys/values.
            return tuple((layer.keys, layer.values) for layer in layers)
        raise TypeError(f"Unsupported cache template for sequence {sequence_id}: {type(cache)!r}")

    @staticmethod
    def _stack_legacy_cache(caches: list[tuple[tuple[torch.Tensor, ...], ...]]) -> tuple[tuple[torch.Tensor, ...], ...]:
        """paged_kv.py:335-347."""
        stacked_layers = []
        for layer_caches in zip(*caches, strict=True):
            stacked_layers.append(tuple(torch.cat(items, dim=0) for items in zip(*layer_caches, strict=True)))
        return tuple(stacked_layers)

    @staticmethod
    def _split_legacy_cache(cache: tuple[tuple[torch.Tensor, ...], ...]) -> list[tuple[tuple[torch.Tensor, ...], ...]]:
        """paged_kv.py:349-360."""
        batch_size = cache[0][0].shape[0]
        return [
            tuple(tuple(state[batch_index : batch_index + 1] for state in layer_cache) for layer_cache in cache)
            for batch_index in range(batch_size)
        ]

    # -- copy-on-write fork (extension) ----------------------------------------
    def fork(self, parent_id: int, child_id: int) -> PagedKVSequenceView:
        """Give ``child_id`` the parent's blocks (shared, copy-on-write) and cache template."""
        view = self.allocator.fork(parent_id, child_id)
        if parent_id in self._cache_templates:
            self._cache_templates[child_id] = self._cache_templates[parent_id]
        if parent_id in self._io_device:
            self._io_device[child_id] = self._io_device[parent_id]
        return view

    def truncate(self, sequence_ids, token_counts) -> None:
        """Shrink sequences (see ``PagedKVAllocator.truncate``); stored chunks are trimmed to match."""
        ids = np.ascontiguousarray(np.atleast_1d(np.asarray(sequence_ids, dtype=np.int64)))
        counts = np.ascontiguousarray(np.atleast_1d(np.asarray(token_counts, dtype=np.int64)))
        if ids.shape != counts.shape:
            raise ValueError("sequence_ids and token_counts must have the same length")
        # One native pass: the blocks past each new end are released, a freed
        # block's fill becomes -1 and a new partial tail keeps what it still holds.
        fill = self._block_fill
        _lib.raise_for_status(lib.pkv_allocator_truncate_fill(self.allocator._handle, ids.ctypes.data,
                                                              counts.ctypes.data, ids.size, fill.ctypes.data,
                                                              fill.size))

    # -- device decode path (extension) -----------------------------------------
    def decode(self, sequence_ids, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, *, layer: int = 0,
               scale: float | None = None, out: torch.Tensor | None = None) -> tuple[torch.Tensor, DecodeStep]:
        """One decode step and its fused append + paged attention for one layer, in one native call.

        Equivalent to ``decode_step(sequence_ids)`` followed by
        ``decode_attention(step, layer, q, k_new, v_new)``; the returned step
        serves the model's other layers.

        With q / k_new / v_new (and ``out``, if given) in host memory the step
        runs through ``pkv_stepper_step_host``: the stepper copies the inputs
        in and the output back out on streams of its own, overlapped with the
        neighbouring steps' kernels (pinned tensors for the copies to be
        asynchronous).  ``out`` is then complete only after
        ``wait_host_outputs()``; the inputs must not change until then.
        """
        pool = self._pool if self._pool is not None else self._require_pool()
        ids = sequence_ids
        if _is_i64_vector(ids) and ids.size:
            p_ids = self.allocator._ptr(ids)
        else:
            ids = self._step_ids(sequence_ids)
            p_ids = ids.ctypes.data
        n = ids.size
        if q.device.type == "cpu":
            return self._decode_host(pool, ids, p_ids, n, q, k_new, v_new, layer, scale, out)
        # The checks of q / k / v / out are skipped when the same tensor
        # objects come back (a decode loop reusing its buffers).
        chk = self._io_checked
        if (out is None or not chk or chk[0] is not q or chk[1] is not k_new or chk[2] is not v_new
                or chk[3] is not out or chk[4] != n):
            out = self._check_decode_io(pool, n, q, k_new, v_new, out)
            self._io_checked = (q, k_new, v_new, out, n, False)
        host, (p_rows, p_lens, p_tokb) = self._host_buffers(n)
        info = _lib.StepInfo()
        with _on_device(pool.device):
            stream = _current_stream(pool.device)
            sc = float(scale if scale is not None else pool.head_dim ** -0.5)
            st = lib.pkv_stepper_step(pool.stepper, p_ids, n, int(layer), q.data_ptr(), k_new.data_ptr(),
                                      v_new.data_ptr(), q.shape[1], sc, out.data_ptr(), stream, ctypes.byref(info),
                                      p_rows, p_lens, p_tokb, None, 0)
            if st != _lib.PKV_OK and self._needs_retry(pool, st, info):
                st = self._upload_retry(pool, stream, info, st)
                if st == _lib.PKV_OK:
                    st = lib.pkv_stepper_attention(pool.stepper, int(layer), q.data_ptr(), k_new.data_ptr(),
                                                   v_new.data_ptr(), q.shape[1], sc, out.data_ptr(), stream)
        step = self._finish_step(pool, st, ids, info, host)
        step.committed = True
        return out, step

    @staticmethod
    def _needs_retry(pool: KVPool, st: int, info) -> bool:
        """A step that failed only for want of table room or of fixed-step work-item capacity."""
        return st == _lib.PKV_ERR_CAPACITY or (st == _lib.PKV_ERR_UNSUPPORTED and info.need_items > 0)

    @staticmethod
    def _upload_retry(pool: KVPool, stream: int, info, st: int) -> int:
        """Make the room a begun step asked for, then upload it again (until it fits or fails otherwise)."""
        for _ in range(4):
            if st == _lib.PKV_ERR_CAPACITY:
                pool.grow(info.need_rows, info.need_cols)
            elif st == _lib.PKV_ERR_UNSUPPORTED and info.need_items > 0:
                # Fixed-step mode: a new block with room for the step (graphs
                # recorded on the old one are dropped by their owners).
                pool.fix_steps(pool.fixed_batch, max_items=int(info.need_items * 5 // 4 + 64))
            else:
                return st
            info.need_items = 0
            st = lib.pkv_stepper_upload(pool.stepper, stream, ctypes.byref(info), None, 0)
        return st

    def _decode_host(self, pool: KVPool, ids, p_ids: int, n: int, q, k_new, v_new, layer: int, scale, out):
        """``decode`` with host tensors: inputs staged and output returned by the native stepper."""
        chk = self._io_checked
        if (out is None or not chk or chk[0] is not q or chk[1] is not k_new or chk[2] is not v_new
                or chk[3] is not out or chk[4] != n):
            if k_new is None or v_new is None:
                raise ValueError("a host-tensor decode step needs k_new and v_new")
            out = self._check_decode_io(pool, n, q, k_new, v_new, out, device=torch.device("cpu"))
            # One copy moves q, k and v only when they are consecutive parts of one allocation.
            base = q.untyped_storage().data_ptr()
            packed = (k_new.untyped_storage().data_ptr() == base and v_new.untyped_storage().data_ptr() == base
                      and k_new.data_ptr() == q.data_ptr() + q.nbytes
                      and v_new.data_ptr() == k_new.data_ptr() + k_new.nbytes)
            self._io_checked = (q, k_new, v_new, out, n, packed)
        host, (p_rows, p_lens, p_tokb) = self._host_buffers(n)
        info = _lib.StepInfo()
        with _on_device(pool.device):
            stream = _current_stream(pool.device)
            sc = float(scale if scale is not None else pool.head_dim ** -0.5)
            st = lib.pkv_stepper_step_host(pool.stepper, p_ids, n, int(layer), q.data_ptr(), k_new.data_ptr(),
                                           v_new.data_ptr(), int(self._io_checked[5]), q.shape[1], sc,
                                           out.data_ptr(), stream, ctypes.byref(info), p_rows, p_lens, p_tokb)
            if st != _lib.PKV_OK and self._needs_retry(pool, st, info):
                st = self._upload_retry(pool, stream, info, st)
                if st == _lib.PKV_OK:
                    st = lib.pkv_stepper_attention_host(pool.stepper, int(layer), q.shape[1], sc, out.data_ptr(),
                                                        stream)
        step = self._finish_step(pool, st, ids, info, host)
        step.committed = True
        return out, step

    def wait_host_outputs(self) -> None:
        """Block until the outputs of every host-tensor ``decode`` issued so far are in host memory."""
        pool = self._require_pool()
        with _on_device(pool.device):
            _lib.raise_for_status(lib.pkv_stepper_host_fence(pool.stepper, _current_stream(pool.device)))
            torch.cuda.current_stream(pool.device).synchronize()

    def fence_host_outputs(self) -> None:
        """Make the current stream wait for the output copies of the host-tensor steps issued so far."""
        pool = self._require_pool()
        with _on_device(pool.device):
            _lib.raise_for_status(lib.pkv_stepper_host_fence(pool.stepper, _current_stream(pool.device)))

    def _host_buffers(self, n: int):
        """Rows / lengths / token blocks [3, n] for the stepper to fill, and their addresses (reused)."""
        buf = self._host3
        if buf is None or buf.shape[1] < n:
            cap = max(n, 256)
            buf = self._host3 = np.empty((3, cap), dtype=np.int32)
            base = buf.ctypes.data
            self._host3_ptrs = (base, base + 4 * cap, base + 8 * cap)
        return buf[:, :n], self._host3_ptrs

    def decode_step(self, sequence_ids) -> DecodeStep:
        """Append one token to each sequence and upload the step for the decode kernels.

        The allocator side equals calling ``append_tokens(seq, 1)`` for each id in
        order (agentrl/generation/continuous.py:492-493); the host work runs in
        the native stepper (one call to append, one to plan and upload).
        """
        pool = self._require_pool()
        ids = self._step_ids(sequence_ids)
        n = ids.size
        info = _lib.StepInfo()
        host, (p_rows, p_lens, p_tokb) = self._host_buffers(n)
        st = lib.pkv_stepper_begin(pool.stepper, ids.ctypes.data, n, ctypes.byref(info), p_rows, p_lens, p_tokb)
        if st == _lib.PKV_OK:
            with _on_device(pool.device):
                stream = _current_stream(pool.device)
                st = lib.pkv_stepper_upload(pool.stepper, stream, ctypes.byref(info), None, 0)
                if st != _lib.PKV_OK and self._needs_retry(pool, st, info):
                    st = self._upload_retry(pool, stream, info, st)
        return self._finish_step(pool, st, ids, info, host)

    def decode_attention(self, step: DecodeStep, layer: int, q: torch.Tensor, k_new: torch.Tensor | None = None,
                         v_new: torch.Tensor | None = None, *, scale: float | None = None,
                         out: torch.Tensor | None = None) -> torch.Tensor:
        """Paged GQA decode for one layer: ``q [B, Hq, D]`` -> ``[B, Hq, D]``.

        With ``k_new``/``v_new`` ``[B, Hkv, D]`` the kernel first appends the
        step's token into its page (and updates the device block table and
        lengths); without them the step's K/V must already be in the pool
        (``append_step_kv``).
        """
        pool = self._require_pool()
        if step.serial != pool.step_serial:
            raise RuntimeError("this decode step is stale: a later decode_step replaced its device descriptor")
        if (k_new is None) != (v_new is None):
            raise ValueError("pass both k_new and v_new or neither")
        out = self._check_decode_io(pool, step.batch, q, k_new, v_new, out)
        if k_new is None and not step.committed:
            # The step's new blocks and lengths reach the device tables here,
            # since no fused append will store them.
            lib.pkv_allocator_touch_rows(self.allocator._handle, step.host_rows.ctypes.data, step.batch)
            self._sync()
            step.committed = True
        with _on_device(pool.device):
            st = lib.pkv_stepper_attention(
                pool.stepper, int(layer), q.data_ptr(), k_new.data_ptr() if k_new is not None else None,
                v_new.data_ptr() if v_new is not None else None, q.shape[1],
                float(scale if scale is not None else pool.head_dim ** -0.5), out.data_ptr(),
                _current_stream(pool.device))
        _lib.raise_for_status(st)
        if k_new is not None:
            step.committed = True
        return out

    def append_step_kv(self, step: DecodeStep, layer: int, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Write the step's K/V ``[B, Hkv, D]`` into the pool without attention."""
        pool = self._require_pool()
        if step.serial != pool.step_serial:
            raise RuntimeError("this decode step is stale: a later decode_step replaced its device descriptor")
        pool.scatter(layer, k_new.permute(1, 0, 2).unsqueeze(0), v_new.permute(1, 0, 2).unsqueeze(0),
                     int(step.info.slots), step.batch)

    # -- device chunked-prefill / speculative-verify path (extension) -----------
    def prefill_step(self, sequence_ids, q_lens, num_q_heads: int, buffers: dict | None = None) -> PrefillStep:
        """Lay out one prefill / verify forward: each sequence's chunk is its last ``q_lens[i]``
        tokens (already reserved / appended in the allocator).  Records the chunks' block fills,
        plans the attention launch and uploads slots and work items once for all layers.

        ``buffers`` (``{"slots": int64, "records": int32 [n, 8]}`` device tensors) makes the
        upload go into those fixed addresses -- a forward recorded in a CUDA graph reads them
        there -- and requires the plan to have exactly ``buffers["n_items"]`` work items and
        no split-key combine entries (ValueError otherwise)."""
        pool = self._require_pool()
        ids = self._step_ids(sequence_ids)
        n = ids.size
        q_lens = np.asarray(q_lens, dtype=np.int64).reshape(-1)
        if q_lens.size != n or (q_lens < 0).any():
            raise ValueError("q_lens must give one non-negative chunk length per sequence")
        hq = int(num_q_heads)
        if hq <= 0 or hq % pool.num_kv_heads:
            raise ValueError("num_q_heads must be a positive multiple of the pool's KV heads")
        # Device tables up to date and copy-on-write copies applied (they carry
        # their source block's fill) before the chunk's fills are recorded.
        self._sync()
        q_lens = np.ascontiguousarray(q_lens, dtype=np.int64)
        rows = np.empty(n, dtype=np.int32)
        past = np.empty(n, dtype=np.int32)
        total_q = int(q_lens.sum())
        slots = np.empty(total_q, dtype=np.int64)
        fill = self._block_fill
        # Rows, past lengths and chunk slots in one native pass (fills raised to cover the chunks).
        _lib.raise_for_status(lib.pkv_allocator_chunk_slots(self.allocator._handle, ids.ctypes.data,
                                                            q_lens.ctypes.data, n, rows.ctypes.data,
                                                            past.ctypes.data, slots.ctypes.data, slots.size,
                                                            fill.ctypes.data, fill.size))
        if total_q == 0:
            return PrefillStep(ids, q_lens, hq, 0, None, None, None)
        if _device.VERIFY_KERNEL and verify_supported(hq, pool.num_kv_heads, pool.head_dim, pool.block_size,
                                                      int(q_lens.max())):
            # Short chunks (a verify step): the kernel with keys on the tensor-core rows.  A
            # recorded launch (buffers) needs a fixed record count: no key-range split.
            plan = plan_verify(rows, past, q_lens, hq, pool.num_kv_heads, 0 if buffers is not None else pool.num_sms)
        else:
            plan = plan_prefill(rows, past, q_lens, hq, pool.num_kv_heads, pool.num_sms)
        with _on_device(pool.device):
            if buffers is None:
                slots_d = pool.h2d.to_device(torch.from_numpy(slots), pool.device)
                records_d = pool.h2d.to_device(torch.from_numpy(plan.records), pool.device)
            else:
                if plan.n_combine or plan.n_items != buffers["n_items"] or slots.size > buffers["slots"].numel():
                    raise ValueError("the prefill plan does not fit the recorded launch")
                slots_d = buffers["slots"][:slots.size]
                records_d = buffers["records"][:plan.n_items]
                slots_d.copy_(pool.h2d.to_device(torch.from_numpy(slots), pool.device))
                records_d.copy_(pool.h2d.to_device(torch.from_numpy(plan.records), pool.device))
        return PrefillStep(ids, q_lens, hq, total_q, plan, slots_d, records_d)

    def prefill_attention(self, sequence_ids, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                          q_lens=None, layer: int = 0, scale: float | None = None,
                          out: torch.Tensor | None = None, step: PrefillStep | None = None) -> torch.Tensor:
        """Causal attention of chunks of queries over the paged cache, one layer.

        Sequence i's chunk is its last ``q_lens[i]`` tokens (already reserved /
        appended in the allocator): ``k``/``v`` ``[total_q, Hkv, D]`` are
        written into those slots, then each query ``[total_q, Hq, D]`` (packed in
        ``sequence_ids`` order) attends to its sequence's earlier tokens and the
        chunk up to itself -- the attention of one HF forward over a prefill
        chunk with a past cache (agentrl/generation/prefill.py:96-104).
        ``q_lens`` defaults to an equal split of ``total_q``.  ``step`` (from
        ``prefill_step`` for the same sequences and chunk lengths) skips the
        per-call layout work, for the layers after the first of a forward.
        """
        pool = self._require_pool()
        total_q = q.shape[0] if q.dim() == 3 else -1
        if step is None:
            ids = self._step_ids(sequence_ids)
            n = ids.size
            if q_lens is None:
                if n == 0 or total_q % n:
                    raise ValueError("q_lens is required when the queries do not split evenly over the sequences")
                q_lens = np.full(n, total_q // n, dtype=np.int64)
            q_lens = np.asarray(q_lens, dtype=np.int64).reshape(-1)
            if q_lens.size != n or (q_lens < 0).any() or int(q_lens.sum()) != total_q:
                raise ValueError("q_lens must give one non-negative chunk length per sequence summing to q.shape[0]")
        if q.dim() != 3 or q.shape[2] != pool.head_dim or q.shape[1] % pool.num_kv_heads:
            raise ValueError("q must be [total_q, num_q_heads, head_dim] with num_q_heads a multiple of num_kv_heads")
        if q.dtype != pool.dtype or q.device != pool.device or not q.is_contiguous():
            raise ValueError("q must be a contiguous tensor of the pool's dtype on the pool's device")
        shape = (total_q, pool.num_kv_heads, pool.head_dim)
        for t in (k, v):
            if t.shape != shape or t.dtype != pool.dtype or t.device != pool.device or not t.is_contiguous():
                raise ValueError("k/v must be contiguous [total_q, num_kv_heads, head_dim] pool-dtype tensors")
        if out is None:
            out = torch.empty_like(q)
        elif out.shape != q.shape or out.dtype != q.dtype or out.device != q.device or not out.is_contiguous():
            raise ValueError("out must be a contiguous tensor shaped and typed like q")
        if step is None:
            step = self.prefill_step(sequence_ids, q_lens, q.shape[1])
        elif step.total_q != total_q or step.num_q_heads != q.shape[1]:
            raise ValueError("the prefill step was laid out for other chunk lengths or query heads")
        if total_q == 0:
            return out
        with _on_device(pool.device):
            pool.scatter(layer, k.permute(1, 0, 2).unsqueeze(0), v.permute(1, 0, 2).unsqueeze(0), step.slots)
            pool.prefill(layer, q, step.plan, step.records, q.shape[1],
                         float(scale if scale is not None else pool.head_dim ** -0.5), out)
        return out

    def verify_attention(self, sequence_ids, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                         layer: int = 0, scale: float | None = None, step: PrefillStep | None = None) -> torch.Tensor:
        """The k+1-query speculative-verify read, one layer: ``q [B, k+1, Hq, D]`` -> same shape.

        Each sequence already holds its last accepted token and k draft tokens
        (appended in the allocator); ``k``/``v`` ``[B, k+1, Hkv, D]`` are their
        K/V.  The rows equal rows ``prefix_len-1 .. prefix_len-1+k`` of the
        reference's full causal verify forward (agentrl/generation/speculative.py:229-264).
        Rejected drafts are dropped afterwards with ``truncate``.  ``step``:
        ``prefill_step(sequence_ids, [k+1] * B, Hq)``, shared by the layers.
        """
        if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
            raise ValueError("verify inputs are q [B, k+1, Hq, D] and k/v [B, k+1, Hkv, D]")
        b, t = q.shape[0], q.shape[1]
        out = self.prefill_attention(sequence_ids, q.reshape(b * t, q.shape[2], q.shape[3]),
                                     k.reshape(b * t, k.shape[2], k.shape[3]), v.reshape(b * t, v.shape[2], v.shape[3]),
                                     q_lens=np.full(b, t, dtype=np.int64), layer=layer, scale=scale, step=step)
        return out.view(q.shape)

    @staticmethod
    def _step_ids(sequence_ids) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(sequence_ids, dtype=np.int64).reshape(-1))
        if ids.size == 0:
            raise ValueError("a decode step needs at least one sequence")
        return ids

    @staticmethod
    def _check_decode_io(pool: KVPool, n: int, q, k_new, v_new, out, device: torch.device | None = None):
        dev = pool.device if device is None else device
        if q.dim() != 3 or q.shape[0] != n or q.shape[2] != pool.head_dim:
            raise ValueError("q must be [batch, num_q_heads, head_dim]")
        if q.shape[1] <= 0 or q.shape[1] % pool.num_kv_heads:
            raise ValueError("num_q_heads must be a positive multiple of the pool's KV heads")
        if q.dtype != pool.dtype or q.device != dev or not q.is_contiguous():
            raise ValueError("q must be a contiguous tensor of the pool's dtype on the pool's device "
                             "(or all in host memory)")
        shape = (n, pool.num_kv_heads, pool.head_dim)
        for t in (k_new, v_new):
            if t is not None and (t.shape != shape or t.dtype != pool.dtype or t.device != dev
                                  or not t.is_contiguous()):
                raise ValueError("k_new/v_new must be contiguous [batch, num_kv_heads, head_dim] pool-dtype tensors "
                                 "on q's device")
        if out is None:
            return torch.empty(q.shape, dtype=q.dtype, pin_memory=True) if dev.type == "cpu" else torch.empty_like(q)
        if out.shape != q.shape or out.dtype != q.dtype or out.device != q.device or not out.is_contiguous():
            raise ValueError("out must be a contiguous tensor shaped and typed like q")
        return out

    def _finish_step(self, pool: KVPool, st: int, ids, info, host) -> DecodeStep:
        rows, lens, tok_blocks = host[0], host[1], host[2]
        if st != _lib.PKV_OK:
            # The appends made before the failure stay (as with the reference's
            # sequential append_tokens); their tokens have no stored K/V yet.
            # (The message is read first: the sync below makes library calls.)
            msg = _lib.last_error()
            k = int(info.batch)
            bs = self.allocator.block_size_tokens
            self._sync()
            self._block_fill[tok_blocks[:k]] = (lens[:k] - 1) % bs + 1
            _lib.raise_for_status(st, message=msg)
        # Block fills of the step (and of its copy-on-write copies) were set by
        # the native stepper.
        pool.step_serial += 1
        return DecodeStep(sequence_ids=ids, info=info, serial=pool.step_serial, host_rows=rows.copy(),
                          host_lens=lens.copy())

    # -- helpers -----------------------------------------------------------------
    def _ensure_pool(self, num_layers: int, num_kv_heads: int, head_dim: int, dtype: torch.dtype,
                     device: torch.device) -> KVPool:
        if self._pool is None:
            dev = device if device.type == "cuda" else None
            self._pool = self._new_pool(num_layers, num_kv_heads, head_dim, dtype, dev)
        p = self._pool
        if (p.num_layers, p.num_kv_heads, p.head_dim, p.dtype) != (num_layers, num_kv_heads, head_dim, dtype):
            raise ValueError(
                f"cache geometry (layers={num_layers}, kv_heads={num_kv_heads}, head_dim={head_dim}, {dtype}) does "
                f"not match the pool (layers={p.num_layers}, kv_heads={p.num_kv_heads}, head_dim={p.head_dim}, "
                f"{p.dtype})"
            )
        return p

    def _new_pool(self, num_layers: int, num_kv_heads: int, head_dim: int, dtype: torch.dtype, device) -> KVPool:
        pool = KVPool(self.allocator, num_layers, num_kv_heads, head_dim, dtype, device)
        # The native stepper keeps the per-block stored-token counts of decode
        # steps (and of copy-on-write copies) current in this array.
        _lib.raise_for_status(lib.pkv_stepper_bind_fill(pool.stepper, self._block_fill.ctypes.data,
                                                        self._block_fill.size))
        return pool

    def _require_pool(self) -> KVPool:
        if self._pool is None:
            raise RuntimeError("the KV pool does not exist yet: write a cache first or pass its geometry")
        return self._pool

    def _sync(self) -> None:
        """Bring the device tables up to date (the stepper carries block fills over copy-on-write copies)."""
        pool = self._pool
        if pool is None:
            return
        pool.sync()

    def _slots(self, blocks, fills, bs: int) -> torch.Tensor:
        parts = [np.arange(f, dtype=np.int64) + int(b) * bs for b, f in zip(blocks, fills) if f > 0]
        host = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
        return torch.from_numpy(host).to(self._pool.device)

    def _gather_legacy(self, blocks, fills, n: int, io_device) -> tuple[tuple[torch.Tensor, ...], ...]:
        pool = self._pool
        self._sync()
        slots = self._slots(blocks, fills, pool.block_size)[:n]
        out = torch.empty((pool.num_layers, 2, pool.num_kv_heads, n, pool.head_dim), dtype=pool.dtype,
                          device=pool.device)
        if n:
            pool.gather(0, out[:, 0], out[:, 1], slots)
        if io_device is not None and io_device != pool.device:
            out = out.to(io_device)
        return tuple((out[layer, 0].unsqueeze(0), out[layer, 1].unsqueeze(0)) for layer in range(pool.num_layers))
