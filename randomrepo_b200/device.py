"""Device side of the paged-KV store: the KV pool and the block-table mirror.

``KVPool`` owns, on one CUDA device:

* the pool ``[layers, blocks, 2 (K/V), kv_heads, block_size, head_dim]`` --
  a block's K (or V) rows for one KV head are one contiguous run, which is
  what the decode kernel's TMA boxes read;
* the device mirror of the allocator's state: block tables
  ``int32 [rows, cols]``, context lengths ``int32 [rows]`` and refcounts
  ``int32 [blocks]``.

The host allocator (C++, ``libpkv_b200``) stays authoritative.  It records
which entries changed; ``sync()`` drains that record into one pinned buffer,
copies it to the device with one ``cudaMemcpyAsync`` and applies it with one
kernel (plus the copy-on-write block copies).  Everything runs on the current
torch stream without host synchronisation.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from ._lib import lib

DTYPE_CODES = {torch.float32: _lib.PKV_F32, torch.float16: _lib.PKV_F16, torch.bfloat16: _lib.PKV_BF16}


def _stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class KVPool:
    """KV pool plus device block tables for one ``PagedKVAllocator``."""

    def __init__(self, allocator, num_layers: int, num_kv_heads: int, head_dim: int, dtype: torch.dtype,
                 device: torch.device | str | int | None = None) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("the paged-KV pool needs a CUDA device (there is no CPU path)")
        if dtype not in DTYPE_CODES:
            raise ValueError(f"unsupported KV dtype {dtype}")
        self.allocator = allocator
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("the paged-KV pool lives on a CUDA device")
        self.dtype = dtype
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.block_size = int(allocator.block_size_tokens)
        self.num_blocks = int(allocator.total_blocks)
        self.geom = _lib.PoolGeom(self.num_layers, self.num_blocks, self.num_kv_heads, self.block_size,
                                  self.head_dim, DTYPE_CODES[dtype])
        self._geom_ref = ctypes.byref(self.geom)
        nbytes = lib.pkv_pool_bytes(self._geom_ref)
        elem = torch.tensor([], dtype=dtype).element_size()
        self.pool = torch.zeros(nbytes // elem, dtype=dtype, device=self.device).view(
            self.num_layers, self.num_blocks, 2, self.num_kv_heads, self.block_size, self.head_dim)
        self.refcounts = torch.zeros(self.num_blocks, dtype=torch.int32, device=self.device)
        self.tables = torch.full((0, 0), -1, dtype=torch.int32, device=self.device)
        self.context_lens = torch.zeros(0, dtype=torch.int32, device=self.device)
        self._workspace = torch.zeros(0, dtype=torch.uint8, device=self.device)
        # Kernel launches issued through this pool (for launch accounting).
        self.launches = 0
        self.sync()

    # -- device tables ------------------------------------------------------
    def ensure_capacity(self) -> None:
        st = self.allocator._stats()
        rows_need, cols_need = int(st.row_capacity), int(st.max_blocks_per_row)
        rows, cols = self.tables.shape
        if rows_need <= rows and cols_need <= cols:
            return
        new_rows = max(rows, _round_up(max(rows_need, 1), 64))
        new_cols = max(cols, _round_up(max(cols_need, 1), 64))
        tables = torch.full((new_rows, new_cols), -1, dtype=torch.int32, device=self.device)
        tables[:rows, :cols] = self.tables
        lens = torch.zeros(new_rows, dtype=torch.int32, device=self.device)
        lens[:rows] = self.context_lens
        self.tables, self.context_lens = tables, lens

    def drain(self) -> torch.Tensor | None:
        """Drain the allocator's pending updates into a pinned int32 buffer."""
        a = self.allocator._handle
        nt, nr, nl, nc = (ctypes.c_int64() for _ in range(4))
        lib.pkv_allocator_pending_updates(a, ctypes.byref(nt), ctypes.byref(nr), ctypes.byref(nl), ctypes.byref(nc))
        if nt.value + nr.value + nl.value + nc.value == 0:
            return None
        cap = 4 + 3 * nt.value + 2 * nr.value + 2 * nl.value + 2 * nc.value
        buf = torch.empty(cap, dtype=torch.int32, pin_memory=True)
        written = ctypes.c_int64()
        _lib.raise_for_status(lib.pkv_allocator_drain_updates(a, buf.data_ptr(), cap, ctypes.byref(written)))
        return buf[: written.value]

    def sync(self, drained: torch.Tensor | None = None) -> torch.Tensor | None:
        """Bring the device tables, lengths and refcounts up to the host state."""
        self.ensure_capacity()
        buf = self.drain() if drained is None else drained
        if buf is None:
            return None
        dev = buf.to(self.device, non_blocking=True)
        rows, cols = self.tables.shape
        st = lib.pkv_apply_updates(self._geom_ref, self.pool.data_ptr(), self.tables.data_ptr(), cols, rows,
                                   self.refcounts.data_ptr(), self.context_lens.data_ptr(), dev.data_ptr(),
                                   buf.data_ptr(), _stream_ptr())
        _lib.raise_for_status(st)
        self.launches += 1 + _copy_waves(buf)
        return buf

    # -- data movement --------------------------------------------------------
    def scatter(self, layer0: int, k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor) -> None:
        """Write token rows: k/v ``[n_layers, kv_heads, n_tokens, head_dim]`` (any strides with a
        contiguous innermost dim, equal strides for k and v) into ``slots`` (int64 device)."""
        self._check_rows(k, v)
        st = lib.pkv_scatter_tokens(self._geom_ref, self.pool.data_ptr(), layer0, k.shape[0], k.data_ptr(),
                                    v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), slots.data_ptr(),
                                    slots.numel(), _stream_ptr())
        _lib.raise_for_status(st)
        self.launches += 1

    def gather(self, layer0: int, k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor) -> None:
        """Inverse of ``scatter``: fill k/v ``[n_layers, kv_heads, n_tokens, head_dim]``."""
        self._check_rows(k, v)
        st = lib.pkv_gather_tokens(self._geom_ref, self.pool.data_ptr(), layer0, k.shape[0], k.data_ptr(),
                                   v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), slots.data_ptr(),
                                   slots.numel(), _stream_ptr())
        _lib.raise_for_status(st)
        self.launches += 1

    def _check_rows(self, k: torch.Tensor, v: torch.Tensor) -> None:
        if k.dtype != self.dtype or v.dtype != self.dtype:
            raise ValueError(f"K/V dtype {k.dtype} does not match the pool dtype {self.dtype}")
        if k.device != self.device or v.device != self.device:
            raise ValueError("K/V must live on the pool's device")
        if k.dim() != 4 or k.shape != v.shape or k.stride() != v.stride():
            raise ValueError("k and v must be [n_layers, kv_heads, n_tokens, head_dim] with equal strides")
        if k.shape[1] != self.num_kv_heads or k.shape[3] != self.head_dim or k.stride(3) != 1:
            raise ValueError("K/V rows do not match the pool geometry")

    # -- decode ---------------------------------------------------------------
    def workspace(self, nbytes: int) -> torch.Tensor:
        if self._workspace.numel() < nbytes:
            self._workspace = torch.zeros(_round_up(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
        return self._workspace

    def decode_error_flag(self) -> int:
        """Error word the decode kernel writes on a bounded-wait timeout (0 = none). Synchronises."""
        if self._workspace.numel() < 4:
            return 0
        return int(self._workspace[:4].view(torch.int32).item())


def _copy_waves(buf: torch.Tensor) -> int:
    """Launches pkv_apply_updates issues for the copy-on-write pairs of a drained buffer."""
    h = buf.numpy()
    nt, nr, nl, nc = (int(x) for x in h[:4])
    if nc == 0:
        return 0
    pairs = h[4 + 3 * nt + 2 * nr + 2 * nl :].reshape(nc, 2)
    waves, touched = 1, set()
    for src, dst in pairs.tolist():
        if src in touched or dst in touched:
            waves += 1
            touched = set()
        touched.update((src, dst))
    return waves


def plan_splits(lens: np.ndarray, num_kv_heads: int, block_size: int = 16, sms: int = 148,
                max_splits_per_seq: int = 64) -> tuple[int, np.ndarray]:
    """Choose pages per split work item and lay out the work items.

    Aims at several waves of CTAs over the GPU (2 resident CTAs per SM) while
    keeping each work item at 4..32 pages so its 4 warps stream enough data.
    Returns (pages_per_split, split_offsets[int32, n+1]).
    """
    pages = (lens.astype(np.int64) + block_size - 1) // block_size
    total = int(pages.sum()) * num_kv_heads
    target_ctas = sms * 2 * 4
    pps = max(4, min(32, math.ceil(total / target_ctas)))
    pps = max(pps, math.ceil(int(pages.max(initial=1)) / max_splits_per_seq))
    nsplits = np.maximum((pages + pps - 1) // pps, 1)
    offsets = np.zeros(len(lens) + 1, dtype=np.int32)
    np.cumsum(nsplits, out=offsets[1:])
    return pps, offsets
