"""Device side of the paged-KV store: the KV pool and the block-table mirror.

``KVPool`` owns, on one CUDA device:

* the pool ``[layers, blocks, kv_heads, 2 (K/V), block_size, head_dim]`` --
  a block's K and V pages of all KV heads are one contiguous run, which the
  decode kernel moves with one bulk copy per head group; pages whose rows are
  a multiple of 128 bytes are stored pre-swizzled (see include/pkv_b200.h), so
  the pool is read and written through the scatter / gather kernels only;
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
import weakref
from dataclasses import dataclass

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


class PinnedStaging:
    """Host-to-device copies of a step's small inputs (positions, token ids, slots, work items)
    through a ring of page-locked buffers.  A copy from pageable memory makes the host wait until
    the stream has drained up to it; from page-locked memory it is queued and the host runs on.
    A buffer is written again only after the copy that read it has run (one event per slot)."""

    def __init__(self, slots: int = 16) -> None:
        self._bufs: list[torch.Tensor | None] = [None] * slots
        self._events: list = [None] * slots
        self._next = 0

    def to_device(self, x, device: torch.device, dtype: torch.dtype | None = None) -> torch.Tensor:
        src = torch.as_tensor(x)
        if dtype is not None and src.dtype != dtype:
            src = src.to(dtype)
        if device.type != "cuda":
            return src.to(device)
        src = src.contiguous()
        nbytes = src.numel() * src.element_size()
        out = torch.empty(src.shape, dtype=src.dtype, device=device)
        if nbytes == 0:
            return out
        i = self._next
        self._next = (i + 1) % len(self._bufs)
        ev = self._events[i]
        if ev is not None:
            ev.synchronize()  # the copy that last read this buffer has run
        buf = self._bufs[i]
        if buf is None or buf.numel() < nbytes:
            buf = self._bufs[i] = torch.empty(max(nbytes, 4096), dtype=torch.uint8).pin_memory()
        staged = buf[:nbytes].view(src.dtype).view(src.shape)
        staged.copy_(src)
        # The copy runs on the destination device's current stream, so the
        # guard is recorded there too, whichever device is current.
        stream = torch.cuda.current_stream(device)
        with torch.cuda.stream(stream):
            out.copy_(staged, non_blocking=True)
        if ev is None or ev.device != stream.device:
            ev = self._events[i] = torch.cuda.Event()
        ev.record(stream)
        return out


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
            self.num_layers, self.num_blocks, self.num_kv_heads, 2, self.block_size, self.head_dim)
        self.refcounts = torch.zeros(self.num_blocks, dtype=torch.int32, device=self.device)
        self.tables = torch.full((64, 64), -1, dtype=torch.int32, device=self.device)
        self.context_lens = torch.zeros(64, dtype=torch.int32, device=self.device)
        # Error word of the prefill / verify kernel (0 = none).
        self.prefill_error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._prefill_ws = torch.empty(0, dtype=torch.uint8, device=self.device)
        self.h2d = PinnedStaging()
        self.num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        # Kernel launches issued from Python through this pool (the stepper counts its own).
        self.launches = 0
        status = ctypes.c_int32()
        with torch.cuda.device(self.device):
            self.stepper = lib.pkv_stepper_create(allocator._handle, self._geom_ref, self.pool.data_ptr(),
                                                  ctypes.byref(status))
        if not self.stepper:
            _lib.raise_for_status(status.value)
        weakref.finalize(self, lib.pkv_stepper_destroy, self.stepper)
        self.step_serial = 0
        self.fixed_batch = 0  # fixed-step mode capacity (0: off)
        self.fixed_items = 0
        self.fixed_serial = 0  # bumped by every fix_steps (graphs hold the fixed block's address)
        self._timing_cap = 0
        self._pending = [ctypes.pointer(ctypes.c_int64()) for _ in range(4)]
        self._bind()
        self.sync()

    # -- device tables ------------------------------------------------------
    def _bind(self) -> None:
        rows, cols = self.tables.shape
        lib.pkv_stepper_bind_tables(self.stepper, self.tables.data_ptr(), cols, rows, self.context_lens.data_ptr(),
                                    self.refcounts.data_ptr())

    def grow(self, rows_need: int, cols_need: int) -> None:
        """Grow the device tables to at least rows_need x cols_need (contents kept)."""
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
        self._bind()

    def fix_steps(self, max_batch: int, max_items: int = 0) -> None:
        """Switch decode steps to fixed-step mode (``pkv_stepper_fix_steps``) so that their attention
        launches can be recorded in a CUDA graph and replayed for later steps."""
        with torch.cuda.device(self.device):
            _lib.raise_for_status(lib.pkv_stepper_fix_steps(self.stepper, int(max_batch), int(max_items),
                                                            _stream_ptr()))
        b, i = ctypes.c_int32(), ctypes.c_int32()
        lib.pkv_stepper_fixed_capacity(self.stepper, ctypes.byref(b), ctypes.byref(i))
        self.fixed_batch, self.fixed_items = int(b.value), int(i.value)
        self.fixed_serial += 1

    def pending_copies(self) -> int:
        c = self._pending
        lib.pkv_allocator_pending_updates(self.allocator._handle, c[0], c[1], c[2], c[3])
        return int(c[3].contents.value)

    def sync(self) -> np.ndarray:
        """Bring the device tables, lengths and refcounts up to the host allocator's state.

        Returns the copy-on-write (src, dst) block pairs applied, int32 [n, 2].
        """
        cap = self.pending_copies()
        copies = np.empty((max(cap, 1), 2), dtype=np.int32)
        n, need_r, need_c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        with torch.cuda.device(self.device):
            stream = _stream_ptr()
            st = lib.pkv_stepper_sync(self.stepper, stream, copies.ctypes.data, cap, ctypes.byref(n),
                                      ctypes.byref(need_r), ctypes.byref(need_c))
            if st == _lib.PKV_ERR_CAPACITY:
                self.grow(need_r.value, need_c.value)
                st = lib.pkv_stepper_sync(self.stepper, stream, copies.ctypes.data, cap, ctypes.byref(n),
                                          ctypes.byref(need_r), ctypes.byref(need_c))
        _lib.raise_for_status(st)
        return copies[: n.value]

    def time_launches(self, count: int, every: int = 1) -> None:
        """Time ``count`` of the next decode-attention launches, every ``every``-th one (0 = off)."""
        _lib.raise_for_status(lib.pkv_stepper_time_launches(self.stepper, int(count), int(every)))
        self._timing_cap = int(count)

    def launch_times_ms(self) -> np.ndarray:
        """Device milliseconds of the launches timed since ``time_launches``."""
        out = np.zeros(max(1, int(self._timing_cap)), dtype=np.float32)
        n = ctypes.c_int64()
        _lib.raise_for_status(lib.pkv_stepper_launch_times(self.stepper, out.ctypes.data, out.size, ctypes.byref(n)))
        return out[: n.value]

    def launch_count(self) -> int:
        return self.launches + int(lib.pkv_stepper_launches(self.stepper))

    def decode_error_flag(self) -> int:
        """Error word the decode kernels write (0 = none); synchronises with the device."""
        err = ctypes.c_int32()
        _lib.raise_for_status(lib.pkv_stepper_error(self.stepper, ctypes.byref(err)))
        return int(err.value)

    def prefill_error_flag(self) -> int:
        """Error word the prefill / verify kernel writes (0 = none); synchronises with the device."""
        return int(self.prefill_error.item())

    def prefill(self, layer: int, q: torch.Tensor, plan: "PrefillPlan", records: torch.Tensor, num_q_heads: int,
                scale: float, out: torch.Tensor) -> None:
        """Launch paged prefill / verify attention on the current stream: ``pkv_prefill_attention``
        for a ``plan_prefill`` plan, ``pkv_verify_attention`` for a ``plan_verify`` one.

        ``records`` is the device copy of ``plan.records``; key-range partials
        go to a workspace the pool keeps (grown on demand, never shrunk).
        """
        need = int(lib.pkv_prefill_workspace_bytes(plan.n_slots, self.head_dim))
        if need > self._prefill_ws.numel():
            self._prefill_ws = torch.empty(_round_up(need, 1 << 20), dtype=torch.uint8, device=self.device)
        rows, cols = self.tables.shape
        head = (self._geom_ref, self.pool.data_ptr(), int(layer), q.data_ptr(), self.tables.data_ptr(), cols, rows,
                records.data_ptr(), plan.n_items)
        tail = (plan.n_combine, q.shape[0], int(num_q_heads), float(scale), out.data_ptr(),
                self.prefill_error.data_ptr(), self._prefill_ws.data_ptr(), self._prefill_ws.numel(), plan.n_slots,
                _stream_ptr())
        if plan.kind == "verify":
            st = lib.pkv_verify_attention(*head, plan.n_ctas, *tail)
        else:
            st = lib.pkv_prefill_attention(*head, *tail)
        _lib.raise_for_status(st)
        self.launches += 2 if plan.n_combine else 1

    # -- data movement --------------------------------------------------------
    def scatter(self, layer0: int, k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor | int,
                n_tokens: int | None = None) -> None:
        """Write token rows: k/v ``[n_layers, kv_heads, n_tokens, head_dim]`` (any strides with a
        contiguous innermost dim, equal strides for k and v) into ``slots`` (int64 device tensor,
        or a device pointer with ``n_tokens``)."""
        self._check_rows(k, v)
        ptr = slots if isinstance(slots, int) else slots.data_ptr()
        n = n_tokens if isinstance(slots, int) else slots.numel()
        st = lib.pkv_scatter_tokens(self._geom_ref, self.pool.data_ptr(), layer0, k.shape[0], k.data_ptr(),
                                    v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), ptr, n, _stream_ptr())
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


def plan_decode(lens: np.ndarray, num_kv_heads: int, num_sms: int,
                head_dim: int = 128) -> tuple[int, np.ndarray, int, int]:
    """Plan one decode step (``pkv_decode_plan``).

    Returns (pages_per_split, int32 [n_items + n_combine, 4], n_items,
    n_combine): the work items followed by the split-K combine entries.
    """
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    pps = ctypes.c_int32()
    n = ctypes.c_int64()
    nc = ctypes.c_int64()
    _lib.raise_for_status(lib.pkv_decode_plan(lens.ctypes.data, lens.size, num_kv_heads, head_dim, num_sms,
                                              ctypes.byref(pps), None, 0, ctypes.byref(n), ctypes.byref(nc)))
    items = np.empty((n.value + nc.value, 4), dtype=np.int32)
    _lib.raise_for_status(lib.pkv_decode_plan(lens.ctypes.data, lens.size, num_kv_heads, head_dim, num_sms,
                                              ctypes.byref(pps), items.ctypes.data, items.shape[0], ctypes.byref(n),
                                              ctypes.byref(nc)))
    return int(pps.value), items, int(n.value), int(nc.value)


@dataclass
class PrefillPlan:
    """``pkv_prefill_plan`` / ``pkv_verify_plan`` output: int32 [n_items + n_combine, 8] records,
    their counts, and which kernel they are for (``"prefill"`` or ``"verify"``)."""

    records: np.ndarray
    n_items: int
    n_combine: int
    n_slots: int
    kind: str = "prefill"
    n_ctas: int = 0  # verify: CTAs of the launch (each works through a list of items)


PREFILL_SPLIT_WAVES = 0
# Chunks of few queries (verify steps) go to pkv_verify_attention where it supports the shape.
VERIFY_KERNEL = True


def plan_prefill(rows: np.ndarray, past_lens: np.ndarray, q_lens: np.ndarray, num_q_heads: int,
                 num_kv_heads: int, num_sms: int = 0, split_waves: int | None = None) -> PrefillPlan:
    """Plan one prefill / verify launch (``pkv_prefill_plan``).

    With ``split_waves`` > 0 (default ``PREFILL_SPLIT_WAVES``) and ``num_sms``
    > 0, a launch of few items (a verify step) cuts long key ranges across
    about ``split_waves`` CTAs per SM and merges their partials; 0 keeps one
    CTA per item.
    """
    waves = PREFILL_SPLIT_WAVES if split_waves is None else int(split_waves)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    past_lens = np.ascontiguousarray(past_lens, dtype=np.int32)
    q_lens = np.ascontiguousarray(q_lens, dtype=np.int32)
    if not rows.size == past_lens.size == q_lens.size:
        raise ValueError("rows, past_lens and q_lens must have one entry per sequence")
    n, nc, ns = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    args = (rows.ctypes.data, past_lens.ctypes.data, q_lens.ctypes.data, rows.size, num_q_heads, num_kv_heads,
            int(num_sms), waves)
    _lib.raise_for_status(lib.pkv_prefill_plan(*args, None, 0, ctypes.byref(n), ctypes.byref(nc), ctypes.byref(ns)))
    records = np.empty((n.value + nc.value, 8), dtype=np.int32)
    _lib.raise_for_status(lib.pkv_prefill_plan(*args, records.ctypes.data, records.shape[0], ctypes.byref(n),
                                               ctypes.byref(nc), ctypes.byref(ns)))
    return PrefillPlan(records, int(n.value), int(nc.value), int(ns.value))


def verify_supported(num_q_heads: int, num_kv_heads: int, head_dim: int, block_size: int, q_len: int) -> bool:
    """Whether ``pkv_verify_attention`` takes chunks of ``q_len`` queries in one item per KV head."""
    ppv = int(lib.pkv_verify_positions_per_item(int(num_q_heads), int(num_kv_heads)))
    return head_dim == 128 and block_size == 16 and 0 < q_len <= ppv


def plan_verify(rows: np.ndarray, past_lens: np.ndarray, q_lens: np.ndarray, num_q_heads: int,
                num_kv_heads: int, num_sms: int = 0) -> PrefillPlan:
    """Plan one ``pkv_verify_attention`` launch (``pkv_verify_plan``).

    With ``num_sms`` > 0 the launch is a persistent grid of one CTA per SM,
    each working through a list of items (long key ranges cut, partials merged
    by combine entries); 0 gives one CTA per item and no combine entries.
    """
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    past_lens = np.ascontiguousarray(past_lens, dtype=np.int32)
    q_lens = np.ascontiguousarray(q_lens, dtype=np.int32)
    if not rows.size == past_lens.size == q_lens.size:
        raise ValueError("rows, past_lens and q_lens must have one entry per sequence")
    n, nb, nc, ns = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    args = (rows.ctypes.data, past_lens.ctypes.data, q_lens.ctypes.data, rows.size, num_q_heads, num_kv_heads,
            int(num_sms))
    counts = (ctypes.byref(n), ctypes.byref(nb), ctypes.byref(nc), ctypes.byref(ns))
    _lib.raise_for_status(lib.pkv_verify_plan(*args, None, 0, *counts))
    records = np.empty((n.value + nc.value, 8), dtype=np.int32)
    _lib.raise_for_status(lib.pkv_verify_plan(*args, records.ctypes.data, records.shape[0], *counts))
    return PrefillPlan(records, int(n.value), int(nc.value), int(ns.value), "verify", int(nb.value))
