"""The paged-KV kernels as PyTorch operators (``torch.ops.pkv.*``), over the C ABI.

``PagedKVCacheStore`` and ``KVPool`` call ``libpkv_b200.so`` directly; these
operators expose the same kernels to PyTorch's dispatcher, so that they show up
in traces, run under fake tensors (shape propagation without a GPU) and can sit
inside ``torch.compile``d code.  Each takes device tensors, launches on the
current stream, never synchronises, and raises ``RuntimeError`` with the
library's message when a launch is refused.

The pool is the store's single allocation ``KVPool.pool``; ``geom`` is
``pool_geom(kv_pool)``: ``[num_layers, num_blocks, num_kv_heads, block_size,
head_dim, dtype code]`` (the ``pkv_pool_geom`` of the C ABI).

* ``kv_append(pool, geom, layer, k, v, slot_mapping)``: k / v ``[B, Hkv, D]``
  into token slots (``block * block_size + offset``) -- the per-step append
  (transformers cache_utils.py:119-120) as a scatter into pages.
* ``kv_gather(pool, geom, layer, slot_mapping) -> (k, v)`` ``[n, Hkv, D]``
  (read_sequence_legacy_cache's ``torch.cat`` of blocks, paged_kv.py:302-321).
* ``copy_blocks(pool, geom, src, dst)``: whole blocks, every layer (the
  copy-on-write copy of a forked tail; no reference counterpart).
* ``decode_attention(...) -> out [B, Hq, D]``: fused append + paged GQA decode
  over a ``pkv_decode_plan`` (HF sdpa_attention_forward with GQA over the
  resident caches, continuous.py:476-483).
* ``prefill_attention(...) -> out [T, Hq, D]``: causal attention of query
  chunks after a cached past over a ``pkv_prefill_plan`` -- chunked prefill
  (prefill.py:96-104) and the k+1-row speculative verify read
  (speculative.py:229-264).
* ``verify_attention(...) -> out [T, Hq, D]``: the same read for short chunks
  (a verify step) over a ``pkv_verify_plan``, on the kernel that puts keys on
  the tensor-core rows (``PagedKVCacheStore.prefill_step`` picks it when the
  chunks fit).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import lib

__all__ = ["pool_geom"]


def pool_geom(kv_pool) -> list[int]:
    """``[num_layers, num_blocks, num_kv_heads, block_size, head_dim, dtype code]`` of a ``KVPool``."""
    g = kv_pool.geom
    return [int(g.num_layers), int(g.num_blocks), int(g.num_kv_heads), int(g.block_size), int(g.head_dim),
            int(g.dtype)]


def _geom(geom: list[int]) -> _lib.PoolGeom:
    if len(geom) != 6:
        raise RuntimeError("geom must be [num_layers, num_blocks, num_kv_heads, block_size, head_dim, dtype code]")
    return _lib.PoolGeom(*[int(x) for x in geom])


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check(st: int) -> None:
    _lib.raise_for_status(st)


def _opt(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


@torch.library.custom_op("pkv::kv_append", mutates_args=("pool",), device_types="cuda")
def kv_append(pool: torch.Tensor, geom: list[int], layer: int, k: torch.Tensor, v: torch.Tensor,
              slot_mapping: torch.Tensor) -> None:
    _need(k.dim() == 3 and k.shape == v.shape and k.stride() == v.stride() and k.stride(2) == 1,
          "k and v must be [B, Hkv, D] with equal strides and contiguous rows")
    _need(slot_mapping.dtype == torch.int64 and slot_mapping.numel() == k.shape[0], "slot_mapping: int64 [B]")
    g = _geom(geom)
    _check(lib.pkv_scatter_tokens(ctypes.byref(g), pool.data_ptr(), int(layer), 1, k.data_ptr(), v.data_ptr(),
                                  k.numel(), k.stride(1), k.stride(0), slot_mapping.data_ptr(), k.shape[0],
                                  _stream(pool)))


@kv_append.register_fake
def _(pool, geom, layer, k, v, slot_mapping):
    return None


@torch.library.custom_op("pkv::kv_gather", mutates_args=(), device_types="cuda")
def kv_gather(pool: torch.Tensor, geom: list[int], layer: int,
              slot_mapping: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _need(slot_mapping.dtype == torch.int64 and slot_mapping.dim() == 1, "slot_mapping: int64 [n]")
    g = _geom(geom)
    n = slot_mapping.numel()
    dtype = {_lib.PKV_BF16: torch.bfloat16, _lib.PKV_F16: torch.float16, _lib.PKV_F32: torch.float32}[g.dtype]
    k = torch.empty((n, g.num_kv_heads, g.head_dim), dtype=dtype, device=pool.device)
    v = torch.empty_like(k)
    if n:
        _check(lib.pkv_gather_tokens(ctypes.byref(g), pool.data_ptr(), int(layer), 1, k.data_ptr(), v.data_ptr(),
                                     k.numel(), k.stride(1), k.stride(0), slot_mapping.data_ptr(), n, _stream(pool)))
    return k, v


@kv_gather.register_fake
def _(pool, geom, layer, slot_mapping):
    dtype = {_lib.PKV_BF16: torch.bfloat16, _lib.PKV_F16: torch.float16, _lib.PKV_F32: torch.float32}[int(geom[5])]
    k = pool.new_empty((slot_mapping.shape[0], int(geom[2]), int(geom[4])), dtype=dtype)
    return k, torch.empty_like(k)


@torch.library.custom_op("pkv::copy_blocks", mutates_args=("pool",), device_types="cuda")
def copy_blocks(pool: torch.Tensor, geom: list[int], src: torch.Tensor, dst: torch.Tensor) -> None:
    _need(src.dtype == torch.int32 and dst.dtype == torch.int32 and src.numel() == dst.numel(),
          "src and dst: int32 block ids of equal count")
    g = _geom(geom)
    if src.numel():
        _check(lib.pkv_copy_blocks(ctypes.byref(g), pool.data_ptr(), src.data_ptr(), dst.data_ptr(), src.numel(),
                                   _stream(pool)))


@copy_blocks.register_fake
def _(pool, geom, src, dst):
    return None


@torch.library.custom_op("pkv::decode_attention",
                         mutates_args=("pool", "block_tables", "context_lens", "workspace"), device_types="cuda")
def decode_attention(pool: torch.Tensor, geom: list[int], layer: int, q: torch.Tensor, k_new: torch.Tensor | None,
                     v_new: torch.Tensor | None, block_tables: torch.Tensor, context_lens: torch.Tensor,
                     rows: torch.Tensor, seq_lens: torch.Tensor, new_blocks: torch.Tensor | None,
                     work_items: torch.Tensor, n_items: int, n_combine: int, pages_per_split: int, scale: float,
                     workspace: torch.Tensor) -> torch.Tensor:
    """``pkv_decode_attention``: q ``[B, Hq, D]``; k_new / v_new ``[B, Hkv, D]`` (appended first) or None;
    rows / seq_lens / new_blocks int32 ``[B]``; work_items the int32 plan ``[n_items + n_combine, 4]``;
    workspace ``pkv_decode_workspace_bytes`` bytes, zeroed before its first use."""
    _need(q.dim() == 3 and q.is_contiguous(), "q must be a contiguous [B, Hq, D] tensor")
    _need(block_tables.dtype == torch.int32 and block_tables.dim() == 2, "block_tables: int32 [rows, stride]")
    g = _geom(geom)
    out = torch.empty_like(q)
    _check(lib.pkv_decode_attention(ctypes.byref(g), pool.data_ptr(), int(layer), q.data_ptr(), _opt(k_new),
                                    _opt(v_new), block_tables.data_ptr(), block_tables.shape[1],
                                    block_tables.shape[0], context_lens.data_ptr(), rows.data_ptr(),
                                    seq_lens.data_ptr(), _opt(new_blocks), work_items.data_ptr(), int(n_items),
                                    int(n_combine), q.shape[0], q.shape[1], int(pages_per_split), float(scale),
                                    out.data_ptr(), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                    _stream(q)))
    return out


@decode_attention.register_fake
def _(pool, geom, layer, q, k_new, v_new, block_tables, context_lens, rows, seq_lens, new_blocks, work_items,
      n_items, n_combine, pages_per_split, scale, workspace):
    return torch.empty_like(q)


@torch.library.custom_op("pkv::prefill_attention", mutates_args=("error_word", "workspace"), device_types="cuda")
def prefill_attention(pool: torch.Tensor, geom: list[int], layer: int, q: torch.Tensor, block_tables: torch.Tensor,
                      work_items: torch.Tensor, n_items: int, n_combine: int, n_slots: int, scale: float,
                      error_word: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
    """``pkv_prefill_attention``: q ``[T, Hq, D]`` (the chunks' queries, packed); work_items the int32
    records of ``pkv_prefill_plan`` ``[n_items + n_combine, 8]``; error_word an int32 device scalar."""
    _need(q.dim() == 3 and q.is_contiguous(), "q must be a contiguous [T, Hq, D] tensor")
    g = _geom(geom)
    out = torch.empty_like(q)
    _check(lib.pkv_prefill_attention(ctypes.byref(g), pool.data_ptr(), int(layer), q.data_ptr(),
                                     block_tables.data_ptr(), block_tables.shape[1], block_tables.shape[0],
                                     work_items.data_ptr(), int(n_items), int(n_combine), q.shape[0], q.shape[1],
                                     float(scale), out.data_ptr(), error_word.data_ptr(),
                                     workspace.data_ptr() if workspace.numel() else None,
                                     workspace.numel() * workspace.element_size(), int(n_slots), _stream(q)))
    return out


@prefill_attention.register_fake
def _(pool, geom, layer, q, block_tables, work_items, n_items, n_combine, n_slots, scale, error_word, workspace):
    return torch.empty_like(q)


@torch.library.custom_op("pkv::verify_attention", mutates_args=("error_word", "workspace"), device_types="cuda")
def verify_attention(pool: torch.Tensor, geom: list[int], layer: int, q: torch.Tensor, block_tables: torch.Tensor,
                     work_items: torch.Tensor, n_items: int, n_ctas: int, n_combine: int, n_slots: int, scale: float,
                     error_word: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
    """``pkv_verify_attention``: q ``[T, Hq, D]``; work_items the int32 records of ``pkv_verify_plan``
    ``[n_items + n_combine, 8]`` and its CTA count; workspace ``pkv_prefill_workspace_bytes(n_slots, 128)``
    bytes (may be empty when n_slots is 0); error_word an int32 device scalar."""
    _need(q.dim() == 3 and q.is_contiguous(), "q must be a contiguous [T, Hq, D] tensor")
    g = _geom(geom)
    out = torch.empty_like(q)
    _check(lib.pkv_verify_attention(ctypes.byref(g), pool.data_ptr(), int(layer), q.data_ptr(),
                                    block_tables.data_ptr(), block_tables.shape[1], block_tables.shape[0],
                                    work_items.data_ptr(), int(n_items), int(n_ctas), int(n_combine), q.shape[0],
                                    q.shape[1], float(scale), out.data_ptr(), error_word.data_ptr(),
                                    workspace.data_ptr() if workspace.numel() else None,
                                    workspace.numel() * workspace.element_size(), int(n_slots), _stream(q)))
    return out


@verify_attention.register_fake
def _(pool, geom, layer, q, block_tables, work_items, n_items, n_ctas, n_combine, n_slots, scale, error_word,
      workspace):
    return torch.empty_like(q)
