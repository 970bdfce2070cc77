"""ctypes binding of libpkv_b200.so (the C ABI declared in include/pkv_b200.h).

The library is built in-tree (``python -m randomrepo_b200.build``) and loaded
from this package directory.  There is no fallback: if the library is missing
or stale the import fails loudly, because every entry point of this package
runs on it.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpkv_b200.so"

PKV_OK = 0
PKV_ERR_VALUE = 1
PKV_ERR_KEY = 2
PKV_ERR_RUNTIME = 3
PKV_ERR_INDEX = 4
PKV_ERR_ARG = 5
PKV_ERR_CUDA = 6
PKV_ERR_UNSUPPORTED = 7
PKV_ERR_CAPACITY = 8

PKV_F32 = 0
PKV_F16 = 1
PKV_BF16 = 2


class PoolGeom(ctypes.Structure):
    """``pkv_pool_geom``."""

    _fields_ = [
        ("num_layers", c_int32),
        ("num_blocks", c_int32),
        ("num_kv_heads", c_int32),
        ("block_size", c_int32),
        ("head_dim", c_int32),
        ("dtype", c_int32),
    ]


class AllocatorStats(ctypes.Structure):
    """``pkv_allocator_stats``."""

    _fields_ = [
        ("total_blocks", c_int64),
        ("block_size_tokens", c_int64),
        ("free_block_count", c_int64),
        ("used_block_count", c_int64),
        ("block_reuse_count", c_int64),
        ("max_blocks_in_use", c_int64),
        ("resident_sequence_count", c_int64),
        ("row_capacity", c_int64),
        ("max_blocks_per_row", c_int64),
        ("shared_block_count", c_int64),
    ]


class StepInfo(ctypes.Structure):
    """``pkv_step_info``."""

    _fields_ = [
        ("batch", c_int32),
        ("pages_per_split", c_int32),
        ("n_items", c_int32),
        ("n_combine", c_int32),
        ("n_copies", c_int32),
        ("need_rows", c_int32),
        ("need_cols", c_int32),
        ("need_items", c_int32),
        ("rows", c_void_p),
        ("seq_lens", c_void_p),
        ("new_blocks", c_void_p),
        ("items", c_void_p),
        ("slots", c_void_p),
    ]


I32P = POINTER(c_int32)
I64P = POINTER(c_int64)

# name -> (restype, argtypes)
_SIGNATURES: dict[str, tuple] = {
    "pkv_last_error": (c_char_p, []),
    "pkv_version": (c_char_p, []),
    "pkv_allocator_create": (c_void_p, [c_int64, c_int64, I32P]),
    "pkv_allocator_destroy": (None, [c_void_p]),
    "pkv_allocator_reserve": (c_int32, [c_void_p, c_int64, c_int64]),
    "pkv_allocator_append_tokens": (c_int32, [c_void_p, c_int64, c_int64]),
    "pkv_allocator_release": (c_int32, [c_void_p, c_int64]),
    "pkv_allocator_fork": (c_int32, [c_void_p, c_int64, c_int64]),
    "pkv_allocator_logical_to_physical": (c_int32, [c_void_p, c_int64, c_int64, I64P]),
    "pkv_allocator_view": (c_int32, [c_void_p, c_int64, I64P, c_void_p, c_int64, I64P]),
    "pkv_allocator_has_sequence": (c_int32, [c_void_p, c_int64]),
    "pkv_allocator_get_stats": (c_int32, [c_void_p, POINTER(AllocatorStats)]),
    "pkv_allocator_refcount": (c_int32, [c_void_p, c_int64, I32P]),
    "pkv_allocator_row": (c_int32, [c_void_p, c_int64, I32P]),
    "pkv_allocator_decode_step": (
        c_int32, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, I64P]
    ),
    "pkv_allocator_touch_rows": (c_int32, [c_void_p, c_void_p, c_int64]),
    "pkv_allocator_truncate": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64]),
    "pkv_allocator_truncate_fill": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int64]),
    "pkv_allocator_token_counts": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p]),
    "pkv_allocator_growth_blocks": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p]),
    "pkv_allocator_chunk_slots": (
        c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int64]
    ),
    "pkv_allocator_pending_updates": (c_int32, [c_void_p, I64P, I64P, I64P, I64P]),
    "pkv_allocator_drain_updates": (c_int32, [c_void_p, c_void_p, c_int64, I64P]),
    "pkv_pool_bytes": (c_int64, [POINTER(PoolGeom)]),
    "pkv_apply_updates": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "pkv_scatter_tokens": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p,
         c_int64, c_void_p],
    ),
    "pkv_gather_tokens": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p,
         c_int64, c_void_p],
    ),
    "pkv_copy_blocks": (c_int32, [POINTER(PoolGeom), c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "pkv_decode_heads_per_item": (c_int32, [c_int32]),
    "pkv_decode_plan": (
        c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int32, I32P, c_void_p, c_int64, I64P, I64P]
    ),
    "pkv_decode_workspace_bytes": (c_int64, [c_int32, c_int32, c_int32, c_int64]),
    "pkv_decode_attention": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_void_p,
         c_void_p, c_int64, c_void_p],
    ),
    "pkv_decode_attention_noalloc": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_void_p,
         c_void_p],
    ),
    "pkv_decode_noalloc_error": (c_int32, [I32P, c_void_p]),
    "pkv_prefill_positions_per_item": (c_int32, [c_int32, c_int32]),
    "pkv_prefill_plan": (
        c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64,
                  I64P, I64P, I64P]
    ),
    "pkv_prefill_workspace_bytes": (c_int64, [c_int64, c_int32]),
    "pkv_prefill_attention": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32,
         c_int64, c_int32, c_float, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p],
    ),
    "pkv_verify_positions_per_item": (c_int32, [c_int32, c_int32]),
    "pkv_verify_plan": (
        c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, I64P, I64P,
                  I64P, I64P]
    ),
    "pkv_verify_attention": (
        c_int32,
        [POINTER(PoolGeom), c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32,
         c_int32, c_int64, c_int32, c_float, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p],
    ),
    "pkv_stepper_create": (c_void_p, [c_void_p, POINTER(PoolGeom), c_void_p, I32P]),
    "pkv_stepper_destroy": (None, [c_void_p]),
    "pkv_stepper_bind_tables": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "pkv_stepper_bind_fill": (c_int32, [c_void_p, c_void_p, c_int64]),
    "pkv_stepper_fix_steps": (c_int32, [c_void_p, c_int32, c_int32, c_void_p]),
    "pkv_stepper_fixed_capacity": (c_int32, [c_void_p, I32P, I32P]),
    "pkv_stepper_sync": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, I32P, I32P, I32P]),
    "pkv_stepper_begin": (c_int32, [c_void_p, c_void_p, c_int32, POINTER(StepInfo), c_void_p, c_void_p, c_void_p]),
    "pkv_stepper_upload": (c_int32, [c_void_p, c_void_p, POINTER(StepInfo), c_void_p, c_int64]),
    "pkv_stepper_attention": (
        c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_float, c_void_p, c_void_p]
    ),
    "pkv_stepper_step": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_float, c_void_p, c_void_p,
         POINTER(StepInfo), c_void_p, c_void_p, c_void_p, c_void_p, c_int64],
    ),
    "pkv_stepper_step_host": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p,
         c_void_p, POINTER(StepInfo), c_void_p, c_void_p, c_void_p],
    ),
    "pkv_stepper_attention_host": (c_int32, [c_void_p, c_int32, c_int32, c_float, c_void_p, c_void_p]),
    "pkv_stepper_host_fence": (c_int32, [c_void_p, c_void_p]),
    "pkv_host_alloc": (c_int32, [c_int64, c_int32, POINTER(c_void_p)]),
    "pkv_host_free": (c_int32, [c_void_p]),
    "pkv_stepper_copies": (c_int32, [c_void_p, c_void_p, c_int64, I64P]),
    "pkv_stepper_error": (c_int32, [c_void_p, I32P]),
    "pkv_stepper_launches": (c_int64, [c_void_p]),
    "pkv_stepper_host_wait_ns": (c_int64, [c_void_p]),
    "pkv_stepper_time_launches": (c_int32, [c_void_p, c_int64, c_int64]),
    "pkv_stepper_launch_times": (c_int32, [c_void_p, c_void_p, c_int64, I64P]),
    "pkv_rms_norm": (
        c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_float, c_int32, c_void_p]
    ),
    "pkv_rope": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
         c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p],
    ),
    "pkv_silu_mul": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p]),
    "pkv_sampling_workspace_bytes": (c_int64, [c_int64, c_int32]),
    "pkv_token_logprobs": (
        c_int32,
        [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    ),
    "pkv_sample_tokens": (
        c_int32,
        [c_void_p, c_void_p, c_int64, c_int32, c_int32, c_float, c_int32, c_uint64, c_uint64, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    ),
    "pkv_spec_workspace_bytes": (c_int64, [c_int32, c_int32, c_int32]),
    "pkv_spec_tickets": (c_int64, [c_int32, c_int32]),
    "pkv_spec_accept": (
        c_int32,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_float, c_int32,
         c_int64, c_uint64, c_uint64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
         c_void_p],
    ),
}

# Entry points added after the first build; bound when present.
_OPTIONAL: dict[str, tuple] = {}


class PKVError(RuntimeError):
    """A kernel entry point of libpkv_b200 failed (bad argument or CUDA error)."""


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m randomrepo_b200.build` "
            "(the paged-KV path has no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in {**_SIGNATURES, **_OPTIONAL}.items():
        try:
            fn = getattr(lib, name)
        except AttributeError:
            if name in _OPTIONAL:
                continue
            raise ImportError(f"{LIB_PATH} does not export {name}: rebuild it") from None
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


def exported_symbols() -> list[str]:
    """Names this binding requires from the library."""
    return sorted(_SIGNATURES)


def last_error() -> str:
    msg = lib.pkv_last_error()
    return msg.decode() if msg else ""


def raise_for_status(status: int, *, key: object | None = None, message: str | None = None) -> None:
    """Translate a status into the exception the reference raises for it (``message``: the
    failure's text when it was read before later library calls replaced it)."""
    if status == PKV_OK:
        return
    msg = last_error() if message is None else message
    if status == PKV_ERR_VALUE:
        raise ValueError(msg)
    if status == PKV_ERR_KEY:
        raise KeyError(key if key is not None else msg)
    if status == PKV_ERR_RUNTIME:
        raise RuntimeError(msg)
    if status == PKV_ERR_INDEX:
        raise IndexError(msg)
    raise PKVError(f"libpkv_b200 status {status}: {msg}")
