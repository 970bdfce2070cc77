"""The decode entry point for callers that may not allocate device memory.

A serving framework that owns all GPU memory through its own arena, or a
plugin host that only hands the library pre-allocated buffers, cannot let the
library allocate a decode workspace.  ``pkv_decode_attention_noalloc`` serves
them from a fixed scratch array inside the library.  This test calls it
through the C ABI, twice in a row, and checks each result against
``pkv_decode_attention`` given a workspace allocated here, with the decode
tolerance used throughout (its results are in fact identical: same kernels,
same plan), and reads the calls' device error word through
``pkv_decode_noalloc_error``.  It also checks that an oversized step is
refused before anything runs, and that a block id outside the pool is
reported (error 4) and cleared by the next call.  The file is named to be collected last, and it builds its own store so
it passes alone in a fresh process as well as after the other tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _setup(device):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    gen = torch.Generator().manual_seed(17)
    lengths = [1, 15, 16, 17, 100, 333, 1000, 2048, 40, 777]
    hq, hkv, d = 12, 2, 128
    store = PagedKVCacheStore(PagedKVAllocator(2048, 16), num_layers=1, num_kv_heads=hkv, head_dim=d,
                              dtype=torch.bfloat16, device=device)
    for sid, n in enumerate(lengths):
        store.reserve(sid, n - 1)
        if n > 1:
            k = torch.randn((1, hkv, n - 1, d), generator=gen).to(torch.bfloat16).to(device)
            v = torch.randn((1, hkv, n - 1, d), generator=gen).to(torch.bfloat16).to(device)
            store.write_sequence_cache(sid, ((k, v),), None)
    b = len(lengths)
    q = torch.randn((b, hq, d), generator=gen).to(torch.bfloat16).to(device)
    kn = torch.randn((b, hkv, d), generator=gen).to(torch.bfloat16).to(device)
    vn = torch.randn((b, hkv, d), generator=gen).to(torch.bfloat16).to(device)
    # A fused step appends the step's tokens and fixes the device tables; the
    # attention-only calls below then all read the same pages.
    _, step = store.decode(list(range(b)), q, kn, vn)
    return store, step, q


def _args(store, step, q, out):
    pool = store.pool
    info = step.info
    rows_t, cols_t = pool.tables.shape
    return [pool._geom_ref, pool.pool.data_ptr(), 0, q.data_ptr(), None, None, pool.tables.data_ptr(), cols_t,
            rows_t, pool.context_lens.data_ptr(), info.rows, info.seq_lens, info.new_blocks, info.items,
            info.n_items, info.n_combine, info.batch, q.shape[1], info.pages_per_split, q.shape[2] ** -0.5,
            out.data_ptr()]


def test_no_alloc_decode_matches_workspace_entry_point(cuda_device):
    from randomrepo_b200._lib import lib, raise_for_status

    store, step, q = _setup(cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    info = step.info
    ws_bytes = lib.pkv_decode_workspace_bytes(info.batch, store.pool.num_kv_heads, store.pool.head_dim,
                                              info.n_items)
    workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda_device)
    want = torch.empty_like(q)
    raise_for_status(lib.pkv_decode_attention(*_args(store, step, q, want), workspace.data_ptr(), ws_bytes, stream))
    torch.cuda.synchronize()
    assert int(workspace[:4].view(torch.int32).item()) == 0
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        raise_for_status(lib.pkv_decode_attention_noalloc(*_args(store, step, q, got), stream))
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), want.float().cpu().numpy(), rtol=RTOL, atol=ATOL)
        assert _noalloc_error(stream) == 0


def _noalloc_error(stream) -> int:
    from randomrepo_b200._lib import lib, raise_for_status

    err = ctypes.c_int32(-1)
    raise_for_status(lib.pkv_decode_noalloc_error(ctypes.byref(err), stream))
    return int(err.value)


def test_no_alloc_reports_a_bad_block_id_and_clears_it_on_the_next_call(cuda_device):
    """A table entry outside the pool is replaced by block 0 in the kernel (no access leaves the pool)
    and reported as error 4; the error word is readable after the call and cleared by the next one."""
    from randomrepo_b200._lib import lib, raise_for_status

    store, step, q = _setup(cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    pool = store.pool
    row = int(step.host_rows[3])  # the 17-token sequence: its page 0 comes from the table
    saved = int(pool.tables[row, 0].item())
    pool.tables[row, 0] = pool.num_blocks + 5
    out = torch.empty_like(q)
    raise_for_status(lib.pkv_decode_attention_noalloc(*_args(store, step, q, out), stream))
    assert _noalloc_error(stream) == 4
    pool.tables[row, 0] = saved
    raise_for_status(lib.pkv_decode_attention_noalloc(*_args(store, step, q, out), stream))
    assert _noalloc_error(stream) == 0


def test_no_alloc_rejects_steps_beyond_its_scratch(cuda_device):
    from randomrepo_b200._lib import PKV_ERR_ARG, last_error, lib

    store, step, q = _setup(cuda_device)
    out = torch.empty_like(q)
    args = _args(store, step, q, out)
    args[14] = 1 << 20  # a plan of a million work items needs far more than 16 MiB of scratch
    status = lib.pkv_decode_attention_noalloc(*args, torch.cuda.current_stream().cuda_stream)
    assert status == PKV_ERR_ARG
    assert "16 MiB static scratch" in last_error()
    torch.cuda.synchronize()
