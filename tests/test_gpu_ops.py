"""``torch.ops.pkv`` operators on the GPU give exactly what the store's own calls give (same kernels, same
plans): the append and gather bit-exact against the store's pages, decode and prefill / verify attention
bit-identical to the store path and within the attention tolerance of the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention as oracle_decode

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _store(device, lengths, hkv=2, d=128, seed=0):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    gen = torch.Generator().manual_seed(seed)
    store = PagedKVCacheStore(PagedKVAllocator(1024, 16), num_layers=1, num_kv_heads=hkv, head_dim=d,
                              dtype=torch.bfloat16, device=device)
    kv = []
    for sid, n in enumerate(lengths):
        k = torch.randn((1, hkv, n, d), generator=gen).to(torch.bfloat16)
        v = torch.randn((1, hkv, n, d), generator=gen).to(torch.bfloat16)
        store.reserve(sid, n)
        store.write_sequence_cache(sid, ((k.to(device), v.to(device)),), None)
        kv.append((k, v))
    return store, kv


def _slots(store, sid) -> torch.Tensor:
    view = store.allocator.view(sid)
    t = np.arange(view.token_count)
    blocks = np.array(view.physical_blocks, dtype=np.int64)
    return torch.from_numpy(blocks[t // 16] * 16 + t % 16)


def test_gather_append_and_copy_blocks_ops(cuda_device):
    from randomrepo_b200.ops import pool_geom

    store, kv = _store(cuda_device, [40, 17])
    pool = store.pool
    geom = pool_geom(pool)
    k, v = torch.ops.pkv.kv_gather(pool.pool, geom, 0, _slots(store, 0).to(cuda_device))
    assert torch.equal(k.cpu(), kv[0][0][0].permute(1, 0, 2)) and torch.equal(v.cpu(), kv[0][1][0].permute(1, 0, 2))
    # append two rows to sequence 1 through the op, read them back through the store
    store.append_tokens(1, 2)
    new_k = torch.randn((2, 2, 128), device=cuda_device).to(torch.bfloat16)
    new_v = torch.randn((2, 2, 128), device=cuda_device).to(torch.bfloat16)
    slots = _slots(store, 1)[-2:].to(cuda_device)
    torch.ops.pkv.kv_append(pool.pool, geom, 0, new_k, new_v, slots)
    k2, v2 = torch.ops.pkv.kv_gather(pool.pool, geom, 0, slots)
    assert torch.equal(k2, new_k) and torch.equal(v2, new_v)
    # whole-block copy: block of sequence 0's first page -> a free block
    src = torch.tensor([store.allocator.view(0).physical_blocks[0]], dtype=torch.int32, device=cuda_device)
    dst = torch.tensor([1000], dtype=torch.int32, device=cuda_device)
    torch.ops.pkv.copy_blocks(pool.pool, geom, src, dst)
    a, _ = torch.ops.pkv.kv_gather(pool.pool, geom, 0, (src.long() * 16 + torch.arange(16, device=cuda_device)))
    b, _ = torch.ops.pkv.kv_gather(pool.pool, geom, 0, (dst.long() * 16 + torch.arange(16, device=cuda_device)))
    assert torch.equal(a, b)


def test_decode_attention_op_equals_the_store_path(cuda_device):
    from randomrepo_b200._lib import lib
    from randomrepo_b200.device import plan_decode
    from randomrepo_b200.ops import pool_geom

    lengths = [1, 15, 16, 17, 100, 700, 2048]
    store, kv = _store(cuda_device, lengths, seed=3)
    gen = torch.Generator().manual_seed(4)
    b = len(lengths)
    q = torch.randn((b, 12, 128), generator=gen).to(torch.bfloat16).to(cuda_device)
    kn = torch.randn((b, 2, 128), generator=gen).to(torch.bfloat16).to(cuda_device)
    vn = torch.randn((b, 2, 128), generator=gen).to(torch.bfloat16).to(cuda_device)
    want, step = store.decode(list(range(b)), q, kn, vn)
    pool = store.pool
    lens = step.host_lens.astype(np.int32)
    pps, items, n_items, n_combine = plan_decode(lens, 2, pool.num_sms)
    ws = torch.zeros(int(lib.pkv_decode_workspace_bytes(b, 2, 128, n_items)), dtype=torch.uint8, device=cuda_device)
    i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(cuda_device)  # noqa: E731
    got = torch.ops.pkv.decode_attention(pool.pool, pool_geom(pool), 0, q, None, None, pool.tables,
                                         pool.context_lens, i32(step.host_rows), i32(lens), None, i32(items),
                                         n_items, n_combine, pps, 128 ** -0.5, ws)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert int(ws[:4].view(torch.int32).item()) == 0
    for i in range(b):
        kk = torch.cat([kv[i][0][0].permute(1, 0, 2), kn[i:i + 1].cpu()]).float().numpy()
        vv = torch.cat([kv[i][1][0].permute(1, 0, 2), vn[i:i + 1].cpu()]).float().numpy()
        np.testing.assert_allclose(got[i].float().cpu().numpy(),
                                   oracle_decode(q[i].float().cpu().numpy(), kk, vv, 128 ** -0.5), rtol=RTOL,
                                   atol=ATOL)


def test_prefill_attention_op_equals_the_store_path(cuda_device):
    """A verify-shaped read: 5 queries after prefix - 1 cached tokens per sequence."""
    from randomrepo_b200.device import plan_prefill
    from randomrepo_b200.ops import pool_geom

    lengths = [130, 300, 1000]
    store, _ = _store(cuda_device, lengths, seed=5)
    pool = store.pool
    store._sync()
    rows = np.array([store.allocator.row(s) for s in range(3)])
    past = np.array([n - 5 for n in lengths])
    qls = np.full(3, 5)
    plan = plan_prefill(rows, past, qls, 12, 2, pool.num_sms)
    records = torch.from_numpy(plan.records).to(cuda_device)
    q = torch.randn((15, 12, 128), generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).to(cuda_device)
    want = torch.empty_like(q)
    pool.prefill(0, q, plan, records, 12, 128 ** -0.5, want)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ws = torch.empty(0, dtype=torch.uint8, device=cuda_device)
    got = torch.ops.pkv.prefill_attention(pool.pool, pool_geom(pool), 0, q, pool.tables, records, plan.n_items,
                                          plan.n_combine, plan.n_slots, 128 ** -0.5, err, ws)
    torch.cuda.synchronize()
    assert torch.equal(got, want) and int(err.item()) == 0 and pool.prefill_error_flag() == 0


@pytest.mark.parametrize("lengths", [[130, 300, 1000], [5000, 9000, 300, 17]])
def test_verify_attention_op_equals_the_store_path(cuda_device, lengths):
    """The verify kernel through the operator: whole items, and long prefixes whose key ranges are
    cut and merged (workspace partials and the combine launch)."""
    from randomrepo_b200._lib import lib
    from randomrepo_b200.device import plan_verify
    from randomrepo_b200.ops import pool_geom

    store, _ = _store(cuda_device, lengths, seed=7)
    pool = store.pool
    store._sync()
    n = len(lengths)
    rows = np.array([store.allocator.row(s) for s in range(n)])
    past = np.array([m - 5 for m in lengths])
    qls = np.full(n, 5)
    plan = plan_verify(rows, past, qls, 12, 2, pool.num_sms)
    assert (plan.n_combine > 0) == (max(lengths) > 2000)
    records = torch.from_numpy(plan.records).to(cuda_device)
    q = torch.randn((5 * n, 12, 128), generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).to(cuda_device)
    want = torch.empty_like(q)
    pool.prefill(0, q, plan, records, 12, 128 ** -0.5, want)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ws = torch.empty(max(1, int(lib.pkv_prefill_workspace_bytes(plan.n_slots, 128))), dtype=torch.uint8,
                     device=cuda_device)
    got = torch.ops.pkv.verify_attention(pool.pool, pool_geom(pool), 0, q, pool.tables, records, plan.n_items,
                                         plan.n_ctas, plan.n_combine, plan.n_slots, 128 ** -0.5, err, ws)
    torch.cuda.synchronize()
    assert torch.equal(got, want) and int(err.item()) == 0 and pool.prefill_error_flag() == 0

