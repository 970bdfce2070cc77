"""GPU parity of the device store: append / gather / block tables / copy-on-write.

Everything here is integer or byte work, so the bar is bit-exact equality
with the reference's own store outputs (golden fixtures) and with the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.allocator import OracleAllocator
from oracle.store import OracleStore
from tests.conftest import load_npz

pytestmark = pytest.mark.gpu

STORE = load_npz("store_roundtrip.npz")
CASES = {"f32_bs2": (torch.float32, 2, [3, 1, 4]), "bf16_bs16": (torch.bfloat16, 16, [1, 16, 17, 40]),
         "bf16_bs2": (torch.bfloat16, 2, [5, 2])}


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _tensor(bits: np.ndarray, dtype: torch.dtype, device) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(bits.copy()).to(device)


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("io", ["cuda", "cpu"])
def test_store_roundtrip_matches_reference_fixture(cuda_device, name, io):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    dtype, bs, lengths = CASES[name]
    device = cuda_device if io == "cuda" else torch.device("cpu")
    store = PagedKVCacheStore(PagedKVAllocator(64, bs))
    for sid, n in enumerate(lengths):
        view = store.reserve(sid, n)
        assert list(view.physical_blocks) == STORE[f"{name}/{sid}/blocks"].tolist()
    legacies = {}
    for sid, _ in enumerate(lengths):
        legacy = tuple(tuple(_tensor(STORE[f"{name}/{sid}/{li}/{si}"], dtype, device) for si in range(2))
                       for li in range(2))
        legacies[sid] = legacy
        store.write_sequence_cache(sid, legacy, legacy)
    for sid, _ in enumerate(lengths):
        restored = store.read_sequence_legacy_cache(sid)
        for li in range(2):
            for si in range(2):
                got = restored[li][si]
                assert got.device.type == device.type and got.dtype == dtype
                assert np.array_equal(_bits(got), STORE[f"{name}/{sid}/{li}/{si}"])
    batched = store.read_batched_legacy_cache([0]) if len(lengths) else None
    assert batched is not None and np.array_equal(_bits(batched[0][0]), STORE[f"{name}/0/0/0"])


def test_store_error_paths_match_reference(cuda_device):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    store = PagedKVCacheStore(PagedKVAllocator(8, 2))
    store.reserve(0, 4)
    short = torch.zeros((1, 1, 2, 8), device=cuda_device)
    with pytest.raises(ValueError, match="chunk count"):  # paged_kv.py:263-267
        store.write_sequence_cache(0, ((short, short),), None)
    full = torch.arange(32, dtype=torch.float32, device=cuda_device).view(1, 1, 4, 8)
    store.write_sequence_cache(0, ((full, full),), None)
    store.append_tokens(0, 1)  # grows into a block that holds no stored chunk
    with pytest.raises(KeyError):
        store.read_sequence_legacy_cache(0)
    with pytest.raises(KeyError):
        store.release(99)
    with pytest.raises(KeyError):
        store.set_resident_cache(99, None)
    with pytest.raises(ValueError, match="Batched legacy cache"):
        store.write_batched_legacy_cache([0, 1], ((full, full),), None)
    store.release(0)
    assert not store.has_sequence(0)


def test_resident_cache_path(cuda_device):
    """paged_kv.py:218-243,283-292: a resident cache wins over the blocks; clearing writes it back."""
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    store = PagedKVCacheStore(PagedKVAllocator(8, 2))
    store.reserve(1, 3)
    first = (torch.arange(3.0, device=cuda_device).view(1, 1, 3, 1).expand(1, 1, 3, 4).contiguous(),) * 2
    store.write_sequence_cache(1, (first,), (first,))
    store.append_tokens(1, 1)
    resident = ((torch.arange(16.0, device=cuda_device).view(1, 1, 4, 4),
                 torch.arange(16.0, 32.0, device=cuda_device).view(1, 1, 4, 4)),)
    store.set_resident_cache(1, resident, resident)
    got = store.read_sequence_legacy_cache(1)
    assert torch.equal(got[0][0], resident[0][0]) and torch.equal(got[0][1], resident[0][1])
    store.clear_resident_cache(1)
    assert not store.has_resident_cache(1)
    got = store.read_sequence_legacy_cache(1)
    assert torch.equal(got[0][0], resident[0][0]) and torch.equal(got[0][1], resident[0][1])


def _check_device_mirror(store):
    pool = store.pool
    store._sync()
    tables = pool.tables.cpu().numpy()
    lens = pool.context_lens.cpu().numpy()
    refs = pool.refcounts.cpu().numpy()
    alloc = store.allocator
    for sid in list(store._live):
        view = alloc.view(sid)
        row = alloc.row(sid)
        assert lens[row] == view.token_count
        assert tuple(tables[row, : view.logical_block_count]) == view.physical_blocks
    assert [int(r) for r in refs] == [alloc.refcount(b) for b in range(alloc.total_blocks)]


def test_device_tables_follow_host_allocator(cuda_device):
    """Block tables, lengths and refcounts on the device equal the host allocator bit for bit."""
    import random

    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    rng = random.Random(0)
    store = PagedKVCacheStore(PagedKVAllocator(1024, 16), num_layers=2, num_kv_heads=2, head_dim=64,
                              dtype=torch.bfloat16, device=cuda_device)
    store._live = []
    next_id = 0
    for step in range(400):
        r = rng.random()
        if r < 0.25 or not store._live:
            try:
                store.reserve(next_id, rng.randint(0, 200))
                store._live.append(next_id)
            except RuntimeError:  # pool exhausted: the reference's partial effects stay
                pass
            next_id += 1
        elif r < 0.4:
            store.fork(rng.choice(store._live), next_id)
            store._live.append(next_id)
            next_id += 1
        elif r < 0.85:
            try:
                store.append_tokens(rng.choice(store._live), rng.choice([1, 1, 16, rng.randint(0, 40)]))
            except RuntimeError:
                pass
        else:
            sid = rng.choice(store._live)
            store.release(sid)
            store._live.remove(sid)
        if step % 50 == 49:
            _check_device_mirror(store)
    _check_device_mirror(store)


def _rand_bf16(shape, gen):
    return torch.randn(shape, generator=gen).to(torch.bfloat16)


def test_group_fork_cow_matches_oracle(cuda_device):
    """A GRPO group shares its prompt pages; each member's decode appends diverge after a COW copy.

    The semantic pin: every member gathers exactly what an independent prefill
    of the same prompt plus its own appended tokens would hold (the reference
    prefills each member separately, continuous.py:88-99,955-975).
    """
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    gen = torch.Generator().manual_seed(5)
    layers, hkv, d, group = 2, 2, 64, 4
    store = PagedKVCacheStore(PagedKVAllocator(256, 16))
    ora = OracleStore(OracleAllocator(256, 16))
    prompt_len = 37
    prompt = tuple((_rand_bf16((1, hkv, prompt_len, d), gen), _rand_bf16((1, hkv, prompt_len, d), gen))
                   for _ in range(layers))
    store.reserve(0, prompt_len)
    store.write_sequence_cache(0, tuple((k.to(cuda_device), v.to(cuda_device)) for k, v in prompt), None)
    ora.allocator.reserve(0, prompt_len)
    ora.write_sequence_cache(0, tuple((_bits(k), _bits(v)) for k, v in prompt))
    for m in range(1, group):
        store.fork(0, m)
        ora.allocator.fork(0, m)
    q = torch.zeros((group, hkv * 2, d), dtype=torch.bfloat16, device=cuda_device)
    for _ in range(20):
        step = store.decode_step(list(range(group)))
        for m in range(group):
            ora.allocator.append_tokens(m, 1)
        while ora.allocator.cow_log:
            _sid, src, dst = ora.allocator.cow_log.pop(0)
            ora.copy_block(src, dst)
        for layer in range(layers):
            kn = _rand_bf16((group, hkv, d), gen)
            vn = _rand_bf16((group, hkv, d), gen)
            store.decode_attention(step, layer, q, kn.to(cuda_device), vn.to(cuda_device))
            for m in range(group):
                ora.append_token(m, layer, _bits(kn[m]), _bits(vn[m]))
    for m in range(group):
        assert store.allocator.view(m).physical_blocks == ora.allocator.view(m).physical_blocks
        got = store.read_sequence_legacy_cache(m)
        want = ora.read_sequence_legacy_cache(m)
        for li in range(layers):
            for si in range(2):
                assert np.array_equal(_bits(got[li][si]), want[li][si]), (m, li, si)
        # the shared prompt pages are the parent's
        assert np.array_equal(_bits(got[0][0])[:, :, :32], _bits(prompt[0][0])[:, :, :32])
    assert store.allocator.refcount(0) == group and store.allocator.refcount(1) == group
    for m in range(group):
        store.release(m)
    assert store.allocator.free_block_count == 256


def test_scatter_gather_roundtrip_at_microbench_scale(cuda_device):
    """Size-independent property at the microbench's scale: gather(scatter(x)) == x for 256 ragged sequences."""
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    gen = torch.Generator().manual_seed(11)
    lengths = torch.randint(64, 2049, (256,), generator=gen).tolist()
    store = PagedKVCacheStore(PagedKVAllocator(40000, 16))
    hkv, d = 2, 128
    checks = []
    for sid, n in enumerate(lengths):
        store.reserve(sid, n)
        k = torch.randn((1, hkv, n, d), generator=gen, dtype=torch.float32).to(torch.bfloat16).to(cuda_device)
        v = torch.randn((1, hkv, n, d), generator=gen, dtype=torch.float32).to(torch.bfloat16).to(cuda_device)
        store.write_sequence_cache(sid, ((k, v),), None)
        if sid % 37 == 0:
            checks.append((sid, k, v))
    for sid, k, v in checks:
        got = store.read_sequence_legacy_cache(sid)
        assert torch.equal(got[0][0], k) and torch.equal(got[0][1], v)
    total_blocks = sum((n + 15) // 16 for n in lengths)
    assert store.allocator.used_block_count == total_blocks
