"""GPU parity of the verify kernel (pkv_verify_attention: keys on the tensor-core rows).

Floating-point bar as for the prefill kernel: |out - oracle| <= 2e-2 + 1e-2 *
|oracle| elementwise (bf16/f16 inputs and probabilities, fp32 accumulation in
tensor memory).  The oracle is oracle/attention.py's verify_attention (HF
``sdpa_attention_forward`` with a causal mask after prefix_len-1 cached
tokens); the HF golden verify fixtures run through this kernel in
tests/test_gpu_prefill.py.  Cases cover every head grouping up to 32 query
columns, prefixes on and around page (16) and KV-tile (128) boundaries, long
prefixes whose keys are cut across CTAs (partials merged by the combine
kernel) and the same launch without the cut, f16 pools, forked prefixes and
the second layer of a pool.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import verify_attention

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2

PREFIXES = [1, 2, 15, 16, 17, 100, 127, 128, 129, 255, 256, 257, 700, 1280, 3001]

SHAPES = [
    # (hq, hkv, k drafts, dtype): query columns per item = (k + 1) * hq / hkv <= 32
    (12, 2, 4, torch.bfloat16),   # Qwen2.5-1.5B target: 30 columns
    (12, 2, 0, torch.bfloat16),   # one query per sequence: 6 columns
    (28, 4, 3, torch.bfloat16),   # Qwen2.5-7B grouping, 28 columns
    (16, 2, 3, torch.float16),    # exactly 32 columns, f16
    (32, 1, 0, torch.bfloat16),   # 32 heads of one position
    (8, 8, 31, torch.bfloat16),   # no grouping, 32 positions
    (4, 2, 9, torch.float16),     # 20 columns
]


def _np32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _make_store(hkv, dtype, device, layers=1, blocks=16384):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    return PagedKVCacheStore(PagedKVAllocator(blocks, 16), num_layers=layers, num_kv_heads=hkv, head_dim=128,
                             dtype=dtype, device=device)


def _write(store, sid, k, v, layer=0):
    t = k.shape[0]
    store.reserve(sid, t)
    if t:
        pool = store.pool
        kk = torch.zeros((pool.num_layers, pool.num_kv_heads, t, pool.head_dim), dtype=k.dtype, device=k.device)
        vv = torch.zeros_like(kk)
        kk[layer] = k.permute(1, 0, 2)
        vv[layer] = v.permute(1, 0, 2)
        store.write_sequence_cache(sid, tuple((kk[i:i + 1], vv[i:i + 1]) for i in range(pool.num_layers)), None)


def _run(store, prefixes, hq, hkv, kd, dtype, gen, device, layer=0, fork_from=None):
    """Write the prefixes (or fork them), verify k+1 queries each; returns (out, q, ks, vs)."""
    ks, vs = [], []
    for sid, pre in enumerate(prefixes):
        k = torch.randn((pre + kd, hkv, 128), generator=gen).to(dtype)
        v = torch.randn((pre + kd, hkv, 128), generator=gen).to(dtype)
        if fork_from is not None:
            k[: pre - 1], v[: pre - 1] = fork_from[0][: pre - 1], fork_from[1][: pre - 1]
            store.fork(1000, sid)
        else:
            _write(store, sid, k[: pre - 1].to(device), v[: pre - 1].to(device), layer=layer)
        store.append_tokens(sid, kd + 1)
        ks.append(k), vs.append(v)
    b = len(prefixes)
    q = torch.randn((b, kd + 1, hq, 128), generator=gen).to(dtype)
    kn = torch.stack([k[p - 1:] for k, p in zip(ks, prefixes)])
    vn = torch.stack([v[p - 1:] for v, p in zip(vs, prefixes)])
    out = store.verify_attention(list(range(b)), q.to(device), kn.to(device), vn.to(device), layer=layer)
    torch.cuda.synchronize()
    return out, q, ks, vs


def _check(out, q, ks, vs, prefixes, store):
    got = _np32(out)
    for sid, pre in enumerate(prefixes):
        want = verify_attention(_np32(q[sid]), _np32(ks[sid]), _np32(vs[sid]), 128 ** -0.5, pre)
        np.testing.assert_allclose(got[sid], want, rtol=RTOL, atol=ATOL, err_msg=f"prefix {pre}")
    assert store.pool.prefill_error_flag() == 0


def _planned_kind(store, prefixes, kd, hq):
    step = store.prefill_step(list(range(len(prefixes))), np.full(len(prefixes), kd + 1), hq)
    return step.plan


@pytest.mark.parametrize("shape", range(len(SHAPES)))
@pytest.mark.parametrize("num_sms", ["device", 0, 1])
def test_verify_kernel_matches_oracle(cuda_device, monkeypatch, shape, num_sms):
    """Every prefix edge case in one launch: a persistent grid with key ranges cut (device SMs), one
    CTA per item (0), and one CTA working through every item of the launch (1)."""
    hq, hkv, kd, dtype = SHAPES[shape]
    gen = torch.Generator().manual_seed(300 + shape)
    store = _make_store(hkv, dtype, cuda_device)
    if num_sms != "device":
        monkeypatch.setattr(store.pool, "num_sms", num_sms)
    out, q, ks, vs = _run(store, PREFIXES, hq, hkv, kd, dtype, gen, cuda_device)
    _check(out, q, ks, vs, PREFIXES, store)


def test_verify_kernel_is_the_one_planned(cuda_device):
    """Verify-shaped steps plan for the verify kernel; the long prefix is cut into ranges."""
    store = _make_store(2, torch.bfloat16, cuda_device)
    for sid, pre in enumerate(PREFIXES):
        store.reserve(sid, pre - 1)
        store.append_tokens(sid, 5)
    plan = _planned_kind(store, PREFIXES, 4, 12)
    assert plan.kind == "verify" and plan.n_combine > 0 and plan.n_slots > 0


def test_many_sequences_split_across_the_grid(cuda_device):
    """The bench's verify shape (64 sequences, prefix U[128, 1280], k = 4) plus long prefixes to 8192."""
    rng = np.random.default_rng(11)
    prefixes = [int(p) for p in rng.integers(128, 1281, size=64)] + [4096, 8192, 6000]
    gen = torch.Generator().manual_seed(12)
    store = _make_store(2, torch.bfloat16, cuda_device, blocks=32768)
    out, q, ks, vs = _run(store, prefixes, 12, 2, 4, torch.bfloat16, gen, cuda_device)
    _check(out, q, ks, vs, prefixes, store)


def test_verify_kernel_equals_prefill_kernel(cuda_device, monkeypatch):
    """The two kernels agree with each other as closely as with the oracle."""
    import randomrepo_b200.device as devmod

    prefixes = [3, 64, 200, 999, 1500]
    outs = []
    for flag in (True, False):
        monkeypatch.setattr(devmod, "VERIFY_KERNEL", flag)
        gen = torch.Generator().manual_seed(77)
        store = _make_store(2, torch.bfloat16, cuda_device)
        out, q, ks, vs = _run(store, prefixes, 12, 2, 4, torch.bfloat16, gen, cuda_device)
        _check(out, q, ks, vs, prefixes, store)
        outs.append(_np32(out))
    np.testing.assert_allclose(outs[0], outs[1], rtol=RTOL, atol=ATOL)


def test_verify_over_forked_prefixes(cuda_device):
    """Group members forked from one prompt read the shared blocks (and their own copied tails)."""
    hq, hkv, kd = 12, 2, 4
    gen = torch.Generator().manual_seed(41)
    prompt = 333  # ends inside a block: each child's appends copy that block first
    store = _make_store(hkv, torch.bfloat16, cuda_device)
    pk = torch.randn((prompt, hkv, 128), generator=gen).to(torch.bfloat16)
    pv = torch.randn((prompt, hkv, 128), generator=gen).to(torch.bfloat16)
    _write(store, 1000, pk.to(cuda_device), pv.to(cuda_device))
    prefixes = [prompt + 1] * 8
    out, q, ks, vs = _run(store, prefixes, hq, hkv, kd, torch.bfloat16, gen, cuda_device, fork_from=(pk, pv))
    _check(out, q, ks, vs, prefixes, store)
    (k0, v0), = store.read_sequence_legacy_cache(1000)
    assert torch.equal(k0[0].permute(1, 0, 2).cpu(), pk) and torch.equal(v0[0].permute(1, 0, 2).cpu(), pv)


def test_verify_on_second_layer(cuda_device):
    """Layer offsets: only layer 1's pages are read."""
    gen = torch.Generator().manual_seed(8)
    store = _make_store(2, torch.bfloat16, cuda_device, layers=2)
    prefixes = [90, 260, 1300]
    out, q, ks, vs = _run(store, prefixes, 12, 2, 4, torch.bfloat16, gen, cuda_device, layer=1)
    _check(out, q, ks, vs, prefixes, store)


def test_verify_rejects_unsupported_geometry(cuda_device):
    """head_dim 64 is not the verify kernel's: the step plans for the prefill kernel instead."""
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore
    from randomrepo_b200.device import verify_supported

    assert not verify_supported(12, 2, 64, 16, 5)
    assert not verify_supported(66, 2, 128, 16, 1)  # 33 query heads per KV head
    assert not verify_supported(12, 2, 128, 16, 6)  # 36 columns
    store = PagedKVCacheStore(PagedKVAllocator(256, 16), num_layers=1, num_kv_heads=2, head_dim=64,
                              dtype=torch.bfloat16, device=cuda_device)
    store.reserve(0, 40)
    store.append_tokens(0, 5)
    assert store.prefill_step([0], [5], 12).plan.kind == "prefill"
