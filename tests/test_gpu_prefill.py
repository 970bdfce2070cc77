"""GPU parity of chunked-prefill and speculative-verify attention over pages.

Floating-point bar: |out - oracle| <= 2e-2 + 1e-2 * |oracle| elementwise
(bf16/f16 inputs, fp32 accumulation in tensor memory).  The oracle is the fp32
restatement of HF ``sdpa_attention_forward`` with a causal mask after a cached
past (oracle/attention.py, pinned to the reference by
tests/test_oracle_golden.py); the golden HF outputs of the chunked-prefill and
verify fixtures are also checked directly.  The chunk's K/V rows written into
the pages are compared bit-exactly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import bf16_to_f32, prefill_attention, verify_attention
from tests.conftest import load_npz

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
ATTN = load_npz("attention_sdpa.npz")


def _np32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _from_bits(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)


def _make_store(hkv, d, dtype, device, blocks=8192, layers=1):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    return PagedKVCacheStore(PagedKVAllocator(blocks, 16), num_layers=layers, num_kv_heads=hkv, head_dim=d,
                             dtype=dtype, device=device)


def _write(store, sid, k, v, layer=0):
    """Reserve ``k.shape[0]`` tokens for a new sequence and write them (k/v [T, Hkv, D])."""
    t = k.shape[0]
    store.reserve(sid, t)
    if t:
        pool = store.pool
        kk = torch.zeros((pool.num_layers, pool.num_kv_heads, t, pool.head_dim), dtype=k.dtype, device=k.device)
        vv = torch.zeros_like(kk)
        kk[layer] = k.permute(1, 0, 2)
        vv[layer] = v.permute(1, 0, 2)
        store.write_sequence_cache(sid, tuple((kk[i:i + 1], vv[i:i + 1]) for i in range(pool.num_layers)), None)


n_prefill = len({k.split("/")[1] for k in ATTN if k.startswith("prefill/")})
n_verify = len({k.split("/")[1] for k in ATTN if k.startswith("verify/")})


@pytest.mark.parametrize("i", range(n_prefill))
def test_prefill_matches_hf_sdpa_fixture(cuda_device, i):
    past = int(ATTN[f"prefill/{i}/past"])
    q = _from_bits(ATTN[f"prefill/{i}/q"], cuda_device)   # [Tq, Hq, D]
    k = _from_bits(ATTN[f"prefill/{i}/k"], cuda_device)   # [past + Tq, Hkv, D]
    v = _from_bits(ATTN[f"prefill/{i}/v"], cuda_device)
    tq = q.shape[0]
    store = _make_store(k.shape[1], k.shape[2], torch.bfloat16, cuda_device)
    _write(store, 0, k[:past], v[:past])
    store.append_tokens(0, tq)
    out = store.prefill_attention([0], q.contiguous(), k[past:].contiguous(), v[past:].contiguous())
    torch.cuda.synchronize()
    np.testing.assert_allclose(_np32(out), ATTN[f"prefill/{i}/o"], rtol=RTOL, atol=ATOL)
    assert store.pool.prefill_error_flag() == 0


@pytest.mark.parametrize("i", range(n_verify))
def test_verify_matches_hf_sdpa_fixture(cuda_device, i):
    prefix = int(ATTN[f"verify/{i}/prefix"])
    q = _from_bits(ATTN[f"verify/{i}/q"], cuda_device)    # [k+1, Hq, D]
    k = _from_bits(ATTN[f"verify/{i}/k"], cuda_device)    # [prefix + k, Hkv, D]
    v = _from_bits(ATTN[f"verify/{i}/v"], cuda_device)
    t = q.shape[0]
    store = _make_store(k.shape[1], k.shape[2], torch.bfloat16, cuda_device)
    _write(store, 7, k[: prefix - 1], v[: prefix - 1])
    store.append_tokens(7, t)
    out = store.verify_attention([7], q.unsqueeze(0).contiguous(), k[prefix - 1:].unsqueeze(0).contiguous(),
                                 v[prefix - 1:].unsqueeze(0).contiguous())
    torch.cuda.synchronize()
    np.testing.assert_allclose(_np32(out[0]), ATTN[f"verify/{i}/o"], rtol=RTOL, atol=ATOL)


CASES = [
    # (hq, hkv, d, dtype, [(past, chunk), ...])
    (12, 2, 128, torch.bfloat16, [(0, 1), (0, 16), (0, 21), (15, 22), (100, 37), (0, 300), (1000, 512), (129, 127)]),
    (14, 2, 64, torch.bfloat16, [(0, 5), (200, 64), (511, 18), (37, 1)]),
    (28, 4, 128, torch.bfloat16, [(256, 40), (0, 19), (4000, 96)]),
    (12, 2, 128, torch.float16, [(33, 50), (0, 8)]),
    (8, 8, 128, torch.bfloat16, [(5, 130), (250, 3)]),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_prefill_matches_oracle(cuda_device, case):
    hq, hkv, d, dtype, seqs = CASES[case]
    gen = torch.Generator().manual_seed(100 + case)
    store = _make_store(hkv, d, dtype, cuda_device)
    ks, vs, qs = [], [], []
    for sid, (past, chunk) in enumerate(seqs):
        k = torch.randn((past + chunk, hkv, d), generator=gen).to(dtype)
        v = torch.randn((past + chunk, hkv, d), generator=gen).to(dtype)
        q = torch.randn((chunk, hq, d), generator=gen).to(dtype)
        _write(store, sid, k[:past].to(cuda_device), v[:past].to(cuda_device))
        store.append_tokens(sid, chunk)
        ks.append(k), vs.append(v), qs.append(q)
    q = torch.cat(qs).to(cuda_device)
    kc = torch.cat([k[p:] for k, (p, _) in zip(ks, seqs)]).to(cuda_device)
    vc = torch.cat([v[p:] for v, (p, _) in zip(vs, seqs)]).to(cuda_device)
    out = store.prefill_attention(list(range(len(seqs))), q, kc, vc, q_lens=[c for _, c in seqs])
    torch.cuda.synchronize()
    got = _np32(out)
    scale = d ** -0.5
    off = 0
    for sid, (past, chunk) in enumerate(seqs):
        want = prefill_attention(_np32(qs[sid]), _np32(ks[sid]), _np32(vs[sid]), scale, past)
        np.testing.assert_allclose(got[off:off + chunk], want, rtol=RTOL, atol=ATOL,
                                   err_msg=f"sequence {sid} (past {past}, chunk {chunk})")
        off += chunk
    assert store.pool.prefill_error_flag() == 0
    # The chunk's K/V rows landed bit-exactly in the pages.
    for sid, (past, chunk) in enumerate(seqs):
        (kk, vv), = store.read_sequence_legacy_cache(sid)
        assert torch.equal(kk[0].permute(1, 0, 2).cpu(), ks[sid])
        assert torch.equal(vv[0].permute(1, 0, 2).cpu(), vs[sid])


def test_chunked_prefill_equals_one_shot(cuda_device):
    """A 700-token prompt prefilled in chunks of 256 gives the rows of one causal pass."""
    hq, hkv, d = 12, 2, 128
    gen = torch.Generator().manual_seed(5)
    n = 700
    k = torch.randn((n, hkv, d), generator=gen).to(torch.bfloat16)
    v = torch.randn((n, hkv, d), generator=gen).to(torch.bfloat16)
    q = torch.randn((n, hq, d), generator=gen).to(torch.bfloat16)
    store = _make_store(hkv, d, torch.bfloat16, cuda_device)
    store.reserve(0, 0)
    parts = []
    for c0 in range(0, n, 256):
        c1 = min(n, c0 + 256)
        store.append_tokens(0, c1 - c0)
        parts.append(store.prefill_attention([0], q[c0:c1].to(cuda_device), k[c0:c1].to(cuda_device),
                                             v[c0:c1].to(cuda_device)))
    got = _np32(torch.cat(parts))
    want = prefill_attention(_np32(q), _np32(k), _np32(v), d ** -0.5, 0)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_verify_batch_matches_oracle(cuda_device):
    """Speculative verify at the 1.5B target shape: k = 4 drafts, 5 query rows per sequence."""
    hq, hkv, d, kd = 12, 2, 128, 4
    gen = torch.Generator().manual_seed(9)
    prefixes = [128, 129, 700, 1024, 1280, 5, 16, 17]
    store = _make_store(hkv, d, torch.bfloat16, cuda_device)
    ks, vs = [], []
    for sid, pre in enumerate(prefixes):
        k = torch.randn((pre + kd, hkv, d), generator=gen).to(torch.bfloat16)
        v = torch.randn((pre + kd, hkv, d), generator=gen).to(torch.bfloat16)
        _write(store, sid, k[: pre - 1].to(cuda_device), v[: pre - 1].to(cuda_device))
        store.append_tokens(sid, kd + 1)
        ks.append(k), vs.append(v)
    b = len(prefixes)
    q = torch.randn((b, kd + 1, hq, d), generator=gen).to(torch.bfloat16)
    kn = torch.stack([k[p - 1:] for k, p in zip(ks, prefixes)])
    vn = torch.stack([v[p - 1:] for v, p in zip(vs, prefixes)])
    out = store.verify_attention(list(range(b)), q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    torch.cuda.synchronize()
    got = _np32(out)
    for sid, pre in enumerate(prefixes):
        want = verify_attention(_np32(q[sid]), _np32(ks[sid]), _np32(vs[sid]), d ** -0.5, pre)
        np.testing.assert_allclose(got[sid], want, rtol=RTOL, atol=ATOL, err_msg=f"prefix {pre}")
    # Rejecting the drafts (keep the accepted token plus one draft) leaves the pages of the kept prefix.
    store.truncate(list(range(b)), [p + 1 for p in prefixes])
    for sid, pre in enumerate(prefixes):
        (kk, _), = store.read_sequence_legacy_cache(sid)
        assert torch.equal(kk[0].permute(1, 0, 2).cpu(), ks[sid][: pre + 1])


def test_prefill_into_forked_child_keeps_parent(cuda_device):
    """A group member's chunk written after a copy-on-write fork leaves the shared prompt intact."""
    hq, hkv, d = 12, 2, 128
    gen = torch.Generator().manual_seed(21)
    prompt = 40  # ends inside a block: the child's first chunk write copies that block
    k = torch.randn((prompt, hkv, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    v = torch.randn((prompt, hkv, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    store = _make_store(hkv, d, torch.bfloat16, cuda_device)
    _write(store, 0, k, v)
    store.fork(0, 1)
    chunk = 9
    kc = torch.randn((chunk, hkv, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    vc = torch.randn((chunk, hkv, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    qc = torch.randn((chunk, hq, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    store.append_tokens(1, chunk)
    out = store.prefill_attention([1], qc, kc, vc)
    torch.cuda.synchronize()
    want = prefill_attention(_np32(qc), _np32(torch.cat([k, kc])), _np32(torch.cat([v, vc])), d ** -0.5, prompt)
    np.testing.assert_allclose(_np32(out), want, rtol=RTOL, atol=ATOL)
    (pk, pv), = store.read_sequence_legacy_cache(0)
    assert torch.equal(pk[0].permute(1, 0, 2), k) and torch.equal(pv[0].permute(1, 0, 2), v)
    (ck, _), = store.read_sequence_legacy_cache(1)
    assert torch.equal(ck[0].permute(1, 0, 2), torch.cat([k, kc]))


def test_prefill_on_second_layer(cuda_device):
    """Layer offsets: a two-layer pool, attention over layer 1 only sees layer 1's pages."""
    hq, hkv, d = 12, 2, 128
    gen = torch.Generator().manual_seed(3)
    store = _make_store(hkv, d, torch.bfloat16, cuda_device, layers=2)
    past, chunk = 70, 33
    k = torch.randn((past + chunk, hkv, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    v = torch.randn((past + chunk, hkv, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    q = torch.randn((chunk, hq, d), generator=gen).to(torch.bfloat16).to(cuda_device)
    _write(store, 0, k[:past], v[:past], layer=1)
    store.append_tokens(0, chunk)
    out = store.prefill_attention([0], q, k[past:].contiguous(), v[past:].contiguous(), layer=1)
    want = prefill_attention(_np32(q), _np32(k), _np32(v), d ** -0.5, past)
    np.testing.assert_allclose(_np32(out), want, rtol=RTOL, atol=ATOL)


def test_prefill_rejects_unreserved_chunk(cuda_device):
    store = _make_store(2, 128, torch.bfloat16, cuda_device)
    store.reserve(0, 3)
    q = torch.zeros((5, 12, 128), dtype=torch.bfloat16, device=cuda_device)
    kv = torch.zeros((5, 2, 128), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        store.prefill_attention([0], q, kv, kv)


@pytest.mark.parametrize("waves", [1, 2, 3])
def test_key_split_verify_matches_oracle(cuda_device, monkeypatch, waves):
    """Verify with each sequence's keys cut across CTAs (partials merged by the combine kernel)."""
    import randomrepo_b200.device as devmod

    monkeypatch.setattr(devmod, "PREFILL_SPLIT_WAVES", waves)
    hq, hkv, d, kd = 12, 2, 128, 4
    gen = torch.Generator().manual_seed(40 + waves)
    prefixes = [128, 300, 700, 1024, 1280, 5, 17, 129, 555, 1111]
    store = _make_store(hkv, d, torch.bfloat16, cuda_device)
    ks, vs = [], []
    for sid, pre in enumerate(prefixes):
        k = torch.randn((pre + kd, hkv, d), generator=gen).to(torch.bfloat16)
        v = torch.randn((pre + kd, hkv, d), generator=gen).to(torch.bfloat16)
        _write(store, sid, k[: pre - 1].to(cuda_device), v[: pre - 1].to(cuda_device))
        store.append_tokens(sid, kd + 1)
        ks.append(k), vs.append(v)
    b = len(prefixes)
    q = torch.randn((b, kd + 1, hq, d), generator=gen).to(torch.bfloat16)
    kn = torch.stack([k[p - 1:] for k, p in zip(ks, prefixes)])
    vn = torch.stack([v[p - 1:] for v, p in zip(vs, prefixes)])
    out = store.verify_attention(list(range(b)), q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    torch.cuda.synchronize()
    got = _np32(out)
    for sid, pre in enumerate(prefixes):
        want = verify_attention(_np32(q[sid]), _np32(ks[sid]), _np32(vs[sid]), d ** -0.5, pre)
        np.testing.assert_allclose(got[sid], want, rtol=RTOL, atol=ATOL, err_msg=f"prefix {pre}")
    assert store.pool.prefill_error_flag() == 0

