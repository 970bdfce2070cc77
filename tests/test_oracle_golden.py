"""Pin the oracle against golden fixtures produced by the reference itself.

* store round trips: ``PagedKVCacheStore`` write/read outputs (bit patterns);
* attention: HF ``sdpa_attention_forward`` (the reference's attention) outputs
  for GQA decode, chunked prefill after a cached past and the verify rows.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.allocator import OracleAllocator
from oracle.attention import bf16_to_f32, decode_attention, f32_to_bf16, prefill_attention, verify_attention
from oracle.store import OracleStore
from tests.conftest import load_npz

STORE = load_npz("store_roundtrip.npz")
ATTN = load_npz("attention_sdpa.npz")
CASES = {"f32_bs2": (2, [3, 1, 4]), "bf16_bs16": (16, [1, 16, 17, 40]), "bf16_bs2": (2, [5, 2])}


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_store_roundtrip_matches_reference(name):
    bs, lengths = CASES[name]
    store = OracleStore(OracleAllocator(64, bs))
    for sid, n in enumerate(lengths):
        store.allocator.reserve(sid, n)
        assert list(store.allocator.view(sid).physical_blocks) == STORE[f"{name}/{sid}/blocks"].tolist()
    for sid, _ in enumerate(lengths):
        legacy = tuple(tuple(STORE[f"{name}/{sid}/{li}/{si}"] for si in range(2)) for li in range(2))
        store.write_sequence_cache(sid, legacy)
    for sid, _ in enumerate(lengths):
        restored = store.read_sequence_legacy_cache(sid)
        for li in range(2):
            for si in range(2):
                expect = STORE[f"{name}/{sid}/{li}/{si}"]
                assert restored[li][si].dtype == expect.dtype
                assert np.array_equal(restored[li][si], expect)


def test_oracle_store_chunk_mismatch_raises():  # paged_kv.py:263-267
    store = OracleStore(OracleAllocator(8, 2))
    store.allocator.reserve(0, 4)
    short = np.zeros((1, 1, 2, 1), np.float32)
    with pytest.raises(ValueError, match="chunk count"):
        store.write_sequence_cache(0, ((short, short),))


def _n(prefix):
    return len({k.split("/")[1] for k in ATTN if k.startswith(prefix + "/")})


@pytest.mark.parametrize("i", range(_n("decode")))
def test_oracle_decode_matches_hf_sdpa(i):
    q, k, v = (bf16_to_f32(ATTN[f"decode/{i}/{x}"]) for x in "qkv")
    out = decode_attention(q, k, v, q.shape[-1] ** -0.5)
    np.testing.assert_allclose(out, ATTN[f"decode/{i}/o"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("i", range(_n("prefill")))
def test_oracle_prefill_matches_hf_sdpa(i):
    q, k, v = (bf16_to_f32(ATTN[f"prefill/{i}/{x}"]) for x in "qkv")
    out = prefill_attention(q, k, v, q.shape[-1] ** -0.5, past=int(ATTN[f"prefill/{i}/past"]))
    np.testing.assert_allclose(out, ATTN[f"prefill/{i}/o"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("i", range(_n("verify")))
def test_oracle_verify_matches_hf_sdpa(i):
    q, k, v = (bf16_to_f32(ATTN[f"verify/{i}/{x}"]) for x in "qkv")
    out = verify_attention(q, k, v, q.shape[-1] ** -0.5, prefix_len=int(ATTN[f"verify/{i}/prefix"]))
    np.testing.assert_allclose(out, ATTN[f"verify/{i}/o"], rtol=1e-5, atol=1e-5)


def test_bf16_rounding_matches_torch():
    import torch

    x = torch.randn(4096, generator=torch.Generator().manual_seed(3)) * 100
    x[:4] = torch.tensor([0.0, -0.0, 1e-40, 3.0e38])
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(f32_to_bf16(x.numpy()), ref)
    assert np.array_equal(bf16_to_f32(ref), x.to(torch.bfloat16).float().numpy())
