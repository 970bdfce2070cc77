"""The torch restatements of the reference's two CPU decode paths (the timed CPU baseline) agree with the
fp32 attention oracle and with each other, and their rollback restores the allocator's lengths."""

from __future__ import annotations

import numpy as np
import torch

from oracle.attention import decode_attention
from oracle.decode_step import TorchBlockStoreDecodeBatch, TorchResidentDecodeBatch


def test_resident_and_block_store_paths_match_the_oracle():
    lens = [5, 16, 17, 40, 40, 100]
    a = TorchResidentDecodeBatch(lens, 12, 2, 128, seed=1, dtype=torch.float32)
    b = TorchBlockStoreDecodeBatch(lens, 12, 2, 128, seed=1, dtype=torch.float32)
    k0 = [k.clone() for k in a.keys]
    v0 = [v.clone() for v in a.values]
    g = torch.Generator().manual_seed(2)
    ids = list(range(len(lens)))
    for step in range(3):
        q = torch.randn(len(lens), 12, 128, generator=g)
        kn = torch.randn(len(lens), 2, 128, generator=g)
        vn = torch.randn(len(lens), 2, 128, generator=g)
        oa = a.step(ids, q, kn, vn)
        ob = b.step(ids, q, kn, vn)
        assert torch.equal(oa, ob)
        for i in ids:
            k0[i] = torch.cat([k0[i], kn[i:i + 1].unsqueeze(2)], dim=2)
            v0[i] = torch.cat([v0[i], vn[i:i + 1].unsqueeze(2)], dim=2)
            want = decode_attention(q[i].numpy(), k0[i][0].transpose(0, 1).numpy(), v0[i][0].transpose(0, 1).numpy(),
                                    128 ** -0.5)
            np.testing.assert_allclose(oa[i].numpy(), want, atol=1e-5, rtol=1e-5)
    assert [a.allocator.view(i).token_count for i in ids] == [n + 3 for n in lens]
    a.rollback(ids)
    b.rollback(ids)
    assert [a.allocator.view(i).token_count for i in ids] == [n + 2 for n in lens]
    assert [b.allocator.view(i).token_count for i in ids] == [n + 2 for n in lens]
    assert [int(k.shape[2]) for k in a.keys] == [n + 2 for n in lens]
