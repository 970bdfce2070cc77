"""The PyTorch operator layer over the C ABI (``randomrepo_b200.ops``): registered under ``torch.ops.pkv``
and traceable with fake tensors (output shapes without running a kernel, as torch.compile traces them)."""

from __future__ import annotations

import pytest
import torch

import randomrepo_b200.ops  # noqa: F401 - registers the operators


def test_operators_are_registered():
    for name in ("kv_append", "kv_gather", "copy_blocks", "decode_attention", "prefill_attention",
                 "verify_attention"):
        assert hasattr(torch.ops.pkv, name)


def test_fake_tensor_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    geom = [1, 64, 2, 16, 128, 2]  # bf16
    with FakeTensorMode(allow_non_fake_inputs=False) as mode:
        dev = torch.device("cuda", 0)
        pool = torch.empty(1 << 20, dtype=torch.uint8, device=dev)
        q = torch.empty((5, 12, 128), dtype=torch.bfloat16, device=dev)
        kn = torch.empty((5, 2, 128), dtype=torch.bfloat16, device=dev)
        i32 = lambda *s: torch.empty(s, dtype=torch.int32, device=dev)  # noqa: E731
        out = torch.ops.pkv.decode_attention(pool, geom, 0, q, kn, kn, i32(8, 4), i32(8), i32(5), i32(5), i32(5),
                                             i32(9, 4), 7, 2, 4, 0.088, pool)
        assert out.shape == q.shape and out.dtype == q.dtype
        k, v = torch.ops.pkv.kv_gather(pool, geom, 0, torch.empty(33, dtype=torch.int64, device=dev))
        assert k.shape == (33, 2, 128) and v.shape == (33, 2, 128) and k.dtype == torch.bfloat16
        o = torch.ops.pkv.prefill_attention(pool, geom, 0, torch.empty((40, 12, 128), dtype=torch.bfloat16,
                                                                        device=dev),
                                            i32(8, 4), i32(3, 8), 3, 0, 0, 0.088, i32(1), pool)
        assert o.shape == (40, 12, 128)
        o = torch.ops.pkv.verify_attention(pool, geom, 0, torch.empty((15, 12, 128), dtype=torch.bfloat16,
                                                                       device=dev),
                                           i32(8, 4), i32(6, 8), 6, 6, 0, 0, 0.088, i32(1), pool)
        assert o.shape == (15, 12, 128) and o.dtype == torch.bfloat16
    assert mode is not None


def test_geometry_is_checked():
    from randomrepo_b200.ops import _geom

    with pytest.raises(RuntimeError):
        _geom([1, 2, 3])
