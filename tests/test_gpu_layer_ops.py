"""GPU parity of the fused decoder-layer ops against the HF modules they replace.

``pkv_rope`` and ``pkv_silu_mul`` round where torch rounds, so they equal HF's
``apply_rotary_pos_emb`` and ``act_fn(gate) * up`` bit for bit (bar: every
element equal, bf16 and f16).  ``pkv_rms_norm`` sums x^2 in another order than
torch's mean, so its variance can differ in the last fp32 bits, which can move
x * rsqrt(var) to the neighbouring value of the dtype and, after the product
with the weight, the output by up to two units in the last place; bar: at most
two, and at least 99 % of elements equal.  The residual sum it folds in equals torch's ``a + b`` bit for bit.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _qwen2_modules(hidden: int, dtype, device):
    from transformers.models.qwen2 import modeling_qwen2 as m

    norm = m.Qwen2RMSNorm(hidden, eps=1e-6).to(device=device, dtype=dtype)
    with torch.no_grad():
        norm.weight.copy_(torch.randn(hidden, generator=torch.Generator().manual_seed(1)).to(dtype) * 0.5 + 1)
    return m, norm


def _ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in units in the last place of a's dtype (same-sign finite values)."""
    ia = a.view(torch.int16).to(torch.int32)
    ib = b.view(torch.int16).to(torch.int32)
    return (ia - ib).abs()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hidden,rows", [(1536, 32), (3584, 7), (896, 513), (100, 9)])  # 100: the general kernel
def test_rms_norm_matches_hf(cuda_device, dtype, hidden, rows):
    from randomrepo_b200.hf import fused_rms_norm

    _, norm = _qwen2_modules(hidden, dtype, cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(hidden + rows)
    x = (torch.randn((rows, hidden), generator=g, device=cuda_device) * 3).to(dtype)
    r = torch.randn((rows, hidden), generator=g, device=cuda_device).to(dtype)
    with torch.no_grad():
        want = norm(x)
        want_sum = r + x
        want2 = norm(want_sum)
    got = fused_rms_norm(x, norm)
    got2, got_sum = fused_rms_norm(x, norm, residual=r)
    torch.cuda.synchronize()
    assert torch.equal(got_sum, want_sum)
    for a, b in ((got, want), (got2, want2)):
        u = _ulps(a, b)
        assert int(u.max()) <= 2
        assert float((u == 0).float().mean()) >= 0.99


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d,b,t", [(12, 2, 128, 32, 1), (28, 4, 128, 1, 300), (14, 2, 64, 3, 17),
                                          (4, 2, 40, 2, 5)])  # d = 40: the general kernel
def test_rope_equals_hf(cuda_device, dtype, hq, hkv, d, b, t):
    from randomrepo_b200.hf import fused_rope
    from transformers import Qwen2Config
    from transformers.models.qwen2 import modeling_qwen2 as m

    g = torch.Generator(device=cuda_device).manual_seed(hq * d + t)
    q = torch.randn((b, t, hq * d), generator=g, device=cuda_device).to(dtype)
    k = torch.randn((b, t, hkv * d), generator=g, device=cuda_device).to(dtype)
    cfg = Qwen2Config(hidden_size=hq * d, num_attention_heads=hq, num_key_value_heads=hkv, head_dim=d,
                      rope_theta=1e6, max_position_embeddings=32768)
    rot = m.Qwen2RotaryEmbedding(cfg).to(cuda_device)
    pos = torch.randint(0, 4000, (b, t), generator=g, device=cuda_device)
    cos, sin = rot(q, pos)
    want_q, want_k = m.apply_rotary_pos_emb(q.view(b, t, hq, d).transpose(1, 2), k.view(b, t, hkv, d).transpose(1, 2),
                                            cos, sin)
    got_q, got_k = fused_rope(q, k, cos, sin, d)
    torch.cuda.synchronize()
    assert torch.equal(got_q.view(b, t, hq, d), want_q.transpose(1, 2))
    assert torch.equal(got_k.view(b, t, hkv, d), want_k.transpose(1, 2))


@pytest.mark.parametrize("hq,hkv,d,b,t", [(12, 2, 128, 32, 1), (28, 4, 128, 1, 70), (14, 2, 64, 2, 9)])
def test_rope_on_a_packed_qkv_row_equals_hf(cuda_device, hq, hkv, d, b, t):
    """One packed projection row q | k | v per token (the concatenated-weight GEMM's output)."""
    from randomrepo_b200.hf import fused_rope_qkv
    from transformers import Qwen2Config
    from transformers.models.qwen2 import modeling_qwen2 as m

    dtype = torch.bfloat16
    g = torch.Generator(device=cuda_device).manual_seed(hq + d + t)
    qkv = torch.randn((b, t, (hq + 2 * hkv) * d), generator=g, device=cuda_device).to(dtype)
    q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    cfg = Qwen2Config(hidden_size=hq * d, num_attention_heads=hq, num_key_value_heads=hkv, head_dim=d,
                      rope_theta=1e6, max_position_embeddings=32768)
    rot = m.Qwen2RotaryEmbedding(cfg).to(cuda_device)
    pos = torch.randint(0, 4000, (b, t), generator=g, device=cuda_device)
    cos, sin = rot(qkv, pos)
    want_q, want_k = m.apply_rotary_pos_emb(q.reshape(b, t, hq, d).transpose(1, 2),
                                            k.reshape(b, t, hkv, d).transpose(1, 2), cos, sin)
    got_q, got_k, got_v = fused_rope_qkv(qkv, cos, sin, hq, hkv, d)
    torch.cuda.synchronize()
    assert torch.equal(got_q.view(b, t, hq, d), want_q.transpose(1, 2))
    assert torch.equal(got_k.view(b, t, hkv, d), want_k.transpose(1, 2))
    assert torch.equal(got_v.view(b, t, hkv * d), v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(32, 8960), (5, 18944), (700, 4864), (1, 3)])
def test_silu_mul_equals_hf(cuda_device, dtype, rows, cols):
    from randomrepo_b200.hf import fused_silu_mul, fused_silu_mul_packed

    g = torch.Generator(device=cuda_device).manual_seed(rows + cols)
    gate = (torch.randn((rows, cols), generator=g, device=cuda_device) * 4).to(dtype)
    up = torch.randn((rows, cols), generator=g, device=cuda_device).to(dtype)
    want = torch.nn.functional.silu(gate) * up
    got = fused_silu_mul(gate, up)
    packed = fused_silu_mul_packed(torch.cat([gate, up], dim=-1))
    torch.cuda.synchronize()
    assert torch.equal(packed, got)
    u = _ulps(got, want)
    assert int(u.max()) <= 1
    assert float((u == 0).float().mean()) >= 0.999


def test_layer_ops_reject_bad_arguments(cuda_device):
    from randomrepo_b200._lib import PKV_ERR_ARG, PKV_ERR_UNSUPPORTED, PKV_F32, PKV_BF16, lib

    x = torch.zeros((2, 16), dtype=torch.bfloat16, device=cuda_device)
    assert lib.pkv_rms_norm(x.data_ptr(), None, None, x.data_ptr(), x.data_ptr(), 2, 9000, 1e-6, PKV_BF16,
                            None) == PKV_ERR_ARG
    assert lib.pkv_rms_norm(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), x.data_ptr(), 2, 16, 1e-6, PKV_BF16,
                            None) == PKV_ERR_ARG
    p = x.data_ptr()
    assert lib.pkv_rope(p, p, None, p, p, p, p, None, 2, 16, 16, 0, 1, 1, 15, PKV_BF16, None) == PKV_ERR_ARG  # odd D
    assert lib.pkv_rope(p, p, None, p, p, p, p, None, 2, 8, 16, 0, 1, 1, 16, PKV_BF16, None) == PKV_ERR_ARG  # q_ld
    assert lib.pkv_rope(p, p, p, p, p, p, p, None, 2, 16, 16, 16, 1, 1, 16, PKV_BF16, None) == PKV_ERR_ARG  # v alone
    assert lib.pkv_silu_mul(x.data_ptr(), x.data_ptr(), x.data_ptr(), 2, 16, 8, PKV_BF16, None) == PKV_ERR_ARG
    assert lib.pkv_silu_mul(x.data_ptr(), x.data_ptr(), x.data_ptr(), 2, 16, 16, PKV_F32, None) == PKV_ERR_UNSUPPORTED
