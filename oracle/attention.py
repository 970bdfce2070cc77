"""Oracle restatement of the reference's attention arithmetic (test infrastructure).

The reference's attention is HF ``sdpa_attention_forward`` (transformers 5.5.0,
integrations/sdpa_attention.py:40-62) called from ``Qwen2Attention.forward``
(models/qwen2/modeling_qwen2.py:206-245): softmax(q k^T * scale) v in fp32 with
grouped-query attention (query head h reads KV head h // (Hq / Hkv), the
``repeat_kv`` mapping at sdpa_attention.py:16-25) and a causal mask for a chunk
that follows ``past`` cached tokens (query i sees keys 0 .. past + i).

All inputs are converted to float32 before the arithmetic; bf16 inputs arrive
as their uint16 bit patterns and are widened exactly with ``bf16_to_f32``.
"""

from __future__ import annotations

import numpy as np


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even narrowing of float32 to bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))
    out = (rounded >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def gqa_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, past: int | None = None) -> np.ndarray:
    """One sequence: q [Tq, Hq, D], k/v [Tk, Hkv, D] -> out [Tq, Hq, D] (float32).

    ``past=None`` lets every query see every key (the decode call, where HF
    passes no causal mask for a single query, sdpa_attention.py:77).  Otherwise
    query i sees keys ``0 .. past + i`` (HF's causal mask for a chunk after a
    cache of ``past`` tokens).
    """
    q = q.astype(np.float32)
    k = k.astype(np.float32)
    v = v.astype(np.float32)
    tq, hq, _ = q.shape
    tk, hkv, _ = k.shape
    group = hq // hkv
    out = np.empty(q.shape, dtype=np.float32)
    if past is not None:
        qpos = past + np.arange(tq)[:, None]
        visible = np.arange(tk)[None, :] <= qpos
    for h in range(hq):
        kh = k[:, h // group, :]
        vh = v[:, h // group, :]
        s = (q[:, h, :] @ kh.T) * np.float32(scale)
        if past is not None:
            s = np.where(visible, s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h, :] = p @ vh
    return out


def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """Single-query decode: q [Hq, D], k/v [T, Hkv, D] -> [Hq, D]."""
    return gqa_attention(q[None], k, v, scale, past=None)[0]


def prefill_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, past: int) -> np.ndarray:
    """Chunk of Tq queries after ``past`` cached tokens; k/v hold past + Tq tokens."""
    if k.shape[0] != past + q.shape[0]:
        raise ValueError("keys must cover the past tokens plus the chunk")
    return gqa_attention(q, k, v, scale, past=past)


def verify_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, prefix_len: int) -> np.ndarray:
    """The k+1-query speculative-verify read (agentrl/generation/speculative.py:229-264).

    The reference runs a full causal forward over ``prefix + k draft`` tokens
    and reads rows ``prefix_len - 1 .. prefix_len - 1 + k``.  Those rows are the
    queries at those positions under the causal mask, i.e. a chunk of k+1
    queries after ``prefix_len - 1`` cached tokens over ``prefix_len + k`` keys.
    """
    return prefill_attention(q, k, v, scale, past=prefix_len - 1)
