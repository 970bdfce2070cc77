"""B200-native paged-KV path of AgentRL's continuous-batching rollout.

Public API (drop-in for ``agentrl.generation.paged_kv``):

* ``PagedKVSequenceView``, ``PagedKVAllocator``, ``PagedKVCacheStore``;
* the device paths of the store: ``decode_step`` / ``decode_attention``
  (fused append + paged GQA decode), ``prefill_attention`` /
  ``verify_attention`` (chunked prefill and speculative verify on tcgen05),
  copy-on-write ``fork`` and ``truncate``;
* ``PagedGenerator`` (``randomrepo_b200.hf``): HF Qwen2-family models
  prefilling and decoding through the store (CUDA-graph decode steps, fused
  norm / rotary / SiLU launches);
* ``host_input_tensor``: page-locked, write-combined host memory for the
  q / k / v a host hands to ``PagedKVCacheStore.decode`` (the host-buffer
  decode path);
* ``assign_groups`` / ``StepGather`` (``randomrepo_b200.sharding``): GRPO
  groups per GPU and the per-step gather of sampled tokens and logprobs;
* ``randomrepo_b200.ops``: the kernels as PyTorch operators
  (``torch.ops.pkv.kv_append`` / ``kv_gather`` / ``copy_blocks`` /
  ``decode_attention`` / ``prefill_attention``, with fake-tensor shapes),
  registered when that module is imported.

All device work runs in ``libpkv_b200.so`` (hand-written sm_100a kernels),
built in-tree by ``python -m randomrepo_b200.build``.  The library is loaded
on first use of these names (so the build module itself imports without it);
if it is missing that first use raises ImportError -- there is no fallback.
"""

from __future__ import annotations

_EXPORTS = {
    "DecodeStep": "paged_kv",
    "PagedKVAllocator": "paged_kv",
    "PagedKVCacheStore": "paged_kv",
    "PagedKVSequenceView": "paged_kv",
    "host_input_tensor": "paged_kv",
    "PagedGenerator": "hf",
    "SamplingConfig": "hf",
    "StepGather": "sharding",
    "assign_groups": "sharding",
}

__all__ = sorted(_EXPORTS)


def __getattr__(name: str):
    module = _EXPORTS.get(name)
    if module is None:
        raise AttributeError(f"module 'randomrepo_b200' has no attribute {name!r}")
    import importlib

    value = getattr(importlib.import_module(f".{module}", __name__), name)
    globals()[name] = value
    return value
