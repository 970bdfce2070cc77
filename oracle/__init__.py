"""CPU oracle for the paged-KV path: test infrastructure, never the product.

This package restates, in plain Python and numpy, what AgentRL's paged-KV path
computes, so that the CUDA kernels and the host allocator of ``randomrepo_b200``
can be checked against it on identical seeded inputs:

* ``oracle.allocator`` -- ``PagedKVAllocator`` (agentrl/generation/paged_kv.py:25-175),
  plus the copy-on-write fork/refcount extension that the reference lacks.
* ``oracle.store`` -- ``PagedKVCacheStore`` block storage, write and gather
  (agentrl/generation/paged_kv.py:178-360).
* ``oracle.attention`` -- fp32 GQA attention as HF ``sdpa_attention_forward``
  computes it (transformers 5.5.0, integrations/sdpa_attention.py:40-62) for
  decode, chunked prefill with a past offset, and the k+1-query verify read.
* ``oracle.decode_step`` -- the reference's resident-cache decode step
  (agentrl/generation/continuous.py:407-497,1090-1121) used as the timed CPU
  baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline
leg and its ``--impl reference`` arm) may import this package, and only as the
checker or the timed CPU baseline.  The product path in ``randomrepo_b200``
never imports it.

Pinning: the allocator and store restatements are pinned against fixtures
produced by running the reference itself (``tests/golden/make_golden.py``) and
against the reference's own known-answer tests (tests/test_paged_kv.py).  The
attention restatement is pinned against HF ``sdpa_attention_forward`` outputs
committed as fixtures by the same script.  The fork/refcount extension has no
reference counterpart: its parity is unpinned by the reference and is checked
semantically (every fork member gathers exactly what an independent prefill
would have stored).  The speculative loop (``speculative.py``) is pinned
against a recorded run of the reference's own orchestrator, acceptance draws
included (``speculative_c1_trace.json``, made by the same script).
"""
