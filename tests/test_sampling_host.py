"""Host side of the vocabulary-row kernels on CPU: workspace sizing, argument checks, no CPU path.

Every call below is rejected (or sized) before anything is launched, so no GPU
is needed; the kernels themselves run in tests/test_gpu_sampling.py.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from randomrepo_b200 import _lib
from randomrepo_b200._lib import lib

VOCAB = 151936


def test_workspace_sizes_and_tickets():
    spans = -(-VOCAB // 4096)  # most CTAs a row is ever cut into
    assert lib.pkv_sampling_workspace_bytes(4096, VOCAB) == -(-4096 * spans * 32 // 256) * 256
    assert lib.pkv_sampling_workspace_bytes(0, VOCAB) == 0
    assert lib.pkv_sampling_workspace_bytes(-1, VOCAB) == -1
    assert lib.pkv_sampling_workspace_bytes(4, 0) == -1
    assert lib.pkv_spec_tickets(64, 4) == 64 * 10
    assert lib.pkv_spec_tickets(64, 0) == -1 and lib.pkv_spec_tickets(64, 17) == -1
    small = lib.pkv_spec_workspace_bytes(8, 4, VOCAB)
    assert 0 < small < lib.pkv_spec_workspace_bytes(64, 4, VOCAB)
    assert lib.pkv_spec_workspace_bytes(8, 0, VOCAB) == -1


def _status(name: str, *args) -> int:
    return getattr(lib, name)(*args)


def test_token_logprobs_rejects_bad_arguments():
    ws = ctypes.create_string_buffer(1 << 16)
    tk = (ctypes.c_int32 * 64)()
    dummy = ctypes.c_void_p(0x1000)
    # null logits, ld < vocab, a log-prob output without tokens, no output at all, no tickets / workspace
    assert _status("pkv_token_logprobs", None, 512, 4, 512, dummy, dummy, None, tk, ws, len(ws), None) == _lib.PKV_ERR_ARG
    assert _status("pkv_token_logprobs", dummy, 256, 4, 512, dummy, dummy, None, tk, ws, len(ws), None) == _lib.PKV_ERR_ARG
    assert _status("pkv_token_logprobs", dummy, 512, 4, 512, None, dummy, None, tk, ws, len(ws), None) == _lib.PKV_ERR_ARG
    assert _status("pkv_token_logprobs", dummy, 512, 4, 512, None, None, None, tk, ws, len(ws), None) == _lib.PKV_ERR_ARG
    assert _status("pkv_token_logprobs", dummy, 512, 4, 512, dummy, dummy, None, None, ws, len(ws), None) == _lib.PKV_ERR_ARG
    assert _status("pkv_token_logprobs", dummy, 512, 4, 512, dummy, dummy, None, tk, ws, 0, None) == _lib.PKV_ERR_ARG
    assert "workspace" in _lib.last_error()


def test_sample_and_accept_reject_bad_arguments():
    ws = ctypes.create_string_buffer(1 << 20)
    tk = (ctypes.c_int32 * 4096)()
    dummy = ctypes.c_void_p(0x1000)
    # sampling needs a temperature > 0; tokens_out is required
    assert _status("pkv_sample_tokens", dummy, None, 512, 4, 512, 0.0, 1, 0, 0, dummy, None, None, tk, ws,
                   len(ws), None) == _lib.PKV_ERR_ARG
    assert _status("pkv_sample_tokens", dummy, None, 512, 4, 512, 1.0, 0, 0, 0, None, None, None, tk, ws,
                   len(ws), None) == _lib.PKV_ERR_ARG
    args = dict(ld=512, batch=4, vocab=512, temp=1.0)
    for k in (0, 17):
        assert _status("pkv_spec_accept", dummy, dummy, args["ld"], dummy, dummy, None, args["batch"], k,
                       args["vocab"], args["temp"], 0, -1, 0, 0, dummy, dummy, dummy, dummy, tk, ws, len(ws),
                       None) == _lib.PKV_ERR_ARG
    # draft temperature must be > 0
    assert _status("pkv_spec_accept", dummy, dummy, 512, dummy, dummy, None, 4, 4, 512, 0.0, 0, -1, 0, 0, dummy,
                   dummy, dummy, dummy, tk, ws, len(ws), None) == _lib.PKV_ERR_ARG
    # missing outputs
    assert _status("pkv_spec_accept", dummy, dummy, 512, dummy, dummy, None, 4, 4, 512, 1.0, 0, -1, 0, 0, None,
                   dummy, dummy, dummy, tk, ws, len(ws), None) == _lib.PKV_ERR_ARG


def test_device_sampler_has_no_cpu_path():
    from randomrepo_b200.sampling import DeviceSampler, SamplingConfig, _rows

    with pytest.raises(ValueError):
        DeviceSampler("cpu")
    with pytest.raises(ValueError):
        _rows(torch.zeros(2, 8), "test")
    assert SamplingConfig(do_sample=True, temperature=0.7).sampling
    assert not SamplingConfig(do_sample=True, temperature=0.0).sampling
    assert not SamplingConfig().sampling


def test_top_p_filter_matches_the_reference_rule():
    from oracle.sampling import apply_top_p
    from randomrepo_b200.sampling import top_p_filter

    g = torch.Generator().manual_seed(1)
    logits = torch.randn(6, 50, generator=g) * 2
    for p in (0.1, 0.5, 0.9, 0.999, 1.0):
        a = top_p_filter(logits, p)
        b = apply_top_p(logits, p)
        assert torch.equal(torch.isinf(a), torch.isinf(b))
        assert torch.equal(a[~torch.isinf(a)], b[~torch.isinf(b)])
