"""GPU parity of paged GQA decode attention (fused with the step's K/V append).

Floating-point bar (the attention tolerance): |out - oracle| <= 2e-2 + 1e-2 * |oracle|
elementwise, bf16/f16 inputs, fp32 accumulation.  The oracle is the fp32
restatement of HF ``sdpa_attention_forward`` (pinned to the reference's
attention by tests/test_oracle_golden.py); the golden HF outputs themselves are
also checked directly.  The appended K/V rows are compared bit-exactly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import bf16_to_f32, decode_attention
from tests.conftest import load_npz

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
HKV_B = 2  # KV heads of the microbench shape
ATTN = load_npz("attention_sdpa.npz")


def _close(got: torch.Tensor, want: np.ndarray) -> None:
    g = got.float().cpu().numpy()
    np.testing.assert_allclose(g, want, rtol=RTOL, atol=ATOL)


def _from_bits(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)


def _make_store(hkv, d, dtype, device, blocks=4096, layers=1):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore

    return PagedKVCacheStore(PagedKVAllocator(blocks, 16), num_layers=layers, num_kv_heads=hkv, head_dim=d,
                             dtype=dtype, device=device)


def _prefill(store, sid, k, v):
    """Reserve ``k.shape[0]`` tokens and write them (k/v [T, Hkv, D])."""
    t = k.shape[0]
    store.reserve(sid, t)
    if t:
        kk = k.permute(1, 0, 2).unsqueeze(0).contiguous()
        vv = v.permute(1, 0, 2).unsqueeze(0).contiguous()
        store.write_sequence_cache(sid, ((kk, vv),), None)


n_decode = len({k.split("/")[1] for k in ATTN if k.startswith("decode/")})


@pytest.mark.parametrize("i", range(n_decode))
def test_decode_matches_hf_sdpa_fixture(cuda_device, i):
    q = _from_bits(ATTN[f"decode/{i}/q"], cuda_device)  # [Hq, D]
    k = _from_bits(ATTN[f"decode/{i}/k"], cuda_device)  # [T, Hkv, D]
    v = _from_bits(ATTN[f"decode/{i}/v"], cuda_device)
    t = k.shape[0]
    store = _make_store(k.shape[1], k.shape[2], torch.bfloat16, cuda_device)
    _prefill(store, 0, k[: t - 1], v[: t - 1])
    step = store.decode_step([0])
    out = store.decode_attention(step, 0, q[None].contiguous(), k[t - 1 :].contiguous(), v[t - 1 :].contiguous())
    torch.cuda.synchronize()
    _close(out[0], ATTN[f"decode/{i}/o"])
    got = store.read_sequence_legacy_cache(0)
    assert torch.equal(got[0][0][0].permute(1, 0, 2), k) and torch.equal(got[0][1][0].permute(1, 0, 2), v)
    assert store.pool.decode_error_flag() == 0


def _batch_case(device, lengths, hq, hkv, d, dtype, seed, layers=1):
    gen = torch.Generator().manual_seed(seed)
    store = _make_store(hkv, d, dtype, device, blocks=sum((n + 16) // 16 + 1 for n in lengths) + 64, layers=layers)
    ks, vs = [], []
    for sid, n in enumerate(lengths):
        k = torch.randn((n, hkv, d), generator=gen).to(dtype)
        v = torch.randn((n, hkv, d), generator=gen).to(dtype)
        ks.append(k)
        vs.append(v)
        _prefill(store, sid, k[: n - 1].to(device), v[: n - 1].to(device))
    q = torch.randn((len(lengths), hq, d), generator=gen).to(dtype)
    kn = torch.stack([k[-1] for k in ks])
    vn = torch.stack([v[-1] for v in vs])
    return store, q, kn, vn, ks, vs


def _oracle(q, ks, vs, scale):
    out = []
    for b in range(q.shape[0]):
        out.append(decode_attention(q[b].float().numpy(), ks[b].float().numpy(), vs[b].float().numpy(), scale))
    return np.stack(out)


EDGE_LENGTHS = [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 255, 256, 257, 1000, 2048, 2049]


@pytest.mark.parametrize("hq,hkv", [(12, 2), (4, 2), (14, 2), (28, 4), (8, 1), (2, 2)])
@pytest.mark.parametrize("d", [128, 64])
def test_decode_gqa_shapes_match_oracle(cuda_device, hq, hkv, d):
    store, q, kn, vn, ks, vs = _batch_case(cuda_device, EDGE_LENGTHS, hq, hkv, d, torch.bfloat16, seed=hq * 100 + d)
    step = store.decode_step(list(range(len(EDGE_LENGTHS))))
    out = store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    torch.cuda.synchronize()
    _close(out, _oracle(q, ks, vs, d ** -0.5))
    assert store.pool.decode_error_flag() == 0


def test_decode_fp16(cuda_device):
    lengths = [5, 100, 700]
    store, q, kn, vn, ks, vs = _batch_case(cuda_device, lengths, 12, 2, 128, torch.float16, seed=9)
    step = store.decode_step([0, 1, 2])
    out = store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    _close(out, _oracle(q, ks, vs, 128 ** -0.5))


def test_decode_microbench_shape_and_append_bits(cuda_device):
    """256 sequences, ctx U[64, 2048], 12/2 heads, D=128 (the microbench shape)."""
    gen = torch.Generator().manual_seed(0)
    lengths = torch.randint(64, 2049, (256,), generator=gen).tolist()
    store, q, kn, vn, ks, vs = _batch_case(cuda_device, lengths, 12, 2, 128, torch.bfloat16, seed=1)
    step = store.decode_step(list(range(256)))
    assert step.n_items > 256  # split-K is exercised
    out = store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    torch.cuda.synchronize()
    _close(out, _oracle(q, ks, vs, 128 ** -0.5))
    for sid in range(256):
        got = store.read_sequence_legacy_cache(sid)
        assert torch.equal(got[0][0][0].permute(1, 0, 2).cpu(), ks[sid])
        assert torch.equal(got[0][1][0].permute(1, 0, 2).cpu(), vs[sid])
    _check_device_tables(store, range(256), lengths)


def _check_device_tables(store, sids, lengths) -> None:
    """Device block tables and lengths (written by the fused kernel) equal the host allocator, every row."""
    tables = store.pool.tables.cpu().numpy()
    lens = store.pool.context_lens.cpu().numpy()
    for sid in sids:
        view = store.allocator.view(sid)
        row = store.allocator.row(sid)
        assert lens[row] == view.token_count == lengths[sid]
        assert tuple(tables[row, : view.logical_block_count]) == view.physical_blocks


def test_decode_on_the_bench_workload(cuda_device):
    """The microbench's own workload (bench.build_workload): 256 sequences of U[64, 2048] tokens whose
    blocks follow a random permutation of a 40 000-block pool, pool values N(0, 1).  One fused step through
    PagedKVCacheStore.decode (the call the bench times): all 256 outputs against the oracle, every
    sequence's gathered K/V bit-exact (old rows unchanged, the appended row equal to k_new / v_new), every
    device table row and length equal to the allocator.  Then the same step again with host q / k / v and a
    host output (the end-to-end path): outputs bit-identical to the device-buffer step."""
    import bench

    store, lengths, q, kn, vn, _ = bench.build_workload(cuda_device, 0)
    n = len(lengths)
    ids = np.arange(n, dtype=np.int64)
    # The bench fills the pool with N(0, 1) directly; here each sequence's blocks (the bench's random
    # placement) get seeded K/V through the store, so that the oracle knows them.
    gen = torch.Generator().manual_seed(23)
    before = []
    for b in range(n):
        k = torch.randn((1, HKV_B, int(lengths[b]), 128), generator=gen).to(torch.bfloat16)
        v = torch.randn((1, HKV_B, int(lengths[b]), 128), generator=gen).to(torch.bfloat16)
        store.write_sequence_cache(b, ((k.to(cuda_device), v.to(cuda_device)),), None)
        before.append((k, v))
    out, step = store.decode(ids, q, kn, vn, layer=0)
    torch.cuda.synchronize()
    assert step.n_items > n  # split-K is exercised
    ks = [torch.cat([before[b][0][0].permute(1, 0, 2), kn[b:b + 1].cpu()]) for b in range(n)]
    vs = [torch.cat([before[b][1][0].permute(1, 0, 2), vn[b:b + 1].cpu()]) for b in range(n)]
    _close(out, _oracle(q.cpu(), ks, vs, 128 ** -0.5))
    for b in range(n):
        got = store.read_sequence_legacy_cache(int(b))[0]
        assert torch.equal(got[0][0].permute(1, 0, 2).cpu(), ks[b])
        assert torch.equal(got[1][0].permute(1, 0, 2).cpu(), vs[b])
    _check_device_tables(store, range(n), lengths + 1)
    assert store.pool.decode_error_flag() == 0
    # The end-to-end form of the same step (the bench rolls each sequence back the same way).
    from randomrepo_b200 import host_input_tensor

    store.allocator.truncate(ids, lengths)
    inp = host_input_tensor((q.numel() + 2 * kn.numel(),), q.dtype)
    nq, nk = q.numel(), kn.numel()
    inp[:nq].copy_(q.reshape(-1).cpu())
    inp[nq:nq + nk].copy_(kn.reshape(-1).cpu())
    inp[nq + nk:].copy_(vn.reshape(-1).cpu())
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    store.decode(ids, inp[:nq].view(q.shape), inp[nq:nq + nk].view(kn.shape), inp[nq + nk:].view(vn.shape),
                 layer=0, out=out_h)
    store.wait_host_outputs()
    assert torch.equal(out_h, out.cpu())
    _check_device_tables(store, range(n), lengths + 1)
    assert store.pool.decode_error_flag() == 0


def test_multistep_decode_across_layers(cuda_device):
    """Several steps and layers; every step appends and attends through the same descriptor."""
    gen = torch.Generator().manual_seed(3)
    layers, hq, hkv, d = 3, 12, 2, 128
    lengths = [1, 14, 15, 16, 47, 300]
    store = _make_store(hkv, d, torch.bfloat16, cuda_device, blocks=512, layers=layers)
    caches = []
    for sid, n in enumerate(lengths):
        kv = [(torch.randn((n, hkv, d), generator=gen).to(torch.bfloat16),
               torch.randn((n, hkv, d), generator=gen).to(torch.bfloat16)) for _ in range(layers)]
        store.reserve(sid, n)
        store.write_sequence_cache(sid, tuple((k.permute(1, 0, 2)[None].contiguous().to(cuda_device),
                                               v.permute(1, 0, 2)[None].contiguous().to(cuda_device)) for k, v in kv),
                                   None)
        caches.append(kv)
    for _ in range(20):
        step = store.decode_step(list(range(len(lengths))))
        for layer in range(layers):
            q = torch.randn((len(lengths), hq, d), generator=gen).to(torch.bfloat16)
            kn = torch.randn((len(lengths), hkv, d), generator=gen).to(torch.bfloat16)
            vn = torch.randn((len(lengths), hkv, d), generator=gen).to(torch.bfloat16)
            for b in range(len(lengths)):
                k, v = caches[b][layer]
                caches[b][layer] = (torch.cat([k, kn[b : b + 1]]), torch.cat([v, vn[b : b + 1]]))
            out = store.decode_attention(step, layer, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
            want = _oracle(q, [c[layer][0] for c in caches], [c[layer][1] for c in caches], d ** -0.5)
            _close(out, want)
    for b in range(len(lengths)):
        got = store.read_sequence_legacy_cache(b)
        for layer in range(layers):
            assert torch.equal(got[layer][0][0].permute(1, 0, 2).cpu(), caches[b][layer][0])
            assert torch.equal(got[layer][1][0].permute(1, 0, 2).cpu(), caches[b][layer][1])


def test_unfused_append_then_attention_equals_fused(cuda_device):
    lengths = [3, 16, 129]
    outs = []
    for fused in (True, False):
        store, q, kn, vn, ks, vs = _batch_case(cuda_device, lengths, 12, 2, 128, torch.bfloat16, seed=21)
        step = store.decode_step([0, 1, 2])
        if fused:
            out = store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
        else:
            store.append_step_kv(step, 0, kn.to(cuda_device), vn.to(cuda_device))
            out = store.decode_attention(step, 0, q.to(cuda_device))
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1])


def test_long_context_many_splits(cuda_device):
    lengths = [5000, 17]
    store, q, kn, vn, ks, vs = _batch_case(cuda_device, lengths, 12, 2, 128, torch.bfloat16, seed=4)
    step = store.decode_step([0, 1])
    out = store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    _close(out, _oracle(q, ks, vs, 128 ** -0.5))


def test_decode_rejects_bad_inputs(cuda_device):
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore
    from randomrepo_b200._lib import PKVError

    store, q, kn, vn, ks, vs = _batch_case(cuda_device, [4, 5], 12, 2, 128, torch.bfloat16, seed=2)
    step = store.decode_step([0, 1])
    with pytest.raises(ValueError):
        store.decode_attention(step, 0, q.float().to(cuda_device))
    with pytest.raises(ValueError):
        store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), None)
    odd = PagedKVCacheStore(PagedKVAllocator(64, 8), num_layers=1, num_kv_heads=2, head_dim=128,
                            dtype=torch.bfloat16, device=cuda_device)
    odd.reserve(0, 3)
    st = odd.decode_step([0])
    with pytest.raises(PKVError, match="block_size 16"):
        odd.decode_attention(st, 0, q[:1].to(cuda_device))
    with pytest.raises(KeyError):
        store.decode_step([0, 42])


@pytest.mark.parametrize("n_seqs", [6, 256])
def test_host_buffer_decode_equals_device_decode(cuda_device, n_seqs):
    """``decode`` with pinned host q / k / v / out (the stepper stages them) equals the device-tensor call.

    Steps alternate between one packed host buffer (a single input copy; from
    ``host_input_tensor``, write-combined or not) and three separate tensors
    (three copies); every step keeps its own inputs and
    output until ``wait_host_outputs``.  Twenty steps go one and a quarter times
    round the stepper's sixteen staging entries (guarded in rounds of eight),
    so entries are reused while earlier output copies may still be in flight.
    """
    STEPS = 20
    from randomrepo_b200 import host_input_tensor

    gen = torch.Generator().manual_seed(11)
    lengths = torch.randint(64, 2049, (n_seqs,), generator=gen).tolist() if n_seqs > 6 else [1, 15, 16, 17, 300, 2049]
    hq, hkv, d = 12, 2, 128
    dev_store, _, _, _, ks, vs = _batch_case(cuda_device, lengths, hq, hkv, d, torch.bfloat16, seed=5)
    host_store, _, _, _, _, _ = _batch_case(cuda_device, lengths, hq, hkv, d, torch.bfloat16, seed=5)
    ks, vs = [k[:-1] for k in ks], [v[:-1] for v in vs]  # the cases' own step tokens are not used here
    ids = np.arange(n_seqs, dtype=np.int64)
    nq, nk = n_seqs * hq * d, n_seqs * hkv * d
    want, got, keep = [], [], []
    for s in range(STEPS):
        q = torch.randn((n_seqs, hq, d), generator=gen).to(torch.bfloat16)
        kn = torch.randn((n_seqs, hkv, d), generator=gen).to(torch.bfloat16)
        vn = torch.randn((n_seqs, hkv, d), generator=gen).to(torch.bfloat16)
        for b in range(n_seqs):
            ks[b] = torch.cat([ks[b], kn[b : b + 1]])
            vs[b] = torch.cat([vs[b], vn[b : b + 1]])
        out_d, _ = dev_store.decode(ids, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
        want.append(out_d)
        if s % 2 == 0:
            packed = host_input_tensor((nq + 2 * nk,), torch.bfloat16, write_combined=s % 4 == 0)
            packed[:nq].copy_(q.reshape(-1))
            packed[nq : nq + nk].copy_(kn.reshape(-1))
            packed[nq + nk :].copy_(vn.reshape(-1))
            hq_t, hk_t, hv_t = (packed[:nq].view(q.shape), packed[nq : nq + nk].view(kn.shape),
                                packed[nq + nk :].view(vn.shape))
        else:
            hq_t, hk_t, hv_t = q.pin_memory(), kn.pin_memory(), vn.pin_memory()
        out_h = torch.full(q.shape, float("nan"), dtype=torch.bfloat16).pin_memory()
        res, step = host_store.decode(ids, hq_t, hk_t, hv_t, out=out_h)
        assert res is out_h and step.batch == n_seqs
        got.append(out_h)
        keep.append((hq_t, hk_t, hv_t))
    host_store.wait_host_outputs()
    torch.cuda.synchronize()
    for s in range(STEPS):
        assert torch.equal(got[s], want[s].cpu()), f"step {s}"
    _close(got[-1], _oracle(q, ks, vs, d ** -0.5))
    for sid in (0, n_seqs // 2, n_seqs - 1):
        a = host_store.read_sequence_legacy_cache(sid)
        assert torch.equal(a[0][0][0].permute(1, 0, 2).cpu(), ks[sid])
        assert torch.equal(a[0][1][0].permute(1, 0, 2).cpu(), vs[sid])
    assert host_store.pool.decode_error_flag() == 0


def test_host_buffer_decode_rejects_bad_inputs(cuda_device):
    store, q, kn, vn, _, _ = _batch_case(cuda_device, [4, 5], 12, 2, 128, torch.bfloat16, seed=2)
    ids = np.arange(2, dtype=np.int64)
    with pytest.raises(ValueError):
        store.decode(ids, q, kn, None)
    with pytest.raises(ValueError):
        store.decode(ids, q, kn.to(cuda_device), vn)  # mixed host / device
    with pytest.raises(ValueError):
        store.decode(ids, q.float(), kn, vn)
    with pytest.raises(ValueError):
        store.decode(ids, q, kn, vn, out=torch.empty((2, 12, 64), dtype=torch.bfloat16))
    out, _ = store.decode(ids, q, kn, vn)  # a pinned output is made
    store.wait_host_outputs()
    assert out.device.type == "cpu" and out.is_pinned() and torch.isfinite(out.float()).all()


def test_fixed_step_mode_grows_its_work_item_capacity(cuda_device):
    """Fixed-step mode (the descriptor block CUDA graphs replay) with too small a work-item capacity:
    the step reports the items it needs, the store fixes the steps again and the results are unchanged."""
    lengths = [3000, 2049, 700, 64, 17, 1]
    store, q, kn, vn, ks, vs = _batch_case(cuda_device, lengths, 12, 2, 128, torch.bfloat16, seed=8)
    pool = store.pool
    pool.fix_steps(len(lengths), max_items=len(lengths))  # one item per sequence: far too few
    serial, cap = pool.fixed_serial, pool.fixed_items
    assert cap == len(lengths)
    step = store.decode_step(list(range(len(lengths))))
    assert step.n_items > cap and pool.fixed_items >= step.n_items and pool.fixed_serial == serial + 1
    out = store.decode_attention(step, 0, q.to(cuda_device), kn.to(cuda_device), vn.to(cuda_device))
    torch.cuda.synchronize()
    _close(out, _oracle(q, ks, vs, 128 ** -0.5))
    assert pool.decode_error_flag() == 0


def test_host_buffer_decode_separate_allocations(cuda_device):
    """Three separately allocated host inputs -- which the host allocator may place back to back --
    are copied one by one (a single copy across two allocations is an invalid range)."""
    from randomrepo_b200 import host_input_tensor

    for trial in range(4):
        store, q, kn, vn, ks, vs = _batch_case(cuda_device, [37, 5], 12, 2, 128, torch.bfloat16, seed=30 + trial)
        ids = np.arange(2, dtype=np.int64)
        qh = host_input_tensor(q.shape, torch.bfloat16)
        kh = host_input_tensor(kn.shape, torch.bfloat16)
        vh = host_input_tensor(vn.shape, torch.bfloat16)
        qh.copy_(q), kh.copy_(kn), vh.copy_(vn)
        out, _ = store.decode(ids, qh, kh, vh)
        store.wait_host_outputs()
        _close(out, _oracle(q, ks, vs, 128 ** -0.5))
        assert store.pool.decode_error_flag() == 0
