"""Paged-decode microbench of the B200 paged-KV path (one JSON line on stdout).

Workload (the paged-KV kernel microbench at the Qwen2.5-1.5B attention shape):
one decode step = append one token per sequence + paged GQA attention, one
layer, bf16, 12 query / 2 KV heads, head_dim 128, block size 16, 256
sequences per GPU with context lengths U[64, 2048] (seeded), a 40 000-block
pool with every sequence's blocks drawn from a random permutation of it, and
K/V/Q ~ N(0, 1).  After each step the allocator rolls every sequence back by
the token it appended, so every timed step sees the configured length
distribution whatever --steps is.

Arms:
  ours (default)     ``value``: device-timed steps through PagedKVCacheStore
                     (host allocator step + one descriptor upload + the fused
                     sm_100a decode kernel) with inputs resident in HBM;
                     ``e2e``: the same steps given host q/k/v (page-locked,
                     write-combined) and a page-locked host output, every
                     step's copies inside the timed region (the stepper's host
                     path overlaps them with the neighbouring steps' kernels);
                     median of three timed regions.
  --impl reference   the reference's CPU path (the oracle's restatement of the
                     resident-cache decode step) on the host cores, rank 0 only.

At N=1 the line also carries ``tensor_tiles``: the tcgen05 chunked-prefill
attention kernel (Qwen2.5-7B attention shape, 32 prompts of U[256,4096] tokens,
every 512-token chunk in one launch) against the measured bf16 tensor peak, and
the speculative-verify read (1.5B target shape, 64 sequences, k = 4) against
the measured HBM bandwidth, each timed alone with CUDA events and L2 flushed.

It also carries ``vocab_rows``: the fused log-softmax + gather, sampling and
speculative accept kernels over Qwen2's 151 936-column logits rows against
the measured HBM bandwidth; ``decode_7b``: whole decode steps of the
Qwen2.5-7B architecture for 512 sequences of ~2.8k tokens against the step's
HBM bound; ``rollout``: a GRPO rollout of the Qwen2.5-1.5B
architecture (random-init bf16, 4 prompts x group 8, 128 new tokens) through
PagedGenerator with CUDA-graph decode steps, next to stock HF generate on the
same model and batch; ``old_policy``: that rollout's old-policy
log-probabilities through PagedGenerator.score next to the reference's own
padded-forward pass; and ``speculative``: a speculative rollout (1.5B target,
0.5B draft, k = 4, 64 sequences) through PagedSpeculativeGenerator, next to
the plain paged rollout and HF's stock assisted generation.

Multi-GPU (torchrun): every rank owns its own 256 sequences and KV pool (weak
scaling, no data-path collective); the timed region is bracketed by NCCL
barriers and the elapsed time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "paged-decode tokens/s/GPU at Qwen2.5-1.5B shape; paged-attn HBM GB/s vs peak"
HQ, HKV, D, BS, POOL_BLOCKS, SEQS = 12, 2, 128, 16, 40000, 256
L2_BYTES = 126 * 2**20
FALLBACK_HBM_GBS = 6650.0
TIMING_EVERY = 4
FALLBACK_BF16_TFLOPS = 1590.0
E2E_REPEATS = 3
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": "paged KV microbench: one decode step (append 1 token/seq + paged GQA attention), 1 layer, "
                    f"{SEQS} seqs/GPU, ctx U[64,2048], {HQ}q/{HKV}kv heads, head_dim {D}, block {BS}, "
                    f"{POOL_BLOCKS}-block pool, random-permutation block placement, seed 0",
        "seqs_per_gpu": SEQS,
        "global_batch": SEQS * n_gpus,
        "l2": "inputs larger than L2: ~277 MB of K/V read per step vs 126 MB L2",
        "parallelism": f"replicas{n_gpus}: disjoint sequences and KV pool per GPU, no data-path collective",
    }


def algorithmic_bytes(lens: np.ndarray) -> int:
    """HBM bytes one fused decode launch must move (bf16): K/V read incl. the new token,
    the append (read k/v, write the slot), q read + o write, block-table and length reads."""
    b = len(lens)
    kv = int(lens.sum()) * HKV * D * 2 * 2
    append = b * HKV * D * 2 * 2 * 2
    qo = b * HQ * D * 2 * 2
    tables = int(((lens + BS - 1) // BS).sum()) * 4 + b * 4
    return kv + append + qo + tables


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak(sustained: bool = False) -> tuple[float, str]:
    """Dense bf16 TFLOP/s: the burst figure for a kernel timed on its own, the sustained one for a long run."""
    p = ROOT / "MEASURED_PEAKS.json"
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[key]), f"measured {key} (MEASURED_PEAKS.json)"
        except (KeyError, ValueError):
            pass
    return (FALLBACK_BF16_TFLOPS_SUSTAINED if sustained else FALLBACK_BF16_TFLOPS), "fallback bf16 TFLOP/s"


def tiles_traffic(which: str) -> float | None:
    """DRAM bytes per launch of the prefill / verify kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "tensor_tiles.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[which]["dram_bytes_per_launch"])
        except (KeyError, ValueError):
            return None
    return None


def ncu_traffic() -> float | None:
    """DRAM bytes per launch of the decode kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "paged_decode_microbench.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch"])
        except (KeyError, ValueError):
            return None
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML on a thread, from before the warm-up
    to the end of the last timed region; ``summary()`` keeps the samples taken inside the timed
    regions (``mark_start`` / ``mark_end``).  NVML is set up when the sampler is made, so that its
    start-up (tens of ms) never leaves the GPU idle right before a timed region."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.001, enabled: bool = True) -> None:
        self.samples: list[tuple[float, int, int]] = []
        self.windows: list[list[float]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        if not enabled:
            return
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nvml = None
        self.period = period_s

    def _run(self) -> None:
        n = self._nvml
        while not self._stop.is_set():
            try:
                t = time.perf_counter()
                mhz = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((0.5 * (t + time.perf_counter()), mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def mark_start(self) -> None:
        self.windows.append([time.perf_counter(), float("inf")])

    def mark_end(self) -> None:
        self.windows[-1][1] = time.perf_counter()

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        inside = [(m, r) for t, m, r in self.samples if any(a <= t <= b for a, b in self.windows)]
        where = "inside the timed regions"
        if not inside and self.samples and self.windows:
            # Regions shorter than one NVML round trip: the samples nearest to each region.
            where = "nearest to each timed region (no sample fell inside one)"
            for a, b in self.windows:
                _, m, r = min(self.samples, key=lambda x: min(abs(x[0] - a), abs(x[0] - b)))
                inside.append((m, r))
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        mhz = [m for m, _ in inside]
        active = 0
        for _, r in inside:
            active |= r
        reasons = [k for k, bit in self.REASONS.items() if active & bit and k != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_min_mhz": min(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz), "where": where, "regions": len(self.windows),
                "region_ms": round(sum(b - a for a, b in self.windows) * 1e3, 3)}


def build_workload(device: torch.device, seed: int):
    """Store + 256 sequences whose blocks follow a random permutation of the pool."""
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore
    from randomrepo_b200._lib import lib, raise_for_status

    gen = torch.Generator().manual_seed(seed)
    lengths = torch.randint(64, 2049, (SEQS,), generator=gen).numpy().astype(np.int64)
    perm = torch.randperm(POOL_BLOCKS, generator=gen).numpy()
    alloc = PagedKVAllocator(POOL_BLOCKS, BS)
    store = PagedKVCacheStore(alloc, num_layers=1, num_kv_heads=HKV, head_dim=D, dtype=torch.bfloat16,
                              device=device)
    h = alloc._handle
    # Placement through the public allocator: hold every block with a filler
    # sequence, then free exactly the block wanted next and grow into it (the
    # allocator always hands out the lowest free id, here the only one).
    filler0 = 1 << 40
    for b in range(POOL_BLOCKS):
        raise_for_status(lib.pkv_allocator_reserve(h, filler0 + b, 1))
    cursor = 0
    for sid, n in enumerate(lengths.tolist()):
        raise_for_status(lib.pkv_allocator_reserve(h, sid, 0))
        left = n
        while left > 0:
            raise_for_status(lib.pkv_allocator_release(h, filler0 + int(perm[cursor])))
            raise_for_status(lib.pkv_allocator_append_tokens(h, sid, min(BS, left)))
            cursor += 1
            left -= BS
    for b in perm[cursor:].tolist():
        raise_for_status(lib.pkv_allocator_release(h, filler0 + int(b)))
    store.pool.pool.normal_(generator=torch.Generator(device=device).manual_seed(seed))
    store._sync()
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    q = torch.randn((SEQS, HQ, D), device=device, generator=dgen).to(torch.bfloat16)
    kn = torch.randn((SEQS, HKV, D), device=device, generator=dgen).to(torch.bfloat16)
    vn = torch.randn((SEQS, HKV, D), device=device, generator=dgen).to(torch.bfloat16)
    return store, lengths, q, kn, vn, perm[:cursor]


def run_ours(args, rank: int, world: int, device: torch.device) -> dict | None:
    import torch.distributed as dist

    from randomrepo_b200._lib import lib

    store, lengths, q, kn, vn, _ = build_workload(device, args.seed + rank)
    ids = np.arange(SEQS, dtype=np.int64)
    out = torch.empty_like(q)
    alloc = store.allocator
    pool = store.pool

    def step(qq=q, kk=kn, vv=vn, oo=out):
        _, st = store.decode(ids, qq, kk, vv, layer=0, out=oo)
        alloc.truncate(ids, lengths)
        return st

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    # NVML and the launch-timing events are set up before the warm-up, so
    # that nothing leaves the GPU idle (and its clocks falling) between the
    # warm-up and a timed region: each region follows its warm-up steps
    # through one barrier only.
    # Rank 0 samples its GPU's clocks (it prints the line); the other ranks keep NVML off their hosts' CPUs.
    clocks = ClockSampler(device.index or 0, enabled=rank == 0)
    n_timed = args.steps // TIMING_EVERY + 1
    pool.time_launches(n_timed, TIMING_EVERY)
    pool.time_launches(0)
    clocks.__enter__()
    try:
        # The host-buffer regions run first: the first timed region of a
        # process runs a few percent slow (a probe of two ranks measured 62-65
        # against 56-60 us per step for the same region repeated), and their
        # reported figure is the median of three regions.
        # ---- end to end through the public API with host buffers -----------
        # Every step hands the store pinned host q/k/v (one packed buffer) and
        # a pinned host output: the native stepper copies the inputs in on its
        # copy stream ahead of the step descriptor and the output back out on
        # a second stream, so step i+1's input copy and step i-1's output copy
        # run while step i's kernels do.  The region ends after the last
        # output copy.
        from randomrepo_b200 import host_input_tensor

        nq, nk = q.numel(), kn.numel()
        inp_h = host_input_tensor((nq + 2 * nk,), q.dtype)  # page-locked, write-combined
        inp_h[:nq].copy_(q.reshape(-1).cpu())
        inp_h[nq:nq + nk].copy_(kn.reshape(-1).cpu())
        inp_h[nq + nk:].copy_(vn.reshape(-1).cpu())
        q_h, k_h, v_h = inp_h[:nq].view(q.shape), inp_h[nq:nq + nk].view(kn.shape), inp_h[nq + nk:].view(vn.shape)
        out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()

        def e2e_step():
            store.decode(ids, q_h, k_h, v_h, layer=0, out=out_h)
            alloc.truncate(ids, lengths)

        # Three timed regions of K steps each, each right after its warm-up
        # steps: PCIe and host time on these shared hosts vary from run to
        # run (other tenants), so the median is reported and all three are
        # listed.
        e2e_runs = []
        for _ in range(E2E_REPEATS):
            for _ in range(args.warmup):
                e2e_step()
            store.wait_host_outputs()
            barrier()
            clocks.mark_start()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                e2e_step()
            store.fence_host_outputs()  # every output copy issued in the region ends inside it
            e1.record()
            torch.cuda.synchronize(device)
            clocks.mark_end()
            ms = e0.elapsed_time(e1)
            if world > 1:
                t = torch.tensor([ms], device=device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            e2e_runs.append(ms)
        # ---- device-resident timing ----------------------------------------
        for _ in range(args.warmup - 1):
            step()
        # Every step sees the same lengths (each sequence is rolled back after
        # its step), so the algorithmic bytes of one step serve every launch.
        step_bytes = algorithmic_bytes(step().host_lens)
        # CUDA events recorded by the library right around every 4th decode
        # launch of the timed region (re-armed here without a CUDA call).
        pool.time_launches(n_timed, TIMING_EVERY)
        launches0 = pool.launch_count()
        wait0 = lib.pkv_stepper_host_wait_ns(pool.stepper)
        barrier()
        clocks.mark_start()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        h0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        h1 = time.perf_counter()
        t1.record()
        torch.cuda.synchronize(device)
        clocks.mark_end()
        wait_ns = lib.pkv_stepper_host_wait_ns(pool.stepper) - wait0
        launches = pool.launch_count() - launches0
        elapsed_ms = t0.elapsed_time(t1)
        kernel_ms = pool.launch_times_ms().tolist()
        pool.time_launches(0)
        if world > 1:
            t = torch.tensor([elapsed_ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            elapsed_ms = float(t.item())
        barrier()
        err = pool.decode_error_flag()
        if err:
            raise RuntimeError(f"decode kernel reported device error {err}")
        host_wall_us = (h1 - h0) * 1e6 / args.steps
        host_busy_us = ((h1 - h0) * 1e9 - wait_ns) / 1e3 / args.steps

    finally:
        clocks.__exit__(None, None, None)
    e2e_ms = statistics.median(e2e_runs)
    barrier()
    h2d = inp_h.numel() * inp_h.element_size() + (6 * SEQS + 1) * 4
    d2h = out_h.numel() * out_h.element_size()

    # The sharded rollout runs on every rank (its gathers are collectives): at N > 1 before rank 0
    # goes on alone; at N = 1 after the other lines.
    grpo = None
    if world > 1 and not args.no_rollout:
        grpo = run_grpo_rollout(device, args.seed, rank, world)
    if rank != 0:
        return None
    ms_per_step = elapsed_ms / args.steps
    value = world * SEQS * 1000.0 / ms_per_step
    mean_kernel_ms = statistics.mean(kernel_ms)
    achieved = step_bytes / (mean_kernel_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    result = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/Q, ctx U[64,2048])",
        "config": workload_config(world),
        "per_gpu_tokens_per_s": value / world,
        "roofline": {
            "bound": "hbm",
            "kernel": "pkv_decode_attention: paged_decode_kernel<128, 2, bf16> (fused append + split-K GQA "
                      "decode) + paged_decode_combine_kernel, timed together per launch",
            "achieved": achieved,
            "peak": peak,
            "peak_source": f"{peak_kind} hbm_gbs" + (" (MEASURED_PEAKS.json)" if peak_kind == "measured" else ""),
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": ncu_traffic(),
            "algorithmic_bytes_per_launch": step_bytes,
            "kernel_ms_mean": mean_kernel_ms,
            "kernel_timing": f"CUDA events around every {TIMING_EVERY}th decode launch of the timed region "
                             f"({len(kernel_ms)} launches)",
            "kernel_ms_min": min(kernel_ms),
        },
        "e2e": {
            "value": world * SEQS * 1000.0 / (e2e_ms / args.steps),
            "runs_tokens_per_s": [world * SEQS * 1000.0 / (ms / args.steps) for ms in e2e_runs],
            "timing": f"median of {E2E_REPEATS} timed regions of {args.steps} steps (max over ranks each)",
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "path": "PagedKVCacheStore.decode given host q/k/v (one packed page-locked write-combined buffer "
                    "from host_input_tensor) and a page-locked host output: pkv_stepper_step_host copies the "
                    "inputs in on the stepper's copy stream with the step descriptor and the output out on a "
                    "second stream, every step; the region ends after the last output copy",
        },
        "gpu_launches": launches,
        "host_us_per_step": host_busy_us,
        "host_wall_us_per_step": host_wall_us,
        "host_timing": "host_us_per_step: wall time of the timed loop per step minus the time the host spent "
                       "blocked on the stepper's staging ring (pkv_stepper_host_wait_ns), i.e. the host's own "
                       "work per step; host_wall_us_per_step includes those waits",
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_tiles:
        del store, q, kn, vn, out, q_h, k_h, v_h, inp_h, out_h
        torch.cuda.empty_cache()
        result["tensor_tiles"] = run_tensor_tiles(device, args.seed, args.steps, args.warmup)
    if world == 1 and not args.no_tiles:
        result["vocab_rows"] = run_vocab_rows(device, args.seed, args.steps, args.warmup)
    if world == 1 and not args.no_rollout:
        result["rollout"], result["old_policy"] = run_rollout(device, args.seed)
        result["speculative"] = run_speculative(device, args.seed)
        result["decode_7b"] = run_decode_7b(device, args.seed)
        result["rollout_7b"] = run_rollout_7b(device, args.seed)
    if world == 1 and not args.no_rollout:
        grpo = run_grpo_rollout(device, args.seed, rank, world)
    if grpo is not None:
        result["grpo_rollout"] = grpo
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(lengths, args.cpu_seconds)
    # Last key of the line, so that a tail of the output still shows it.
    result["summary"] = summarize(result)
    return result


def summarize(result: dict) -> dict:
    """The line's headline figures in a few short keys (the fractions are of the measured peaks)."""

    def get(*path):
        d = result
        for k in path:
            if not isinstance(d, dict) or k not in d:
                return None
            d = d[k]
        return round(d, 4) if isinstance(d, float) else d

    out = {
        "decode_tokens_per_s": get("value"),
        "e2e_tokens_per_s": get("e2e", "value"),
        "ms_per_step": get("ms_per_step"),
        "kernel_ms_mean": get("roofline", "kernel_ms_mean"),
        "decode_hbm_frac": get("roofline", "frac"),
        "host_us_per_step": get("host_us_per_step"),
        "prefill_tensor_frac": get("tensor_tiles", "prefill", "roofline", "frac"),
        "verify_hbm_frac": get("tensor_tiles", "verify", "roofline", "frac"),
        "verify_long_hbm_frac": get("tensor_tiles", "verify_long", "roofline", "frac"),
        "logprobs_hbm_frac": get("vocab_rows", "token_logprobs", "roofline", "frac"),
        "rollout_tokens_per_s": get("rollout", "tokens_per_s"),
        "speculative_tokens_per_s": get("speculative", "tokens_per_s"),
        "decode_7b_hbm_bound_frac": get("decode_7b", "frac_of_hbm_bound"),
        "rollout_7b_tokens_per_s": get("rollout_7b", "tokens_per_s"),
        "grpo_rollout_tokens_per_s": get("grpo_rollout", "tokens_per_s"),
        "cpu_baseline_tokens_per_s": get("cpu_baseline", "value"),
    }
    return {k: v for k, v in out.items() if v is not None}


PREFILL_SHAPE = {"model": "Qwen2.5-7B attention", "hq": 28, "hkv": 4, "d": 128, "prompts": 32, "len_lo": 256,
                 "len_hi": 4096, "chunk": 512}
VERIFY_LONG_SHAPE = {"model": "Qwen2.5-1.5B target attention", "hq": 12, "hkv": 2, "d": 128, "seqs": 32,
                     "prefix_lo": 4096, "prefix_hi": 16384, "k": 4}
VERIFY_SHAPE = {"model": "Qwen2.5-1.5B target attention", "hq": 12, "hkv": 2, "d": 128, "seqs": 64, "prefix_lo": 128,
                "prefix_hi": 1280, "k": 4}


def _tile_workload(device: torch.device, hq: int, hkv: int, d: int, seqs, seed: int, verify: bool = False):
    """A store whose sequences hold ``total`` tokens of seeded N(0,1) K/V and the planned
    items for the chunks ``(past, q_len)`` of each sequence (``verify``: for pkv_verify_attention,
    as ``prefill_step`` plans short chunks; else for pkv_prefill_attention); q is seeded N(0,1)."""
    from randomrepo_b200 import PagedKVAllocator, PagedKVCacheStore
    from randomrepo_b200.device import plan_prefill, plan_verify

    total = sum(n for n, _ in seqs)
    store = PagedKVCacheStore(PagedKVAllocator(total // BS + len(seqs) + 64, BS), num_layers=1, num_kv_heads=hkv,
                              head_dim=d, dtype=torch.bfloat16, device=device)
    store.pool.pool.normal_(generator=torch.Generator(device=device).manual_seed(seed))
    rows, past, qls = [], [], []
    for sid, (n, chunks) in enumerate(seqs):
        store.reserve(sid, n)
        for p0, ql in chunks:
            rows.append(store.allocator.row(sid))
            past.append(p0)
            qls.append(ql)
    store._sync()
    planner = plan_verify if verify else plan_prefill
    plan = planner(np.array(rows), np.array(past), np.array(qls), hq, hkv, store.pool.num_sms)
    q = torch.randn((sum(qls), hq, d), device=device,
                    generator=torch.Generator(device=device).manual_seed(seed + 1)).to(torch.bfloat16)
    pos_sum = sum(int((np.arange(p0, p0 + ql, dtype=np.int64) + 1).sum()) for p0, ql in zip(past, qls))
    flops = 4 * hq * d * pos_sum
    kv_bytes = sum((p0 + ql) * hkv * d * 2 * 2 for p0, ql in zip(past, qls))
    return store, q, plan, torch.from_numpy(plan.records).to(device), flops, kv_bytes


class _L2Flush:
    """Empties L2 between timed launches: writes a buffer twice the size of L2, then reads a second
    one of that size, so that the written lines have gone back to HBM before the timed launch
    starts (otherwise their write-back would land on the timed kernel's HBM traffic)."""

    def __init__(self, device: torch.device) -> None:
        self.w = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)
        self.r = torch.zeros(2 * L2_BYTES // 4, dtype=torch.int32, device=device)
        self.sink = torch.empty(1, dtype=torch.int64, device=device)

    def __call__(self) -> None:
        self.w.zero_()
        torch.sum(self.r, dim=0, keepdim=True, out=self.sink)


def _time_prefill(store, q, plan, records, steps: int, warmup: int) -> tuple[float, int]:
    """Mean device ms of one pkv_prefill_attention launch (L2 flushed before each) and launches timed."""
    pool = store.pool
    out = torch.empty_like(q)
    scale = q.shape[2] ** -0.5
    for _ in range(warmup):
        pool.prefill(0, q, plan, records, q.shape[1], scale, out)
    flush = _L2Flush(q.device)
    launches0 = pool.launch_count()
    times = []
    for _ in range(steps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        pool.prefill(0, q, plan, records, q.shape[1], scale, out)
        e1.record()
        torch.cuda.synchronize(q.device)
        times.append(e0.elapsed_time(e1))
    if pool.prefill_error_flag():
        raise RuntimeError(f"prefill kernel reported device error {pool.prefill_error_flag()}")
    return statistics.mean(times), pool.launch_count() - launches0


def _verify_line(device: torch.device, vs: dict, rng, seed: int, steps: int, warmup: int, hbm: float,
                 hbm_kind: str, name: str) -> dict:
    """One verify launch shape on the verify kernel, with the 128-query-row prefill kernel timed
    on the same launch for comparison."""
    pre = rng.integers(vs["prefix_lo"], vs["prefix_hi"] + 1, size=vs["seqs"])
    seqs = [(int(p) + vs["k"], [(int(p) - 1, vs["k"] + 1)]) for p in pre]
    store, q, plan, records, flops, kv_bytes = _tile_workload(device, vs["hq"], vs["hkv"], vs["d"], seqs, seed + 2)
    ms_rows, _ = _time_prefill(store, q, plan, records, max(10, steps // 5), warmup)
    del store, q, records
    store, q, plan, records, flops, kv_bytes = _tile_workload(device, vs["hq"], vs["hkv"], vs["d"], seqs, seed + 2,
                                                              verify=True)
    ms, launches = _time_prefill(store, q, plan, records, max(10, steps // 5), warmup)
    achieved = kv_bytes / (ms * 1e-3) / 1e9
    line = {
        "workload": f"speculative-verify attention, 1 layer, {vs['model']} ({vs['hq']}q/{vs['hkv']}kv heads, "
                    f"head_dim {vs['d']}), {vs['seqs']} sequences with prefix U[{vs['prefix_lo']},"
                    f"{vs['prefix_hi']}], k={vs['k']} drafts: {vs['k'] + 1} causal queries each, bf16, seed {seed}",
        "ms": ms, "work_items": plan.n_items, "ctas": plan.n_ctas, "combine_entries": plan.n_combine,
        "gpu_launches": launches,
        "tokens_per_s": vs["seqs"] * (vs["k"] + 1) / (ms * 1e-3),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"{hbm_kind} hbm_gbs", "traffic": tiles_traffic(name), "bytes_per_launch": kv_bytes,
                     "bytes_rule": "K and V of prefix + k tokens per sequence and KV head"},
        "tflops": flops / (ms * 1e-3) / 1e12,
        "kernel": "pkv_verify_attention (keys on the tensor-core rows) + combine",
        "prefill_kernel_ms": ms_rows,
    }
    del store, q, records
    torch.cuda.empty_cache()
    return line


def run_tensor_tiles(device: torch.device, seed: int, steps: int, warmup: int) -> dict:
    """The tcgen05 chunked-prefill and speculative-verify attention kernels on their own workloads."""
    hbm, hbm_kind = measured_peaks()
    tflops_peak, tflops_kind = measured_tensor_peak()
    rng = np.random.default_rng(seed)
    res = {}
    ps = PREFILL_SHAPE
    lens = rng.integers(ps["len_lo"], ps["len_hi"] + 1, size=ps["prompts"])
    seqs = [(int(n), [(c0, min(ps["chunk"], int(n) - c0)) for c0 in range(0, int(n), ps["chunk"])]) for n in lens]
    store, q, plan, records, flops, kv_bytes = _tile_workload(device, ps["hq"], ps["hkv"], ps["d"], seqs, seed)
    ms, launches = _time_prefill(store, q, plan, records, max(5, steps // 10), warmup)
    achieved = flops / (ms * 1e-3) / 1e12
    res["prefill"] = {
        "workload": f"chunked-prefill attention, 1 layer, {ps['model']} ({ps['hq']}q/{ps['hkv']}kv heads, head_dim "
                    f"{ps['d']}), {ps['prompts']} prompts of U[{ps['len_lo']},{ps['len_hi']}] tokens, every "
                    f"{ps['chunk']}-token chunk of every prompt in one launch (causal after its past), bf16, "
                    f"seed {seed}",
        "ms": ms, "work_items": plan.n_items, "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tflops_peak, "unit": "TFLOP/s",
                     "frac": achieved / tflops_peak, "peak_source": tflops_kind, "traffic": tiles_traffic("prefill"),
                     "flops_per_launch": flops, "flops_rule": "4 * Hq * D * sum over queries of (position + 1)"},
        "kv_gb_per_launch": kv_bytes / 1e9,
    }
    del store, q, records
    for name, vs in (("verify", VERIFY_SHAPE), ("verify_long", VERIFY_LONG_SHAPE)):
        res[name] = _verify_line(device, vs, rng, seed, steps, warmup, hbm, hbm_kind, name)
    return res


ROLLOUT_SHAPE = {"prompts": 4, "group": 8, "len_lo": 64, "len_hi": 256, "new_tokens": 128, "temperature": 1.0}
SPEC_SHAPE = {"prompts": 8, "group": 8, "len_lo": 64, "len_hi": 256, "new_tokens": 64, "k": 4, "temperature": 1.0}
QWEN_1P5B = dict(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=28,
                 num_attention_heads=12, num_key_value_heads=2, max_position_embeddings=32768,
                 rope_theta=1000000.0, tie_word_embeddings=True)
QWEN_0P5B = dict(vocab_size=151936, hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                 num_attention_heads=14, num_key_value_heads=2, max_position_embeddings=32768,
                 rope_theta=1000000.0, tie_word_embeddings=True)


def _qwen(device: torch.device, arch: dict, seed: int):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    with torch.device(device):
        return Qwen2ForCausalLM(Qwen2Config(**arch, attn_implementation="sdpa")).to(torch.bfloat16).eval()


def _set_attention(model, name: str) -> None:
    model.config._attn_implementation = name
    for sub in model.modules():
        cfg = getattr(sub, "config", None)
        if cfg is not None:
            cfg._attn_implementation = name


def _timed(device: torch.device, fn):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    e0.record()
    n = fn()
    e1.record()
    torch.cuda.synchronize(device)
    return n, e0.elapsed_time(e1) / 1e3


def run_rollout(device: torch.device, seed: int, iters: int = 2) -> tuple[dict, dict]:
    """GRPO rollout at the Qwen2.5-1.5B architecture, random-init bf16: PagedGenerator (CUDA-graph
    decode steps, packed prefill, forked group prompts) against stock HF generate on the same batch;
    then the old-policy log-probabilities of that rollout (score) against the reference's own pass."""
    from randomrepo_b200.hf import PagedGenerator, SamplingConfig, make_store

    rs = ROLLOUT_SHAPE
    model = _qwen(device, QWEN_1P5B, seed)
    rng = np.random.default_rng(seed)
    lens = rng.integers(rs["len_lo"], rs["len_hi"] + 1, size=rs["prompts"])
    prompts = [torch.from_numpy(rng.integers(0, QWEN_1P5B["vocab_size"], size=int(n))) for n in lens]
    group, new = rs["group"], rs["new_tokens"]

    ids = torch.zeros((len(prompts) * group, int(lens.max())), dtype=torch.long)
    mask = torch.zeros_like(ids)
    for g, p in enumerate(prompts):
        ids[g * group:(g + 1) * group, -p.numel():] = p
        mask[g * group:(g + 1) * group, -p.numel():] = 1
    ids, mask = ids.to(device), mask.to(device)

    def hf():
        with torch.inference_mode():
            out = model.generate(ids, attention_mask=mask, max_new_tokens=new, do_sample=True,
                                 temperature=rs["temperature"], top_p=1.0, top_k=0, pad_token_id=0)
        return (out.shape[1] - ids.shape[1]) * out.shape[0]

    # Stock HF first: PagedGenerator switches the model's attention implementation.
    hf()
    hf_runs = [_timed(device, hf) for _ in range(iters)]
    store = make_store(model, total_blocks=4096)
    gen = PagedGenerator(model, store, prefill_chunk_size=512, cuda_graphs=True)
    last = {}

    def ours(it):
        r = gen.generate(prompts, group_size=group, max_new_tokens=new, first_id=it * 10000,
                         sampling=SamplingConfig(do_sample=True, temperature=rs["temperature"], seed=it))
        last["r"] = r
        return sum(len(t) for t in r["tokens"])

    ours(0)  # records the decode-step graph
    ours_runs = [_timed(device, lambda it=it: ours(it)) for it in range(1, iters + 1)]
    if store.pool.decode_error_flag() or store.pool.prefill_error_flag():
        raise RuntimeError("rollout kernels reported a device error")
    ours_tps = sum(n for n, _ in ours_runs) / sum(t for _, t in ours_runs)
    hf_tps = sum(n for n, _ in hf_runs) / sum(t for _, t in hf_runs)
    rollout = {
        "workload": f"GRPO rollout, Qwen2.5-1.5B architecture (28 layers, 12q/2kv heads, head_dim 128, vocab "
                    f"151936), random-init bf16, {rs['prompts']} prompts x group {group}, prompts "
                    f"U[{rs['len_lo']},{rs['len_hi']}] random ids, {new} new tokens, temperature "
                    f"{rs['temperature']}, seed {seed}",
        "tokens_per_s": ours_tps,
        "path": "PagedGenerator: packed prefill kernel, one prefill per group + copy-on-write forks, CUDA-graph "
                "decode steps (fused append + paged decode per layer; fused RMSNorm / rotary / SiLU launches and "
                "packed q|k|v and gate|up GEMMs), fp32 logits, device sampling kernel",
        "hf_generate_tokens_per_s": hf_tps,
        "hf_generate_path": "stock HF generate on the same model and batch (SDPA + DynamicCache, left-padded)",
        "speedup_vs_hf_generate": ours_tps / hf_tps,
        "timing": f"CUDA events around whole rollouts, mean of {iters} after one warm-up each",
    }
    old = run_old_policy(device, model, gen, prompts, last["r"], group, iters)
    del gen, store, model
    torch.cuda.empty_cache()
    return rollout, old


def run_grpo_rollout(device: torch.device, seed: int, rank: int, world: int, iters: int = 2) -> dict:
    """GRPO rollout sharded by groups, one rank per GPU, with the per-step gather the trainer needs.

    Every rank draws the same 4 x world prompts (Qwen2.5-1.5B architecture, random-init bf16, prompts
    U[64, 256], group 8, 128 new tokens, temperature 1.0), owns the groups ``assign_groups`` gives it
    (balanced by prompt tokens x group size), rolls them out with PagedGenerator (CUDA-graph decode
    steps, its own KV pool) and gathers every decode step's (sequence id, token, log-probability) rows
    of all ranks, GATHER_EVERY steps per NCCL all_gather_into_tensor (StepGather); no KV crosses GPUs.
    Ranks whose loops ran fewer steps add empty steps, so every rank makes the same collectives.  Timed with CUDA events per rank, max over ranks; tokens are summed over ranks."""
    import torch.distributed as dist

    from randomrepo_b200.hf import PagedGenerator, SamplingConfig, make_store
    from randomrepo_b200.sharding import StepGather, assign_groups, balance_ratio, groups_of_rank

    rs = ROLLOUT_SHAPE
    group, new = rs["group"], rs["new_tokens"]
    n_prompts = rs["prompts"] * world
    rng = np.random.default_rng(seed)
    lens = rng.integers(rs["len_lo"], rs["len_hi"] + 1, size=n_prompts)
    prompts = [torch.from_numpy(rng.integers(0, QWEN_1P5B["vocab_size"], size=int(n))) for n in lens]
    assignment = assign_groups(lens, group, world)
    mine = groups_of_rank(assignment, rank)
    model = _qwen(device, QWEN_1P5B, seed)
    store = make_store(model, total_blocks=4096)
    gen = PagedGenerator(model, store, prefill_chunk_size=512, cuda_graphs=True)
    max_rows = group * max(len(groups_of_rank(assignment, r)) for r in range(world))
    gather = StepGather(max_rows * GATHER_EVERY, device) if world > 1 else None
    host = {"s": 0.0, "rows": 0}
    pending: list[tuple] = []

    def flush():
        if pending:
            ids = torch.cat([torch.tensor(i, dtype=torch.int64) for i, _, _ in pending])
            gather.start(ids, torch.cat([t for _, t, _ in pending]), torch.cat([lp for _, _, lp in pending]))
            pending.clear()

    def hook(ids, tok, lp):
        # Every step's rows, gathered GATHER_EVERY steps at a time: one rendezvous of the ranks per
        # GATHER_EVERY decode steps instead of one per step.
        if gather is None:
            return
        t = time.perf_counter()
        pending.append((ids, tok, lp))
        if len(pending) == GATHER_EVERY:
            flush()
        host["s"] += time.perf_counter() - t

    def rollout(it: int) -> tuple[int, float, float]:
        host["s"] = 0.0
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = gen.generate([prompts[g] for g in mine], group_size=group, max_new_tokens=new, first_id=it * 100000,
                         sampling=SamplingConfig(do_sample=True, temperature=rs["temperature"], seed=it),
                         step_callback=hook)
        if gather is not None:
            steps = torch.tensor([r["steps"]], device=device)
            dist.all_reduce(steps, op=dist.ReduceOp.MAX)
            empty = torch.zeros(0, dtype=torch.int64, device=device)
            for _ in range(int(steps.item()) - r["steps"]):
                hook([], empty, torch.zeros(0, device=device))
            flush()
            t = time.perf_counter()
            rows = gather.finish()
            host["wait_s"] = time.perf_counter() - t
            host["rows"] = sum(len(x.tokens) for x in rows)
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        return sum(len(t) for t in r["tokens"]), ms, host["s"] * 1e3

    rollout(0)  # records the decode-step graphs
    runs = [rollout(it) for it in range(1, iters + 1)]
    if store.pool.decode_error_flag() or store.pool.prefill_error_flag():
        raise RuntimeError("rollout kernels reported a device error")
    tokens = sum(n for n, _, _ in runs)
    ms = sum(t for _, t, _ in runs)
    gather_ms = sum(g for _, _, g in runs)
    if world > 1:
        t = torch.tensor([float(tokens), ms, gather_ms], device=device, dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tokens, ms, gather_ms = float(t[0].item()), float(mx[1].item()), float(mx[2].item())
    del gen, store, model
    torch.cuda.empty_cache()
    return {
        "workload": f"GRPO rollout sharded by groups: {rs['prompts']} prompts x group {group} per GPU "
                    f"({n_prompts} prompts on {world} GPU(s)), Qwen2.5-1.5B architecture, random-init bf16, "
                    f"prompts U[{rs['len_lo']},{rs['len_hi']}], {new} new tokens, temperature "
                    f"{rs['temperature']}, seed {seed}",
        "tokens_per_s": tokens / (ms * 1e-3),
        "tokens_per_s_per_gpu": tokens / (ms * 1e-3) / world,
        "ms_per_rollout": ms / iters,
        "gather_host_ms_per_rollout": gather_ms / iters,
        "gather_every_steps": GATHER_EVERY,
        "gathered_rows_per_rollout": host["rows"],
        "group_balance": balance_ratio(lens, group, assignment, world),
        "path": "per rank: PagedGenerator with CUDA-graph decode steps on its own KV pool; one "
                f"NCCL all_gather_into_tensor per {GATHER_EVERY} decode steps of every step's (sequence id, token, "
                "log-probability) rows (StepGather.start: it runs behind the next steps' work; StepGather.finish "
                "collects all rows at the end)"
                if world > 1 else "PagedGenerator with CUDA-graph decode steps (no collective at one GPU)",
        "timing": f"CUDA events around whole rollouts (every gather completed inside), {iters} after one warm-up; "
                  "max over ranks of the time, sum over ranks of the tokens; gather_host_ms = host time in the "
                  "gather calls, the final wait excluded (max over ranks)",
    }


GATHER_EVERY = 16  # decode steps whose rows one gather carries

ROLLOUT_7B_SHAPE = {"prompts": 64, "group": 8, "len_lo": 256, "len_hi": 4096, "new_tokens": 1024,
                    "temperature": 1.0, "pool_fraction": 0.6}


def run_rollout_7b(device: torch.device, seed: int) -> dict:
    """The Qwen2.5-7B rollout under KV pressure: 64 prompts x group 8 = 512 sequences, prompts
    U[256, 4096], 1024 new tokens, temperature 1.0, random-init bf16, through PagedGenerator with a
    KV pool of 60 % of the blocks the rollout's peak would hold (shared prompt blocks + every
    sequence's generated blocks), so growth admission defers sequences and evicts / re-prefills when
    nothing can grow.  Timed once with CUDA events after a short warm-up rollout that records the
    decode graphs."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from randomrepo_b200.hf import PagedGenerator, SamplingConfig, kv_geometry, make_store

    sh = ROLLOUT_7B_SHAPE
    rng = np.random.default_rng(seed)
    lens = rng.integers(sh["len_lo"], sh["len_hi"] + 1, size=sh["prompts"])
    prompts = [torch.from_numpy(rng.integers(0, QWEN_7B["vocab_size"], size=int(n))) for n in lens]
    group, new, bs = sh["group"], sh["new_tokens"], 16
    peak_blocks = int(sum(-(-int(n) // bs) for n in lens)) + sh["prompts"] * group * (-(-new // bs) + 1)
    blocks = int(peak_blocks * sh["pool_fraction"])
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM._from_config(Qwen2Config(**QWEN_7B, attn_implementation="sdpa"),
                                              dtype=torch.bfloat16).eval()
    store = make_store(model, total_blocks=blocks)
    gen = PagedGenerator(model, store, prefill_chunk_size=512, cuda_graphs=True)
    cfg = SamplingConfig(do_sample=True, temperature=sh["temperature"], seed=1)
    gen.generate(prompts[:8], group_size=group, max_new_tokens=32, sampling=cfg)  # records graphs
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    r = gen.generate(prompts, group_size=group, max_new_tokens=new, first_id=100000, sampling=cfg)
    e1.record()
    torch.cuda.synchronize(device)
    s = e0.elapsed_time(e1) / 1e3
    if store.pool.decode_error_flag() or store.pool.prefill_error_flag():
        raise RuntimeError("rollout kernels reported a device error")
    n_tok = sum(len(t) for t in r["tokens"])
    layers, hkv, d = kv_geometry(model.config)
    per_block = layers * hkv * d * 2 * 2 * bs
    timings = dict(gen.last_timings)
    # The same rollout with a pool that holds its peak (no pressure), for comparison.
    del gen, store
    torch.cuda.empty_cache()
    store = make_store(model, total_blocks=peak_blocks + 512)
    gen = PagedGenerator(model, store, prefill_chunk_size=512, cuda_graphs=True)
    gen.generate(prompts[:8], group_size=group, max_new_tokens=32, sampling=cfg)
    torch.cuda.synchronize(device)
    e0.record()
    r2 = gen.generate(prompts, group_size=group, max_new_tokens=new, first_id=200000, sampling=cfg)
    e1.record()
    torch.cuda.synchronize(device)
    s2 = e0.elapsed_time(e1) / 1e3
    if store.pool.decode_error_flag() or store.pool.prefill_error_flag():
        raise RuntimeError("rollout kernels reported a device error")
    out = {
        "workload": f"GRPO rollout, Qwen2.5-7B architecture (28 layers, 28q/4kv heads, head_dim 128, vocab 152064), "
                    f"random-init bf16, {sh['prompts']} prompts x group {group} = {sh['prompts'] * group} sequences, "
                    f"prompts U[{sh['len_lo']},{sh['len_hi']}] random ids, {new} new tokens, temperature "
                    f"{sh['temperature']}, seed {seed}",
        "tokens_per_s": n_tok / s,
        "seconds": s,
        "decode_loop_iterations": r["steps"],
        "kv_pool_gb": blocks * per_block / 1e9,
        "kv_pool_blocks": blocks,
        "kv_peak_demand_blocks": peak_blocks,
        "kv_pressure": r["kv_pressure"],
        "prefill_ms": timings.get("prefill_ms"),
        "decode_ms": timings.get("decode_ms"),
        "unpressured_tokens_per_s": sum(len(t) for t in r2["tokens"]) / s2,
        "unpressured_kv_pool_gb": (peak_blocks + 512) * per_block / 1e9,
        "unpressured_decode_loop_iterations": r2["steps"],
        "path": "PagedGenerator: packed chunked prefill (512), one prefill per group + copy-on-write forks, CUDA-graph "
                "decode steps (eager when a full pool could not take a graph's padding), growth admission with soft "
                "preemption, eviction when more than a quarter of the batch would wait, evicted group members re-prefilled "
                "together (prompt once + forks + their own tokens), device sampling",
        "timing": "CUDA events around one whole rollout after a 32-token warm-up rollout of 8 groups (each pool)",
        "gpu_memory_gb": torch.cuda.max_memory_allocated(device) / 1e9,
    }
    del gen, store, model
    torch.cuda.empty_cache()
    return out


QWEN_7B = dict(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
               num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=32768,
               rope_theta=1000000.0, tie_word_embeddings=False)
DECODE_7B_SHAPE = {"seqs": 512, "prompt_lo": 256, "prompt_hi": 4096, "generated": 512, "steps": 16, "warmup": 3,
                   "temperature": 1.0}


def run_decode_7b(device: torch.device, seed: int) -> dict:
    """Decode steps of a 7B-shape rollout in its KV-bound middle: Qwen2.5-7B architecture (28 layers,
    28q/4kv heads, head_dim 128, vocab 152064), random-init bf16, 512 sequences each holding a prompt
    of U[256, 4096] tokens plus 512 generated ones (random K/V in the pages: the step's cost does not
    depend on their values).  One step = the whole forward for one token per sequence (CUDA graph:
    fused append + paged decode per layer), fp32 logits and the device sampling kernel.  Reported
    against the step's HBM bound: weights (all but the input embedding, of which 512 rows are read)
    + every sequence's K/V + the appended K/V + the fp32 logits, and against the bf16 tensor time of
    its FLOPs."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from randomrepo_b200.hf import PagedGenerator, kv_geometry, make_store

    sh = DECODE_7B_SHAPE
    rng = np.random.default_rng(seed)
    n = sh["seqs"]
    ctx = rng.integers(sh["prompt_lo"], sh["prompt_hi"] + 1, size=n) + sh["generated"]
    total_steps = sh["warmup"] + sh["steps"] + 1
    bs = 16
    blocks = int(sum(-(-(int(c) + total_steps) // bs) for c in ctx)) + 256
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM._from_config(Qwen2Config(**QWEN_7B, attn_implementation="sdpa"),
                                              dtype=torch.bfloat16).eval()
    store = make_store(model, total_blocks=blocks)
    for sid, c in enumerate(ctx.tolist()):
        store.reserve(sid, int(c))
    store.pool.pool.normal_(generator=torch.Generator(device=device).manual_seed(seed))
    gen = PagedGenerator(model, store, cuda_graphs=True)
    gen.reserve_tables(int(ctx.max()) + total_steps + bs)
    sampler = gen.sampler
    ids = list(range(n))
    tok = torch.from_numpy(rng.integers(0, QWEN_7B["vocab_size"], size=n)).to(device)

    def step(t):
        logits = gen.decode_step(ids, t)
        return sampler.sample(logits, temperature=sh["temperature"])[0]

    for _ in range(sh["warmup"]):
        tok = step(tok)
    lens0 = ctx + sh["warmup"]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    e0.record()
    for _ in range(sh["steps"]):
        tok = step(tok)
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / sh["steps"]
    if store.pool.decode_error_flag():
        raise RuntimeError("decode kernels reported a device error")

    layers, hkv, d = kv_geometry(model.config)
    kv_token = layers * hkv * d * 2 * 2
    embed = model.get_input_embeddings().weight
    w_bytes = sum(p.numel() * p.element_size() for p in model.parameters()) - embed.numel() * embed.element_size()
    w_bytes += n * embed.shape[1] * embed.element_size()
    kv_bytes = float(np.mean([(lens0 + i + 1).sum() for i in range(sh["steps"])])) * kv_token
    logit_bytes = n * QWEN_7B["vocab_size"] * 4
    step_bytes = w_bytes + kv_bytes + n * kv_token + logit_bytes
    matmul_params = sum(p.numel() for nm, p in model.named_parameters() if p.dim() == 2 and "embed" not in nm)
    flops = 2.0 * n * matmul_params + 4.0 * QWEN_7B["num_attention_heads"] * d * layers * (kv_bytes / kv_token)
    hbm, hbm_kind = measured_peaks()
    tf, tf_kind = measured_tensor_peak(sustained=True)
    t_hbm = step_bytes / (hbm * 1e9) * 1e3
    t_tensor = flops / (tf * 1e12) * 1e3
    res = {
        "workload": f"decode steps at the Qwen2.5-7B architecture, random-init bf16, {n} sequences of "
                    f"U[{sh['prompt_lo']},{sh['prompt_hi']}] prompt + {sh['generated']} generated tokens "
                    f"(mean context {float(ctx.mean()):.0f}), temperature {sh['temperature']}, seed {seed}",
        "tokens_per_s": n * 1e3 / ms,
        "ms_per_step": ms,
        "path": "PagedGenerator.decode_step (CUDA graph: 28 x fused append + paged decode, fused RMSNorm / "
                "rotary / SiLU launches, packed q|k|v and gate|up GEMMs through cuBLAS, fp32 LM head) + "
                "DeviceSampler.sample",
        "bytes_per_step": step_bytes,
        "bytes_rule": "weights except the input embedding (+ the 512 embedding rows read) + K/V of every "
                      "sequence's context + the appended K/V + fp32 logits",
        "kv_bytes_per_step": kv_bytes,
        "flops_per_step": flops,
        "hbm_bound_ms": t_hbm,
        "tensor_bound_ms": t_tensor,
        "frac_of_hbm_bound": t_hbm / ms,
        "peaks": f"{hbm_kind} hbm_gbs {hbm}; {tf_kind} {tf}",
        "timing": f"CUDA events around {sh['steps']} steps after {sh['warmup']} warm-up steps (the first "
                  f"records the graph); ~{kv_bytes / 1e9:.0f} GB of K/V per step, far above L2",
        "gpu_memory_gb": torch.cuda.max_memory_allocated(device) / 1e9,
    }
    del gen, store, model
    torch.cuda.empty_cache()
    return res


def run_old_policy(device: torch.device, model, gen, prompts, roll: dict, group: int, iters: int) -> dict:
    """Old-policy log-probabilities of a finished rollout (agentrl/core/rollout.py:456-472).

    Reference: its own pass -- one HF forward over the right-padded [B, L]
    batch, log_softmax over [B, L-1, vocab], gather, completion mask.  Ours:
    PagedGenerator.score (group prompt prefilled once + forks, packed prefill,
    logits only for scored rows, fused log-softmax + gather kernel)."""
    rows = [torch.cat([prompts[i // group], torch.tensor(t, dtype=torch.long)]) for i, t in enumerate(roll["tokens"])]
    width = max(r.numel() for r in rows)
    ids = torch.zeros(len(rows), width, dtype=torch.long)
    am = torch.zeros_like(ids)
    cm = torch.zeros(len(rows), width, dtype=torch.bool)
    for i, r in enumerate(rows):
        ids[i, :r.numel()] = r
        am[i, :r.numel()] = 1
        cm[i, prompts[i // group].numel():r.numel()] = True
    ids_d, am_d, cm_d = ids.to(device), am.to(device), cm.to(device)
    scored = int(cm[:, 1:].sum())

    def reference():
        with torch.inference_mode():
            logits = model(input_ids=ids_d, attention_mask=am_d).logits
            token_logprobs = torch.log_softmax(logits[:, :-1, :], dim=-1)
            gathered = token_logprobs.gather(dim=-1, index=ids_d[:, 1:].unsqueeze(-1)).squeeze(-1)
            aligned = torch.zeros_like(ids_d, dtype=logits.dtype)
            aligned[:, 1:] = gathered * cm_d[:, 1:].to(dtype=logits.dtype)
        return aligned

    def ours():
        return gen.score(ids, am, cm, group_size=group)

    _set_attention(model, "sdpa")
    torch.cuda.reset_peak_memory_stats(device)
    base_mem = torch.cuda.memory_allocated(device)
    want = reference()
    ref_runs = [_timed(device, reference) for _ in range(iters)]
    ref_peak = torch.cuda.max_memory_allocated(device) - base_mem
    _set_attention(model, "paged_b200")
    torch.cuda.reset_peak_memory_stats(device)
    got = ours()
    our_runs = [_timed(device, ours) for _ in range(iters)]
    our_peak = torch.cuda.max_memory_allocated(device) - base_mem
    diff = (got.float() - want.float())[cm_d].abs()
    ref_s = statistics.mean(t for _, t in ref_runs)
    our_s = statistics.mean(t for _, t in our_runs)
    return {
        "workload": f"old-policy log-probabilities of that rollout: {len(rows)} sequences (prompt + completion, "
                    f"up to {width} tokens), {scored} scored completion tokens, vocab 151936",
        "scored_tokens_per_s": scored / our_s,
        "ms": our_s * 1e3,
        "path": "PagedGenerator.score: group prompt prefilled once + copy-on-write forks, packed prefill "
                "kernel, LM head only on scored rows (<= 2048 at a time, fp32), fused log-softmax + gather kernel",
        "reference_scored_tokens_per_s": scored / ref_s,
        "reference_ms": ref_s * 1e3,
        "reference_path": "agentrl/core/rollout.py:456-472 as written: HF forward (SDPA) over the right-padded "
                          "batch, log_softmax over [B, L-1, vocab], gather, mask",
        "speedup_vs_reference": ref_s / our_s,
        "peak_extra_bytes": {"ours": int(our_peak), "reference": int(ref_peak)},
        "max_abs_logprob_diff": float(diff.max()),
        "mean_abs_logprob_diff": float(diff.mean()),
        "timing": f"CUDA events around whole passes, mean of {iters} after one warm-up each",
    }


def run_speculative(device: torch.device, seed: int, iters: int = 2) -> dict:
    """Speculative GRPO rollout at the speculative configuration: target Qwen2.5-1.5B architecture,
    draft Qwen2.5-0.5B architecture, k = 4, 64 sequences; random-init bf16 weights."""
    from randomrepo_b200.hf import PagedGenerator, SamplingConfig, make_store
    from randomrepo_b200.speculative import PagedSpeculativeGenerator

    ss = SPEC_SHAPE
    target = _qwen(device, QWEN_1P5B, seed)
    draft = _qwen(device, QWEN_0P5B, seed + 1)
    rng = np.random.default_rng(seed + 7)
    lens = rng.integers(ss["len_lo"], ss["len_hi"] + 1, size=ss["prompts"])
    prompts = [torch.from_numpy(rng.integers(0, QWEN_1P5B["vocab_size"], size=int(n))) for n in lens]
    group, new, k = ss["group"], ss["new_tokens"], ss["k"]
    cfg = SamplingConfig(do_sample=True, temperature=ss["temperature"], seed=0)

    # Stock HF assisted generation (speculative sampling, batch 1 only) on the same models.
    hf_note = None
    hf_tps = None
    try:
        def hf():
            with torch.inference_mode():
                n = 0
                for p in prompts[:2]:
                    x = p.unsqueeze(0).to(device)
                    out = target.generate(x, attention_mask=torch.ones_like(x), assistant_model=draft,
                                          max_new_tokens=new, do_sample=True, temperature=ss["temperature"],
                                          top_p=1.0, top_k=0, pad_token_id=0)
                    n += out.shape[1] - x.shape[1]
            return n
        hf()
        hf_runs = [_timed(device, hf) for _ in range(iters)]
        hf_tps = sum(n for n, _ in hf_runs) / sum(t for _, t in hf_runs)
    except Exception as e:  # noqa: BLE001 - recorded in the line
        hf_note = f"HF assisted generation unavailable: {type(e).__name__}: {str(e)[:160]}"

    t_store = make_store(target, total_blocks=16384)
    d_store = make_store(draft, total_blocks=16384)
    tgen = PagedGenerator(target, t_store, prefill_chunk_size=512, cuda_graphs=True)
    dgen = PagedGenerator(draft, d_store, prefill_chunk_size=512, cuda_graphs=True, sampler=tgen.sampler)
    spec = PagedSpeculativeGenerator(tgen, dgen, k=k)
    stats = {}

    def ours(it, seed):
        r = spec.generate(prompts, group_size=group, max_new_tokens=new, first_id=it * 10000,
                          sampling=SamplingConfig(do_sample=True, temperature=ss["temperature"], seed=seed))
        stats.update(rounds=r["rounds"], proposed=r["proposed"], accepted=r["accepted"])
        return sum(len(t) for t in r["tokens"])

    # Warm-up on the timed draws: sequences finish at different rounds, and
    # each batch size the shrinking batch reaches records its CUDA graphs once.
    for it in range(1, iters + 1):
        ours(100 + it, it)
    runs = [_timed(device, lambda it=it: ours(it, it)) for it in range(1, iters + 1)]
    spec_tps = sum(n for n, _ in runs) / sum(t for _, t in runs)
    for st in (t_store, d_store):
        if st.pool.decode_error_flag() or st.pool.prefill_error_flag():
            raise RuntimeError("speculative kernels reported a device error")
    # The same target without a draft, for context.
    pstore = make_store(target, total_blocks=16384)
    plain = PagedGenerator(target, pstore, prefill_chunk_size=512, cuda_graphs=True)

    def plain_run(it):
        r = plain.generate(prompts, group_size=group, max_new_tokens=new, first_id=it * 10000, sampling=cfg)
        return sum(len(t) for t in r["tokens"])

    plain_run(0)
    pruns = [_timed(device, lambda it=it: plain_run(it)) for it in range(1, iters + 1)]
    plain_tps = sum(n for n, _ in pruns) / sum(t for _, t in pruns)
    rate = stats["accepted"] / max(stats["proposed"], 1)
    del spec, tgen, dgen, plain, t_store, d_store, pstore, target, draft
    torch.cuda.empty_cache()
    out = {
        "workload": f"speculative GRPO rollout: target Qwen2.5-1.5B architecture, draft Qwen2.5-0.5B architecture "
                    f"(24 layers, 14q/2kv heads, head_dim 64), random-init bf16, k={k}, {ss['prompts']} prompts x "
                    f"group {group} = {ss['prompts'] * group} sequences, prompts U[{ss['len_lo']},{ss['len_hi']}], "
                    f"{new} new tokens, temperature {ss['temperature']}",
        "tokens_per_s": spec_tps,
        "path": "PagedSpeculativeGenerator: paged caches for both models (group prompts prefilled once + forks), "
                "CUDA-graph draft decode steps, CUDA-graph target verify forward through the paged verify read "
                "(prefill kernel, k+1 queries per sequence), device accept / reject (pkv_spec_accept), truncate "
                "of rejected drafts",
        "acceptance_rate": rate,
        "rounds": stats["rounds"],
        "acceptance_note": "random-init draft and target are unrelated models, so few drafts are accepted; the "
                           "round cost is the measured machinery, the acceptance rate is the weights'",
        "plain_paged_tokens_per_s": plain_tps,
        "plain_paged_path": "PagedGenerator on the same target and batch, CUDA-graph decode steps",
        "timing": f"CUDA events around whole rollouts, mean of {iters}, each after a warm-up rollout with the "
                  "same draws (a shrinking batch records each batch size's graphs once)",
    }
    if hf_tps is not None:
        out["hf_assisted_tokens_per_s"] = hf_tps
        out["hf_assisted_path"] = "stock HF generate(assistant_model=draft), batch 1 (its only mode), 2 prompts"
        out["speedup_vs_hf_assisted"] = spec_tps / hf_tps
    else:
        out["hf_assisted"] = hf_note
    return out


def run_vocab_rows(device: torch.device, seed: int, steps: int, warmup: int) -> dict:
    """The vocabulary-row kernels at Qwen2's vocabulary against the measured HBM bandwidth."""
    from randomrepo_b200.sampling import DeviceSampler

    g = torch.Generator(device=device).manual_seed(seed)
    vocab, rows = 151936, 4096
    logits = torch.randn(rows, vocab, device=device, generator=g) * 2.0  # 2.49 GB > L2
    tokens = torch.randint(0, vocab, (rows,), device=device, generator=g)
    s = DeviceSampler(device, seed=seed)
    peak, peak_kind = measured_peaks()

    def time_it(fn, n):
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(device)
            ts.append(e0.elapsed_time(e1))
        return statistics.mean(ts)

    n = max(3, min(steps, 20))
    lp_ms = time_it(lambda: s.token_logprobs(logits, tokens), n)
    torch_ms = time_it(lambda: torch.log_softmax(logits, -1).gather(-1, tokens.unsqueeze(-1)), n)
    lp_bytes = rows * vocab * 4 + rows * 12
    sm_ms = time_it(lambda: s.sample(logits[:512], temperature=1.0), n)
    sm_bytes = 512 * vocab * 4 + 512 * 20
    # Speculative accept at the speculative configuration: 64 sequences, k = 4.
    b, k = 64, 4
    tl = torch.randn(b, k + 1, vocab, device=device, generator=g) * 2.0
    dl = tl[:, :k] + 0.7 * torch.randn(b, k, vocab, device=device, generator=g)
    dtok = torch.argmax(dl, dim=-1)
    nd = torch.full((b,), k, dtype=torch.int32, device=device)
    flush = _L2Flush(device)

    ts = []
    for i in range(warmup + n):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _, _, n_out, n_acc = s.spec_accept(tl, dl, dtok, nd, do_sample=True)
        e1.record()
        torch.cuda.synchronize(device)
        if i >= warmup:
            ts.append(e0.elapsed_time(e1))
    acc_ms = statistics.mean(ts)
    rejects = int((n_acc < nd).sum())
    acc_bytes = (b * (k + 1) + b * k) * vocab * 4 + (rejects * 2 + (b - rejects)) * vocab * 4
    del logits, tl, dl, flush
    torch.cuda.empty_cache()

    def line(ms, nbytes):
        ach = nbytes / (ms * 1e-3) / 1e9
        return {"ms": ms, "bytes_per_launch": nbytes, "achieved": ach, "peak": peak, "unit": "GB/s",
                "frac": ach / peak, "peak_source": f"{peak_kind} hbm_gbs"}

    return {
        "token_logprobs": {
            "workload": f"fused log-softmax + gather, {rows} rows x vocab {vocab} fp32 (2.49 GB, > L2)",
            "roofline": line(lp_ms, lp_bytes),
            "torch_log_softmax_gather_ms": torch_ms,
            "speedup_vs_torch": torch_ms / lp_ms,
        },
        "sample_tokens": {
            "workload": f"Gumbel-max draw at temperature 1 + temperature-1 log-prob + argmax, 512 rows x {vocab}",
            "roofline": line(sm_ms, sm_bytes),
        },
        "spec_accept": {
            "workload": f"speculative accept / reject, {b} sequences, k={k}, vocab {vocab}, sampled corrections "
                        f"({rejects} rejections); L2 flushed before each launch",
            "roofline": line(acc_ms, acc_bytes),
            "bytes_rule": "target rows (k+1) + draft rows k per sequence once, then the drawn row (+ its draft "
                          "row on a rejection) again",
        },
        "timing": f"CUDA events per launch, mean of {n} after {warmup} warm-up launches",
        "gpu_launches_per_call": {"token_logprobs": 1, "sample_tokens": 1, "spec_accept": 3},
    }


def _reference_sample(lengths: np.ndarray, sample: int, cls):
    """A bounded sample of the workload for the reference's CPU path: ``sample`` of its sequences (same
    length draw), bf16 caches and inputs, and every host core for torch's intra-op threads."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    rng = np.random.default_rng(7)
    idx = np.sort(rng.choice(len(lengths), size=sample, replace=False))
    batch = cls(lengths[idx].tolist(), HQ, HKV, D, seed=3)
    g = torch.Generator().manual_seed(5)
    q = torch.randn((sample, HQ, D), generator=g).to(torch.bfloat16)
    kn = torch.randn((sample, HKV, D), generator=g).to(torch.bfloat16)
    vn = torch.randn((sample, HKV, D), generator=g).to(torch.bfloat16)
    return batch, list(range(sample)), q, kn, vn, cores


def _time_reference(batch, ids, q, kn, vn, seconds: float | None, steps: int | None = None) -> tuple[float, int]:
    """Mean seconds per step (step + rollback, so every step sees the workload's lengths)."""
    batch.step(ids, q, kn, vn)
    batch.rollback(ids)
    times = []
    t_end = time.perf_counter() + (seconds or 0.0)
    while (steps is None and time.perf_counter() < t_end) or (steps is not None and len(times) < steps):
        t = time.perf_counter()
        batch.step(ids, q, kn, vn)
        batch.rollback(ids)
        times.append(time.perf_counter() - t)
    return statistics.mean(times), len(times)


REFERENCE_PATH_I = ("the reference's resident-cache decode step in its own torch operations (bf16 caches): "
                    "torch.cat stack of equal-length buckets, torch.cat append (DynamicLayer.update), "
                    "scaled_dot_product_attention with GQA, per-sequence clone split, append_tokens "
                    "(oracle.decode_step.TorchResidentDecodeBatch)")
REFERENCE_PATH_II = ("the reference's block-store round trip in torch (bf16): read_sequence_legacy_cache (key "
                     "scan of the whole store + torch.cat of the blocks), torch.cat append, GQA SDPA, "
                     "append_tokens, write_sequence_cache (split + clone per block) "
                     "(oracle.decode_step.TorchBlockStoreDecodeBatch)")


def cpu_baseline(lengths: np.ndarray, seconds: float, sample: int = 32, steps: int | None = None) -> dict:
    """The reference's CPU decode paths (torch restatements, bf16) on bounded samples of the workload."""
    from oracle.decode_step import TorchBlockStoreDecodeBatch, TorchResidentDecodeBatch

    batch, ids, q, kn, vn, cores = _reference_sample(lengths, sample, TorchResidentDecodeBatch)
    per_step, n = _time_reference(batch, ids, q, kn, vn, seconds, steps)
    batch2, ids2, q2, kn2, vn2, _ = _reference_sample(lengths, sample, TorchBlockStoreDecodeBatch)
    per_step2, n2 = _time_reference(batch2, ids2, q2, kn2, vn2, max(1.0, seconds / 4), None if steps is None else 2)
    return {
        "value": sample / per_step,
        "unit": "tokens/s",
        "cores": cores,
        "kind": "port",
        "dtype": "bf16",
        "sample": f"{sample} of the {SEQS} sequences (ctx from the same U[64,2048] draw), {n} decode steps of "
                  + REFERENCE_PATH_I,
        "seconds_per_step": per_step,
        "block_store_path": {
            "value": sample / per_step2, "unit": "tokens/s", "seconds_per_step": per_step2,
            "sample": f"{sample} of the {SEQS} sequences, {n2} decode steps of " + REFERENCE_PATH_II,
        },
    }


def run_reference(args) -> dict:
    """The reference's CPU path (torch restatement of its resident-cache decode step, bf16) on the host cores:
    each step is a 32-sequence sample of the workload, so the run ends within a few minutes."""
    gen = torch.Generator().manual_seed(args.seed)
    lengths = torch.randint(64, 2049, (SEQS,), generator=gen).numpy().astype(np.int64)
    from oracle.decode_step import TorchResidentDecodeBatch

    sample = 32
    batch, ids, q, kn, vn, cores = _reference_sample(lengths, sample, TorchResidentDecodeBatch)
    for _ in range(args.warmup):
        batch.step(ids, q, kn, vn)
        batch.rollback(ids)
    t = time.perf_counter()
    for _ in range(args.steps):
        batch.step(ids, q, kn, vn)
        batch.rollback(ids)
    elapsed = time.perf_counter() - t
    value = sample * args.steps / elapsed
    return {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "impl": "reference",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed * 1000.0 / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded, ctx U[64,2048])",
        "config": workload_config(1),
        "cpu_baseline": {
            "value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"each step: {sample} of the {SEQS} sequences through " + REFERENCE_PATH_I,
        },
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tiles", action="store_true", help="skip the prefill / verify kernel lines (N=1 only)")
    ap.add_argument("--no-rollout", action="store_true", help="skip the end-to-end rollout line (N=1 only)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    sys.path.insert(0, str(ROOT))
    # stdout carries the one JSON line; anything else written to it (library
    # banners such as NCCL's version line, HF messages) goes to stderr.
    line_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), file=line_out, flush=True)
        return

    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    try:
        result = run_ours(args, rank, world, device)
        if result is not None:
            print(json.dumps(result), file=line_out, flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
