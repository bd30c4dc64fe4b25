"""Benchmark of the B200 head_dim-64 attention forward (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (one JSON line on rank 0): BASELINE config 3, the Qwen2.5-0.5B-shaped
causal prefill B=4, H=14, N=4096, d=64, fp16, sharded by (batch, head) over
the N GPUs (fixed total work: strong scaling). A "step" is one prefill of the
rank's share of the 56 heads. `value` is whole-job TFLOP/s (FLOPs 4*B*H*N^2*d,
halved for causal, as the reference's run_bench.py counts them).

Secondary measurements in the same line (`secondary`):
  c2_causal / c2_full  GPT-2-small prefill B=8 H=12 N=1024 (config 2)
  c4_decode            ragged decode B=64 H=12 cap 8192, lengths U[1,8192],
                       batch sharded over ranks balanced by length
  c5_decode            long decode B=1 H=14 S=131072; KV sequence-sharded over
                       ranks, per-rank log-sum-exp partials all-gathered with
                       NCCL and merged
  published_shapes     the reference's published sweep shapes (prefill B1/B8
                       H12 N4096, B4 H12 N2048, config 2; decode B1 H12
                       S128-4096, B8 H12 S2048) with cuDNN / flash_attn
                       kernels timed beside ours (library context only)
  per_rank             each rank's prefill / C4 / C5 times and work share,
                       so a scaling run shows its limiter at each N
`e2e.link` times the pinned host copies alone: link_frac = the longer of
upload and download / the e2e step.
Decode GB/s counts valid K+V rows only (128 B per row each for K and V).

`--impl reference` times the reference's CPU path (src/attention_cpu.py,
restated in oracle/oracle.py) on the host cores, one step = 4 of config 3's
56 (batch, head) evaluations, and prints the same workload config as this
arm; under torchrun only rank 0 runs it.
"""

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "flash-attention-cuda_b200")
ORACLE_DIR = os.path.join(REPO, "oracle")
PROFILES = os.path.join(REPO, "profiles")

HEAD_DIM = 64
SCALE = 1.0 / math.sqrt(HEAD_DIM)
C3 = dict(B=4, H=14, N=4096, causal=True)
C2 = dict(B=8, H=12, N=1024)
C4 = dict(B=64, H=12, cap=8192)
C5 = dict(B=1, H=14, S=131072)
L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0,
                  "bf16_tflops_sustained": 1400.0}


def prefill_flops(b, h, n, causal):
    f = 4.0 * b * h * n * n * HEAD_DIM
    return f * 0.5 if causal else f


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def read_profile_traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary line
    `traffic_bytes_per_launch: <int>` in profiles/<name>.md (None if absent)."""
    path = os.path.join(PROFILES, name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except Exception:
        pass
    return None


def read_profile_clock(name):
    """SM clock (GHz) inside the kernel's ncu capture, from a committed
    summary line `sm_clock_ghz_in_kernel: <float>` (None if absent): the
    clock the power-capped kernel actually ran at, which the NVML samples
    between launches do not show."""
    path = os.path.join(PROFILES, name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("sm_clock_ghz_in_kernel:"):
                return float(line.split(":", 1)[1].strip())
    except Exception:
        pass
    return None


def shard_range(total, world, rank):
    sys.path.insert(0, PKG_DIR)
    from flashattn_cuda.dist import shard_units
    return shard_units(total, world, rank)


def lpt_partition(weights, world):
    sys.path.insert(0, PKG_DIR)
    from flashattn_cuda.dist import lpt_partition as lpt
    return lpt(weights, world)


# ---------------------------------------------------------------------------
# Clock sampling (NVML) during the timed regions
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting",
        0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x10: "sync_boost",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index, interval=0.005):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._interval = interval
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                util = n.nvmlDeviceGetUtilizationRates(self._h).gpu
                mhz = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
                r = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, util, r))
            except Exception:
                pass
            time.sleep(self._interval)

    def __enter__(self):
        if self._nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        busy = [s for s in self.samples if s[1] > 0] or self.samples
        reasons = set()
        for _, _, r in busy:
            for bit, name in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(s[0] for s in busy) if busy else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(reasons),
            "samples": len(busy),
        }


# ---------------------------------------------------------------------------
# Timing helpers (CUDA events on the launching stream)
# ---------------------------------------------------------------------------
class Timer:
    def __init__(self, torch, dist, world):
        self.torch = torch
        self.dist = dist
        self.world = world
        self.flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8,
                                     device="cuda")

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, x):
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def run(self, fn, steps, warmup, flush=True):
        """Total device time of `steps` calls of fn (ms), L2 flushed before
        each call (outside the event pair), max over ranks."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        evs = []
        for _ in range(steps):
            if flush:
                # write a buffer larger than L2, then read it back: the read
                # forces the write-back of the dirty lines before the timed
                # kernel starts, so it neither finds its inputs in L2 nor
                # pays for the flush's DRAM writes
                self.flush_buf.zero_()
                self._sink = self.flush_buf.view(torch.int64).sum()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            evs.append((s, e))
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        total = sum(s.elapsed_time(e) for s, e in evs)
        self.last_all = self.all_ranks(total)
        return max(self.last_all)

    def all_ranks(self, x):
        """x from every rank, in rank order."""
        if self.world == 1:
            return [x]
        t = self.torch.tensor([x], dtype=self.torch.float64, device="cuda")
        out = [self.torch.zeros_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [float(o.item()) for o in out]


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, PKG_DIR)
    import flashattn_cuda as fa

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    peaks, peaks_src = load_peaks()
    timer = Timer(torch, dist, world)
    gen = torch.Generator(device="cuda")
    launches = 0

    def randn(*shape, seed):
        gen.manual_seed(seed)
        return torch.randn(*shape, generator=gen, device="cuda",
                           dtype=torch.float16)

    sampler = ClockSampler(local_rank)
    with sampler:
        # ---------------- headline: C3 causal prefill, heads sharded -------
        bh = C3["B"] * C3["H"]
        u0, u1 = shard_range(bh, world, rank)
        units = u1 - u0
        n = C3["N"]
        q = randn(1, units, n, HEAD_DIM, seed=1000 + rank)
        k = randn(1, units, n, HEAD_DIM, seed=2000 + rank)
        v = randn(1, units, n, HEAD_DIM, seed=3000 + rank)
        step = lambda: fa.prefill(q, k, v, True, SCALE)
        total_ms = timer.run(step, args.steps, args.warmup)
        launches += args.steps
        ms = total_ms / args.steps
        sms = torch.cuda.get_device_properties(local_rank).multi_processor_count
        per_rank = {
            "prefill_ms": [round(x / args.steps, 5) for x in timer.last_all],
            "prefill_heads": [shard_range(bh, world, r)[1] - shard_range(bh, world, r)[0]
                              for r in range(world)],
            "prefill_form_rank0": fa._C._prefill_form(units, n, True, sms),
            "sms": sms}
        flops_total = prefill_flops(C3["B"], C3["H"], n, True)
        value = flops_total / (ms * 1e-3) / 1e12
        flops_rank = prefill_flops(1, units, n, True)
        achieved = flops_rank / (ms * 1e-3) / 1e12  # this rank's kernel
        peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])

        # ---------------- e2e through the public API, host buffers -------
        hq = q.cpu().pin_memory()
        hk = k.cpu().pin_memory()
        hv = v.cpu().pin_memory()
        hout = torch.empty_like(hq).pin_memory()

        # The public host-memory entry (fa_prefill_host): chunks of heads
        # are uploaded, computed and downloaded on overlapping streams.
        def e2e_step():
            fa.prefill_host(hq, hk, hv, True, SCALE, out=hout,
                            non_blocking=True)

        e2e_ms = timer.run(e2e_step, args.steps, args.warmup) / args.steps
        launches += args.steps * fa._C._prefill_host_launches(
            1, units, units, n, HEAD_DIM)

        # The same round trip done serially (copy in, prefill, copy out),
        # for comparison.
        def e2e_serial_step():
            dq = hq.to("cuda", non_blocking=True)
            dk = hk.to("cuda", non_blocking=True)
            dv = hv.to("cuda", non_blocking=True)
            o = fa.prefill(dq, dk, dv, True, SCALE)
            hout.copy_(o, non_blocking=True)

        e2e_serial_ms = timer.run(e2e_serial_step, args.steps,
                                  args.warmup) / args.steps
        launches += args.steps
        h2d = 3 * hq.numel() * 2 * world
        d2h = hq.numel() * 2 * world
        # the link itself: one pinned upload of the step's inputs and one
        # download of its output, each alone, device-timed
        dbuf = torch.empty(3 * hq.numel(), dtype=torch.float16, device="cuda")
        hbuf = torch.empty_like(dbuf, device="cpu").pin_memory()
        up_ms = timer.run(lambda: dbuf.copy_(hbuf, non_blocking=True),
                          args.steps, args.warmup, flush=False) / args.steps
        down_ms = timer.run(
            lambda: hout.view(-1).copy_(dbuf[:hq.numel()], non_blocking=True),
            args.steps, args.warmup, flush=False) / args.steps
        del dbuf, hbuf
        # uploads and downloads overlap in fa_prefill_host (PCIe is full
        # duplex), so the link bound of a step is the longer of the two
        link_ms = max(up_ms, down_ms)
        del q, k, v

        # ---------------- secondary: C2 prefill (replicated per rank) -----
        secondary = {}
        for causal in (True, False):
            q2 = randn(C2["B"], C2["H"], C2["N"], HEAD_DIM, seed=11 + rank)
            k2 = randn(C2["B"], C2["H"], C2["N"], HEAD_DIM, seed=12 + rank)
            v2 = randn(C2["B"], C2["H"], C2["N"], HEAD_DIM, seed=13 + rank)
            t = timer.run(lambda: fa.prefill(q2, k2, v2, causal, SCALE),
                          args.steps, args.warmup) / args.steps
            launches += args.steps
            f = prefill_flops(C2["B"], C2["H"], C2["N"], causal)
            secondary["c2_causal" if causal else "c2_full"] = {
                "ms": round(t, 5), "tflops_per_gpu": round(f / (t * 1e-3) / 1e12, 2),
                "frac_of_measured_bf16_peak": round(f / (t * 1e-3) / 1e12 / peak, 4),
                "scaling": "replicated per GPU"}
            del q2, k2, v2

        # ---------------- secondary: C4 ragged decode ---------------------
        g = torch.Generator().manual_seed(0)
        all_lens = torch.randint(1, C4["cap"] + 1, (C4["B"],), generator=g,
                                 dtype=torch.int32)
        mine = lpt_partition(all_lens.tolist(), world)[rank]
        lens = all_lens[mine].cuda()
        bm = len(mine)
        qd = randn(bm, C4["H"], 1, HEAD_DIM, seed=40 + rank)
        kc = randn(bm, C4["H"], C4["cap"], HEAD_DIM, seed=41 + rank)
        vc = randn(bm, C4["H"], C4["cap"], HEAD_DIM, seed=42 + rank)
        t = timer.run(lambda: fa.decode(qd, kc, vc, lens, SCALE), args.steps,
                      args.warmup) / args.steps
        launches += args.steps
        bytes_all = int(all_lens.sum()) * C4["H"] * HEAD_DIM * 2 * 2
        bytes_rank = int(lens.sum()) * C4["H"] * HEAD_DIM * 2 * 2
        hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        parts = lpt_partition(all_lens.tolist(), world)
        per_rank["c4_ms"] = [round(x / args.steps, 5) for x in timer.last_all]
        per_rank["c4_rows"] = [int(sum(all_lens[i] for i in pr)) for pr in parts]
        secondary["c4_decode"] = {
            "ms": round(t, 5), "gbs_total": round(bytes_all / (t * 1e-3) / 1e9, 1),
            "gbs_per_gpu_rank0": round(bytes_rank / (t * 1e-3) / 1e9, 1),
            "frac_of_measured_hbm": round(bytes_rank / (t * 1e-3) / 1e9 / hbm, 4),
            "tokens_per_s": round(C4["B"] / (t * 1e-3), 1),
            "traffic_bytes_per_launch_ncu": read_profile_traffic("decode_kernel_c4"),
            "scaling": "strong (batch sharded, LPT by length)"}

        # the same step with the new token's K/V row appended in the launch,
        # against the unfused sequence (cache row write, then decode)
        lens_a = (lens - 1).contiguous()
        kn = randn(bm, C4["H"], 1, HEAD_DIM, seed=43 + rank)
        vn = randn(bm, C4["H"], 1, HEAD_DIM, seed=44 + rank)
        rows = torch.arange(bm, device="cuda")
        pos = lens_a.long()
        t_fused = timer.run(
            lambda: fa.decode_append(qd, kn, vn, kc, vc, lens_a, SCALE),
            args.steps, args.warmup) / args.steps
        launches += args.steps

        def unfused():
            kc[rows, :, pos] = kn[:, :, 0]
            vc[rows, :, pos] = vn[:, :, 0]
            return fa.decode(qd, kc, vc, lens, SCALE)

        t_unfused = timer.run(unfused, args.steps, args.warmup) / args.steps
        launches += args.steps
        secondary["c4_decode_append"] = {
            "ms": round(t_fused, 5),
            "gbs_per_gpu_rank0": round(bytes_rank / (t_fused * 1e-3) / 1e9, 1),
            "unfused_ms": round(t_unfused, 5),
            "note": "decode_append (row store + attention in one launch) vs "
                    "two index_put copies + decode"}
        del qd, kc, vc, kn, vn

        # config 4 at head_dim 128 (rank-local batch shard, same lengths)
        qd = randn(bm, C4["H"], 1, 128, seed=45 + rank)
        kc = randn(bm, C4["H"], C4["cap"], 128, seed=46 + rank)
        vc = randn(bm, C4["H"], C4["cap"], 128, seed=47 + rank)
        t = timer.run(lambda: fa.decode(qd, kc, vc, lens, SCALE), args.steps,
                      args.warmup) / args.steps
        launches += args.steps
        b128 = bytes_rank * 2
        secondary["c4_decode_d128"] = {
            "ms": round(t, 5), "gbs_per_gpu_rank0": round(b128 / (t * 1e-3) / 1e9, 1),
            "frac_of_measured_hbm": round(b128 / (t * 1e-3) / 1e9 / hbm, 4),
            "note": "config 4 at head_dim 128 (the reference's named next size)"}
        del qd, kc, vc

        # ---------------- secondary: C5 long decode, sequence-sharded ----
        S = C5["S"]
        c0, c1 = shard_range(S, world, rank)
        qd = randn(1, C5["H"], 1, HEAD_DIM, seed=50)  # same q on every rank
        kc = randn(1, C5["H"], c1 - c0, HEAD_DIM, seed=51 + rank)
        vc = randn(1, C5["H"], c1 - c0, HEAD_DIM, seed=52 + rank)
        lens_local = torch.tensor([c1 - c0], dtype=torch.int32, device="cuda")

        from flashattn_cuda.dist import (PeerExchange, sharded_decode,
                                         sharded_decode_fused)

        b_total = S * C5["H"] * HEAD_DIM * 2 * 2
        b_rank = (c1 - c0) * C5["H"] * HEAD_DIM * 2 * 2
        if world == 1:
            t = timer.run(lambda: sharded_decode(qd, kc, vc, lens_local, SCALE),
                          args.steps, args.warmup) / args.steps
            launches += args.steps
            c5_all = timer.last_all
            scaling = "single GPU"
        else:
            # the combine inside the decode kernel: partials stored into
            # every rank's exchange buffer over NVLink, merged in place
            xchg = PeerExchange(1, C5["H"])
            t = timer.run(
                lambda: sharded_decode_fused(qd, kc, vc, lens_local, SCALE, xchg),
                args.steps, args.warmup) / args.steps
            launches += args.steps
            c5_all = timer.last_all
            xchg.close()
            scaling = ("strong (KV sequence sharded, partials exchanged over "
                       "NVLink peer memory inside the decode kernel)")
            t_nccl = timer.run(
                lambda: sharded_decode(qd, kc, vc, lens_local, SCALE),
                args.steps, args.warmup) / args.steps
            launches += args.steps * 2
            secondary["c5_decode_nccl"] = {
                "ms": round(t_nccl, 5),
                "gbs_total": round(b_total / (t_nccl * 1e-3) / 1e9, 1),
                "note": "decode_partial + NCCL all-gather + merge kernel"}
        per_rank["c5_ms"] = [round(x / args.steps, 5) for x in c5_all]
        per_rank["c5_rows"] = [shard_range(S, world, r)[1] - shard_range(S, world, r)[0]
                               for r in range(world)]
        secondary["per_rank"] = per_rank
        secondary["c5_decode"] = {
            "ms": round(t, 5), "gbs_total": round(b_total / (t * 1e-3) / 1e9, 1),
            "frac_of_measured_hbm_per_gpu": round(
                b_rank / (t * 1e-3) / 1e9 / hbm, 4),
            "scaling": scaling}
        del qd, kc, vc

        # ------- one GPU's share of config 3 at 2 / 4 / 8 GPUs, timed alone:
        # the per-rank kernel time a strong-scaling run is bounded by, with
        # the CTA form each share runs in
        if world == 1:
            shares = {}
            for w in (2, 4, 8):
                hs = C3["B"] * C3["H"] // w
                qs = randn(1, hs, C3["N"], HEAD_DIM, seed=95)
                ks = randn(1, hs, C3["N"], HEAD_DIM, seed=96)
                vs = randn(1, hs, C3["N"], HEAD_DIM, seed=97)
                t = timer.run(lambda: fa.prefill(qs, ks, vs, True, SCALE),
                              args.steps, args.warmup) / args.steps
                launches += args.steps
                fl = prefill_flops(1, hs, C3["N"], True)
                shares[f"gpus{w}_b1_h{hs}"] = {
                    "ms": round(t, 5),
                    "tflops": round(fl / (t * 1e-3) / 1e12, 1),
                    "form": fa._C._prefill_form(hs, C3["N"], True, sms)["form"]}
                del qs, ks, vs
            shares["note"] = ("causal N=4096 prefill of config 3's per-GPU head "
                              "share on one GPU; the scaling run's per-rank time")
            secondary["c3_prefill_per_gpu_share"] = shares

        # ------- grouped-query variants (Qwen2.5-0.5B really has 2 K/V heads):
        # same outputs as the pre-expanded configs without repeating K/V
        if world == 1:
            qg = randn(C3["B"], C3["H"], C3["N"], HEAD_DIM, seed=90)
            kg = randn(C3["B"], 2, C3["N"], HEAD_DIM, seed=91)
            vg = randn(C3["B"], 2, C3["N"], HEAD_DIM, seed=92)
            t = timer.run(lambda: fa.prefill(qg, kg, vg, True, SCALE), args.steps,
                          args.warmup) / args.steps
            launches += args.steps
            qh = randn(C3["B"], C3["H"], C3["N"], 128, seed=96)
            kh = randn(C3["B"], C3["H"], C3["N"], 128, seed=97)
            vh = randn(C3["B"], C3["H"], C3["N"], 128, seed=98)
            t128 = timer.run(lambda: fa.prefill(qh, kh, vh, True, 128 ** -0.5),
                             args.steps, args.warmup) / args.steps
            launches += args.steps
            f128 = prefill_flops(C3["B"], C3["H"], C3["N"], True) * 2
            secondary["c3_prefill_d128"] = {
                "ms": round(t128, 5),
                "tflops": round(f128 / (t128 * 1e-3) / 1e12, 2),
                "frac_of_measured_bf16_peak": round(
                    f128 / (t128 * 1e-3) / 1e12 / peak, 4),
                "note": "config 3 shape at head_dim 128 (the reference's named "
                        "next size), causal"}
            del qh, kh, vh
            # bf16 (the reference's other named next variant): config 3
            # prefill and the config-5 decode with bf16 tensors
            qb, kb, vb = (randn(C3["B"], C3["H"], C3["N"], HEAD_DIM,
                                seed=110 + i).to(torch.bfloat16)
                          for i in range(3))
            tb = timer.run(lambda: fa.prefill(qb, kb, vb, True, SCALE),
                           args.steps, args.warmup) / args.steps
            launches += args.steps
            fb = prefill_flops(C3["B"], C3["H"], C3["N"], True)
            secondary["c3_prefill_bf16"] = {
                "ms": round(tb, 5),
                "tflops": round(fb / (tb * 1e-3) / 1e12, 2),
                "frac_of_measured_bf16_peak": round(
                    fb / (tb * 1e-3) / 1e12 / peak, 4)}
            del qb, kb, vb
            qdb = randn(1, C5["H"], 1, HEAD_DIM, seed=113).to(torch.bfloat16)
            kcb = randn(1, C5["H"], C5["S"], HEAD_DIM, seed=114).to(torch.bfloat16)
            vcb = randn(1, C5["H"], C5["S"], HEAD_DIM, seed=115).to(torch.bfloat16)
            lensb = torch.tensor([C5["S"]], dtype=torch.int32, device="cuda")
            tdb = timer.run(lambda: fa.decode(qdb, kcb, vcb, lensb, SCALE),
                            args.steps, args.warmup) / args.steps
            launches += args.steps
            bb = C5["S"] * C5["H"] * HEAD_DIM * 2 * 2
            secondary["c5_decode_bf16"] = {
                "ms": round(tdb, 5),
                "gbs": round(bb / (tdb * 1e-3) / 1e9, 1),
                "frac_of_measured_hbm": round(bb / (tdb * 1e-3) / 1e9 / hbm, 4)}
            del qdb, kcb, vcb
            # many short prompts (N = 128: two heads per CTA)
            qs, ks, vs = (randn(64, 32, 128, HEAD_DIM, seed=130 + i)
                          for i in range(3))
            tsh = timer.run(lambda: fa.prefill(qs, ks, vs, True, SCALE),
                            args.steps, args.warmup) / args.steps
            launches += args.steps
            secondary["prefill_short_b64_h32_n128"] = {
                "ms": round(tsh, 5),
                "tflops": round(prefill_flops(64, 32, 128, True)
                                / (tsh * 1e-3) / 1e12, 2),
                "note": "causal prefill of 2048 heads of 128 tokens"}
            del qs, ks, vs
            secondary["c3_prefill_gqa_kv2"] = {
                "ms": round(t, 5),
                "tflops": round(prefill_flops(C3["B"], C3["H"], C3["N"], True)
                                / (t * 1e-3) / 1e12, 2)}
            del qg, kg, vg
            qd = randn(1, C5["H"], 1, HEAD_DIM, seed=93)
            kc = randn(1, 2, C5["S"], HEAD_DIM, seed=94)
            vc = randn(1, 2, C5["S"], HEAD_DIM, seed=95)
            lens1 = torch.tensor([C5["S"]], dtype=torch.int32, device="cuda")
            t = timer.run(lambda: fa.decode(qd, kc, vc, lens1, SCALE), args.steps,
                          args.warmup) / args.steps
            launches += args.steps
            kv_bytes = C5["S"] * 2 * HEAD_DIM * 2 * 2
            # grouped decode at head_dim 128 (32 query heads on 8 K/V heads)
            qd8 = randn(8, 32, 1, 128, seed=99)
            kc8 = randn(8, 8, 32768, 128, seed=100)
            vc8 = randn(8, 8, 32768, 128, seed=101)
            lens8 = torch.full((8,), 32768, dtype=torch.int32, device="cuda")
            t8 = timer.run(lambda: fa.decode(qd8, kc8, vc8, lens8, 128 ** -0.5),
                           args.steps, args.warmup) / args.steps
            launches += args.steps
            b8 = 8 * 8 * 32768 * 128 * 2 * 2
            secondary["decode_gqa_d128_b8_h32_kv8"] = {
                "ms": round(t8, 5), "kv_gbs": round(b8 / (t8 * 1e-3) / 1e9, 1),
                "frac_of_measured_hbm": round(b8 / (t8 * 1e-3) / 1e9 / hbm, 4),
                "note": "B=8, 32 query heads on 8 K/V heads, S=32768, head_dim 128"}
            del qd8, kc8, vc8
            secondary["c5_decode_gqa_kv2"] = {
                "ms": round(t, 5),
                "kv_gbs": round(kv_bytes / (t * 1e-3) / 1e9, 1),
                "frac_of_measured_hbm": round(
                    kv_bytes / (t * 1e-3) / 1e9 / hbm, 4),
                "note": "14 query heads over 2 K/V heads, every K/V row read "
                        "once for its 7 query heads; L2 flushed between steps"}
            del qd, kc, vc

        # ------- host cost of a small decode step: eager vs CUDA graph ------
        if world == 1:
            secondary["decode_step_graph"] = graph_step_measure(fa, randn)

        # ------- NVIDIA's library attention on the headline shape (context) --
        # cuDNN's fused attention through torch SDPA: a library kernel, timed
        # beside ours for reference only; nothing of it is on our path.
        if world == 1 and not args.no_library:
            secondary["cudnn_sdpa_c3"] = cudnn_measure(
                timer, randn, args.steps, args.warmup, value)
            d128 = secondary.get("c3_prefill_d128", {}).get("tflops")
            if d128:
                secondary["cudnn_sdpa_c3_d128"] = cudnn_measure(
                    timer, randn, args.steps, args.warmup, d128, d=128)

        # ------- the reference's published sweep shapes, libraries beside ---
        if world == 1 and not args.no_library:
            secondary["published_shapes"] = published_shapes(
                fa, timer, randn, min(args.steps, 10), args.warmup)
            launches += (len(PUB_PREFILL) + 2 + len(PUB_DECODE)) * min(args.steps, 10)

        # ------- the reference's own CUDA kernels on this B200 (baseline) ----
        if world == 1 and not args.no_ref_cuda:
            secondary["reference_cuda_kernels"] = ref_cuda_measure(
                timer, randn, args.steps, args.warmup)

    assert fa.take_device_error() == 0, "device-side error during the bench"
    clocks = sampler.summary()

    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    result = {
        "metric": "causal prefill TFLOP/s (B=4,H=14,N=4096,d=64 fp16)",
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp16 in, fp32 accumulate",
        "data": "synthetic N(0,1) fp16, seeded",
        "config": workload_config(world),
        "e2e": {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 3),
                "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "flashattn_cuda.prefill_host (C ABI fa_prefill_host): "
                       "pinned host q/k/v/out, per-chunk uploads, kernels and "
                       "downloads overlapped",
                "serial_ms_per_step": round(e2e_serial_ms, 4),
                "link": {"h2d_ms": round(up_ms, 4), "d2h_ms": round(down_ms, 4),
                         "h2d_gbs": round(3 * hq.numel() * 2 / (up_ms * 1e-3) / 1e9, 1),
                         "d2h_gbs": round(hq.numel() * 2 / (down_ms * 1e-3) / 1e9, 1),
                         "bound_ms": round(link_ms, 4),
                         "link_frac": round(link_ms / e2e_ms, 4),
                         "note": "pinned copies timed alone on this box; "
                                 "link_frac = bound_ms / ms_per_step"},
                "serial_value": round(flops_total / (e2e_serial_ms * 1e-3) / 1e12, 3)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2),
                     "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4),
                     "peak_source": f"{peaks_src} bf16 cuBLAS burst",
                     "frac_of_nominal_2250": round(achieved / 2250.0, 4),
                     "traffic": read_profile_traffic("prefill_kernel_c3"),
                     "sm_clock_ghz_in_kernel_ncu": read_profile_clock(
                         "prefill_kernel_c3")},
        "gpu_launches": launches,
        "clocks": clocks,
        "secondary": secondary,
    }
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_budget)
    print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def ref_cuda_measure(timer, randn, steps, warmup):
    """Times the reference's own CUDA kernels (built for sm_100 from its
    sources into oracle/_ref by oracle/build_ref.py) on the same configs."""
    import torch

    sys.path.insert(0, ORACLE_DIR)
    try:
        import build_ref
        ref = build_ref.load()
    except Exception as ex:  # not built on this machine
        return {"unavailable": f"oracle/_ref not built: {type(ex).__name__}"}
    out = {}
    n = C3["N"]
    q, k, v = (randn(C3["B"], C3["H"], n, HEAD_DIM, seed=70 + i) for i in range(3))
    t = timer.run(lambda: ref.prefill(q, k, v, True, SCALE), steps, warmup) / steps
    out["c3_prefill"] = {"ms": round(t, 4), "tflops": round(
        prefill_flops(C3["B"], C3["H"], n, True) / (t * 1e-3) / 1e12, 2)}
    del q, k, v
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1, C4["cap"] + 1, (C4["B"],), generator=g,
                         dtype=torch.int32).cuda()
    qd = randn(C4["B"], C4["H"], 1, HEAD_DIM, seed=73)
    kc = randn(C4["B"], C4["H"], C4["cap"], HEAD_DIM, seed=74)
    vc = randn(C4["B"], C4["H"], C4["cap"], HEAD_DIM, seed=75)
    t = timer.run(lambda: ref.decode(qd, kc, vc, lens, SCALE), steps, warmup) / steps
    b = int(lens.sum()) * C4["H"] * HEAD_DIM * 2 * 2
    out["c4_decode"] = {"ms": round(t, 4), "gbs": round(b / (t * 1e-3) / 1e9, 1)}
    del qd, kc, vc
    S = C5["S"]
    qd = randn(1, C5["H"], 1, HEAD_DIM, seed=76)
    kc = randn(1, C5["H"], S, HEAD_DIM, seed=77)
    vc = randn(1, C5["H"], S, HEAD_DIM, seed=78)
    lens = torch.tensor([S], dtype=torch.int32, device="cuda")
    t = timer.run(lambda: ref.decode(qd, kc, vc, lens, SCALE), steps, warmup) / steps
    b = S * C5["H"] * HEAD_DIM * 2 * 2
    out["c5_decode"] = {"ms": round(t, 4), "gbs": round(b / (t * 1e-3) / 1e9, 1)}
    out["note"] = ("reference csrc/prefill.cu + csrc/decode.cu compiled for "
                   "sm_100 from its own sources, same inputs and timing")
    return out


# ---------------------------------------------------------------------------
# CPU path of the reference (numpy restatement in oracle/)
# ---------------------------------------------------------------------------
def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info()
             if i.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_sample_heads(budget_s, heads=None):
    """Runs causal attention_cpu over C3 heads until `budget_s` elapses (or
    exactly `heads` of them); returns (heads done, seconds)."""
    sys.path.insert(0, ORACLE_DIR)
    import oracle

    rng = np.random.default_rng(0)
    n = C3["N"]
    done, t_total = 0, 0.0
    while (done < heads) if heads else (t_total < budget_s or done == 0):
        q, k, v = (rng.standard_normal((n, HEAD_DIM), dtype=np.float32)
                   .astype(np.float16).astype(np.float32) for _ in range(3))
        t0 = time.perf_counter()
        oracle.attention_cpu(q, k, v, SCALE, causal=True)
        t_total += time.perf_counter() - t0
        done += 1
    return done, t_total


def cpu_baseline(budget_s):
    heads, secs = cpu_sample_heads(budget_s)
    flops = prefill_flops(1, heads, C3["N"], True)
    return {"value": round(flops / secs / 1e12, 5), "unit": "TFLOP/s",
            "cores": cpu_threads(), "kind": "port",
            "sample": f"{heads} causal N=4096 (batch, head) evaluations, cycling "
                      f"over config 3's 56 heads, through the numpy restatement "
                      f"of src/attention_cpu.py ({secs:.1f} s)"}


def graph_step_measure(fa, randn, calls=200):
    """Wall time per call of 200 back-to-back tiny decode steps (B=1, H=2,
    256 cached rows: a few us of device work, so the host's per-call cost
    shows), launched eagerly through the Python API and as replays of a
    captured CUDA graph."""
    import time
    import torch
    q = randn(1, 2, 1, HEAD_DIM, seed=120)
    k = randn(1, 2, 256, HEAD_DIM, seed=121)
    v = randn(1, 2, 256, HEAD_DIM, seed=122)
    lens = torch.tensor([256], dtype=torch.int32, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fa.decode(q, k, v, lens, SCALE)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            fa.decode(q, k, v, lens, SCALE)
    torch.cuda.current_stream().wait_stream(side)

    def per_call(fn):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(calls):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / calls * 1e6

    eager = per_call(lambda: fa.decode(q, k, v, lens, SCALE))
    replay = per_call(graph.replay)
    return {"eager_us_per_call": round(eager, 2),
            "graph_us_per_call": round(replay, 2),
            "note": "wall clock per call, 200 calls back to back, B=1 H=2 "
                    "S=256 decode; the graph replays one captured launch"}


# The reference's published sweep shapes (docs/benchmarks.md:28,72,113-117;
# docs/profiles/analysis.md:76,113-114; swept by bench/run_bench.py:122-210),
# measured here on the B200 with a library kernel beside each: cuDNN fused
# attention (torch SDPA) for prefill, flash_attn_with_kvcache for decode.
PUB_PREFILL = [(1, 12, 4096), (8, 12, 4096), (4, 12, 2048)]
PUB_DECODE = [(1, 12, s) for s in (128, 256, 512, 1024, 2048, 4096)] + [(8, 12, 2048)]


def published_shapes(fa, timer, randn, steps, warmup):
    import torch
    out = {}
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
    except Exception:  # pragma: no cover
        sdpa_kernel = None
    try:
        from flash_attn import flash_attn_with_kvcache
    except Exception as exc:
        flash_attn_with_kvcache = None
        out["flash_attn_unavailable"] = f"{type(exc).__name__}: {str(exc)[:80]}"

    def lib_prefill(q, k, v, causal):
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            torch.nn.functional.scaled_dot_product_attention(
                q, k, v, is_causal=causal, scale=SCALE)

    shapes = [(b, h, n, True) for b, h, n in PUB_PREFILL]
    shapes += [(C2["B"], C2["H"], C2["N"], True), (C2["B"], C2["H"], C2["N"], False)]
    for b, h, n, causal in shapes:
        q, k, v = (randn(b, h, n, HEAD_DIM, seed=200 + i) for i in range(3))
        f = prefill_flops(b, h, n, causal)
        t = timer.run(lambda: fa.prefill(q, k, v, causal, SCALE), steps, warmup) / steps
        row = {"us": round(t * 1e3, 2), "tflops": round(f / (t * 1e-3) / 1e12, 1)}
        if sdpa_kernel is not None:
            try:
                tl = timer.run(lambda: lib_prefill(q, k, v, causal), steps, warmup) / steps
                row["cudnn_us"] = round(tl * 1e3, 2)
                row["cudnn_tflops"] = round(f / (tl * 1e-3) / 1e12, 1)
                row["ours_over_cudnn"] = round(tl / t, 3)
            except Exception as exc:
                row["cudnn_unavailable"] = f"{type(exc).__name__}"
        out[f"prefill_b{b}_h{h}_n{n}_{'causal' if causal else 'full'}"] = row
        del q, k, v
    for b, h, s_len in PUB_DECODE:
        q = randn(b, h, 1, HEAD_DIM, seed=210)
        k = randn(b, h, s_len, HEAD_DIM, seed=211)
        v = randn(b, h, s_len, HEAD_DIM, seed=212)
        lens = torch.full((b,), s_len, dtype=torch.int32, device="cuda")
        nbytes = b * h * s_len * HEAD_DIM * 2 * 2
        t = timer.run(lambda: fa.decode(q, k, v, lens, SCALE), steps, warmup) / steps
        row = {"us": round(t * 1e3, 2), "gbs": round(nbytes / (t * 1e-3) / 1e9, 1)}
        if flash_attn_with_kvcache is not None:
            # flash_attn's layout is (batch, seq, heads, dim): converted once,
            # outside the timed region
            qf = q.transpose(1, 2).contiguous()
            kf = k.transpose(1, 2).contiguous()
            vf = v.transpose(1, 2).contiguous()
            try:
                tl = timer.run(lambda: flash_attn_with_kvcache(
                    qf, kf, vf, cache_seqlens=lens, softmax_scale=SCALE),
                    steps, warmup) / steps
                row["flash_attn_us"] = round(tl * 1e3, 2)
                row["ours_over_flash_attn"] = round(tl / t, 3)
            except Exception as exc:
                row["flash_attn_unavailable"] = f"{type(exc).__name__}: {str(exc)[:60]}"
            del qf, kf, vf
        out[f"decode_b{b}_h{h}_s{s_len}"] = row
        del q, k, v
    out["note"] = ("published sweep shapes of the reference, fp16, L2 flushed "
                   "before every step; library kernels are context only")
    return out


def cudnn_measure(timer, randn, steps, warmup, ours_tflops, d=HEAD_DIM):
    """Config 3 (at head_dim d) through torch SDPA restricted to the cuDNN
    backend, with the same inputs shape, L2 flush and timing as ours."""
    import torch
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        q = randn(C3["B"], C3["H"], C3["N"], d, seed=1000)
        k = randn(C3["B"], C3["H"], C3["N"], d, seed=2000)
        v = randn(C3["B"], C3["H"], C3["N"], d, seed=3000)
        scale = d ** -0.5

        def step():
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                torch.nn.functional.scaled_dot_product_attention(
                    q, k, v, is_causal=True, scale=scale)

        ms = timer.run(step, steps, warmup) / steps
        tf = (prefill_flops(C3["B"], C3["H"], C3["N"], True) * d / HEAD_DIM
              / (ms * 1e-3) / 1e12)
        return {"ms": round(ms, 5), "tflops": round(tf, 2),
                "ours_over_cudnn": round(ours_tflops / tf, 3),
                "note": "cuDNN fused attention (torch SDPA, CUDNN_ATTENTION "
                        f"backend) on config 3 at head_dim {d}: library "
                        "kernel, context only"}
    except Exception as exc:  # library missing or backend refused the shape
        return {"unavailable": f"{type(exc).__name__}: {str(exc)[:120]}"}


REF_HEADS_PER_STEP = 4


def workload_config(world):
    """The headline workload's config (both arms print the same one)."""
    return {"workload": "config3_qwen2.5-0.5b_causal_prefill",
            "global_batch": C3["B"], "heads": C3["H"], "seq_len": C3["N"],
            "head_dim": HEAD_DIM, "causal": True,
            "parallelism": f"batch*head sharded over {world} GPU(s)",
            "l2": "flushed before every timed step (512 MiB written then read back)"}


def run_reference(args, rank, world):
    """The reference's CPU path on the host cores, rank 0 only. One timed
    step is REF_HEADS_PER_STEP of config 3's 56 (batch, head) evaluations
    (the whole config would take minutes per step); ms_per_step is the time
    of that step as run, and the rate is the workload's own FLOP rate."""
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_sample_heads(0.0, heads=REF_HEADS_PER_STEP)
    secs = []
    for _ in range(args.steps):
        _, t = cpu_sample_heads(0.0, heads=REF_HEADS_PER_STEP)
        secs.append(t)
    secs_total = sum(secs)
    heads_total = REF_HEADS_PER_STEP * args.steps
    flops = prefill_flops(1, heads_total, C3["N"], True)
    value = flops / secs_total / 1e12
    result = {
        "impl": "reference",
        "metric": "causal prefill TFLOP/s (B=4,H=14,N=4096,d=64 fp16)",
        "value": round(value, 5), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs_total / args.steps * 1e3, 1),
        "step": f"{REF_HEADS_PER_STEP} of config 3's {C3['B'] * C3['H']} "
                f"causal N={C3['N']} (batch, head) evaluations",
        "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 (numpy, inputs rounded to fp16)",
        "data": "synthetic N(0,1), seeded",
        "config": workload_config(world),
        "host": "reference CPU path on the host cores of rank 0 (the L2 flush "
                "and GPU sharding in config describe the GPU arm's timing)",
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s",
                         "cores": cpu_threads(), "kind": "port",
                         "sample": f"{heads_total} heads of config 3 over "
                                   f"{args.steps} steps ({secs_total:.1f} s)"},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-library", action="store_true",
                    help="skip the cuDNN (torch SDPA) comparison line")
    ap.add_argument("--no-ref-cuda", action="store_true",
                    help="skip timing the reference's own CUDA kernels")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if "RANK" not in os.environ:
        world = 1
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
