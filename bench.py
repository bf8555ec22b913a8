#!/usr/bin/env python
"""Benchmark of the B200 attention hot path: causal D=128 forward + deterministic backward.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--S 8192]

One step = one fused-attention forward plus the deterministic backward (autograd through
``fastflashattention_b200.fast_attention``) over one batch of seeded N(0,1) bf16 inputs
of the reference's headline shape B=4, H=16, S=8192, D=128, causal (
the other configs are parity-test cases).  FLOPs follow the reference convention
(bench/common.py:142-153): fwd = 4*B*H*S^2*D*(1/2 if causal), step = 3.5 * fwd.

Multi-GPU (torchrun, one process per GPU): every rank draws the same global batch of
4*N sequences from one seed and owns a disjoint, contiguous block of its (batch, head)
slices (``shard.shard_heads``; weak scaling, no data-path collective); the time is the max
over ranks of the device-timed region.  Beside it, ``configs3_box`` times BASELINE
configs[3] as stated: one global B8 H32 S8192 D128 problem split over the N ranks
(strong scaling).  Rank 0 prints one JSON line.

``--impl reference`` times the reference's CPU path for this hot path — its parity
oracle, fp32 ``F.scaled_dot_product_attention`` forward + autograd backward
(oracle/sdpa_oracle.py) — on the host cores, one (batch, head) slice of the same
workload per step, and prints the same JSON line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = "fwd+bwd attention TFLOP/s (causal, D=128) and % of B200 bf16 tensor peak"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (read + write) per launch of the dK/dV kernel, from one ncu capture of that
# kernel at B2 H16 S8192 D128 causal (32 slices; dram__bytes_read.sum + dram__bytes_write.sum),
# scaled to the bench's (batch, head) slice count: traffic grows in proportion to slices.
DKDV_DRAM_BYTES_PER_SLICE = (284.571648e6 + 106.757120e6) / 32


def attn_flops(B, H, S, D, causal):
    fwd = 4.0 * B * H * S * S * D * (0.5 if causal else 1.0)
    return fwd, 3.5 * fwd


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples the SM clock, power and clock-event reasons of one GPU while running.

    NVML is polled every 2 ms from a thread (the timed region of a step is tens of
    milliseconds, shorter than nvidia-smi's loop period); without NVML, nvidia-smi -lms
    100 is read instead.  Every sample carries a host timestamp and ``stop`` keeps the
    ones inside the window marked by ``begin()`` / ``end()``, the timed region.
    """

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, bus_id: str | None, fallback_index: int = 0):
        self.bus_id = (bus_id or "").lower()
        self.fallback_index = str(fallback_index)
        self.proc = None
        self.samples: list[tuple[float, float, float, float, tuple]] = []  # t, sm, max, W, reasons
        self.lines: list[tuple[float, str]] = []
        self._t = None
        self._stop = threading.Event()
        self._nvml = None
        self.window = (0.0, float("inf"))
        self.source = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                h = pynvml.nvmlDeviceGetHandleByPciBusId(self.bus_id.upper()) if self.bus_id else None
            except pynvml.NVMLError:
                h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(int(self.fallback_index))
            self._nvml = (pynvml, h)
            self.source = "nvml 2 ms"
            self._t = threading.Thread(target=self._poll_nvml, daemon=True)
            self._t.start()
            return
        except Exception:  # noqa: BLE001 - no NVML: fall back to nvidia-smi
            self._nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.source = "nvidia-smi 100 ms"
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _poll_nvml(self):
        nv, h = self._nvml
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                w = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                names = tuple(n for n, b in zip(self.REASONS, bits) if r & b)
                self.samples.append((time.monotonic(), sm, mx, w, names))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def begin(self):
        self.window = (time.monotonic(), float("inf"))

    def end(self):
        self.window = (self.window[0], time.monotonic())

    def stop(self):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        if self.proc is not None:
            allrows = [(t, [x.strip() for x in ln.split(",")]) for t, ln in self.lines]
            allrows = [(t, p) for t, p in allrows if len(p) >= 10]
            rows = [(t, p) for t, p in allrows if self.bus_id and p[1].lower().endswith(self.bus_id[-7:])]
            if not rows:  # bus id unknown or not matched: nvidia-smi index of the local device
                rows = [(t, p) for t, p in allrows if p[0] == self.fallback_index]
            for t, r in rows:
                if r[2].replace(".", "").isdigit() and r[3].replace(".", "").isdigit():
                    w = float(r[4]) if r[4].replace(".", "").isdigit() else 0.0
                    names = tuple(n for i, n in enumerate(self.REASONS) if r[6 + i].lower() == "active")
                    self.samples.append((t, float(r[2]), float(r[3]), w, names))
        if not self.samples:
            return None
        lo, hi = self.window
        inside = [x for x in self.samples if lo <= x[0] <= hi]
        rows = inside or self.samples
        mx = max(x[2] for x in rows)
        sm = [x[1] for x in rows]
        loaded = [v for v in sm if v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted({n for x in rows for n in x[4]}),
                "samples": len(rows), "in_timed_region": bool(inside),
                "power_w_median": round(statistics.median(x[3] for x in rows), 1),
                "power_w_max": round(max(x[3] for x in rows), 1), "source": self.source}


def pci_bus_string(props):
    """nvidia-smi style bus id ("00000000:1B:00.0") of a torch device, or None."""
    try:
        dom, bus, devn = int(props.pci_domain_id), int(props.pci_bus_id), int(props.pci_device_id)
    except (AttributeError, TypeError, ValueError):
        return None
    return "%08X:%02X:%02X.0" % (dom, bus, devn)


# ------------------------------------------------------------------------- CPU oracle
def cpu_reference_sample(S, D, causal, heads=1, reps=1, seed=0):
    """fp32 math-SDPA forward+backward on the host (the reference's parity oracle) for
    `heads` (batch, head) slices of length S.  Returns (seconds per slice, threads)."""
    import torch
    sys.path.insert(0, str(ROOT))
    from oracle.sdpa_oracle import sdpa_fwd_bwd
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    mk = lambda: torch.randn(1, heads, S, D, generator=g).to(torch.bfloat16)  # noqa: E731
    q, k, v, do = mk(), mk(), mk(), mk()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        sdpa_fwd_bwd(q, k, v, do, causal)
        times.append(time.perf_counter() - t0)
    return min(times) / heads, threads


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    B, H, S, D, causal = args.B, args.H, args.S, args.D, True
    _, step_flops_slice = attn_flops(1, 1, S, D, causal)
    secs = []
    threads = 1
    for i in range(args.warmup + args.steps):
        s, threads = cpu_reference_sample(S, D, causal, heads=1, reps=1, seed=i)
        if i >= args.warmup:
            secs.append(s)
    t = statistics.median(secs)
    value = step_flops_slice / t / 1e12
    sample = f"one (batch, head) slice of B{B} H{H} S{S} D{D} causal per step (1/{B * H} of the workload)"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) bf16 inputs, seeded",
        "impl": "reference",
        "config": dict(config_dict(args, world),
                       workload=f"B{B} H{H} S{S} D{D} causal fwd+bwd, sampled: each timed step is one (batch, head) "
                                f"slice, 1/{B * H} of the workload; the rate is FLOP of that slice / its time"),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "fp32 F.scaled_dot_product_attention (math) fwd + autograd bwd on host cores: the reference's "
                "parity oracle (tests/test_parity.py:32-35); ms_per_step is the measured time of one sampled slice",
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(args, world):
    return {
        "workload": f"B{args.B} H{args.H} S{args.S} D{args.D} causal fwd+bwd per GPU (weak scaling: one global "
                    f"problem of B={args.B * world} from one seed, each rank a contiguous block of its slices)",
        "B": args.B, "H": args.H, "S": args.S, "D": args.D, "causal": True,
        "global_batch": args.B * world, "seq_len": args.S,
        "parallelism": f"dp{world} (disjoint batch x head slices, no collective)",
        "l2": "inputs larger than L2: q, k, v, dO are 4 x %d MiB per GPU" % (args.B * args.H * args.S * args.D * 2 >> 20),
    }


# ------------------------------------------------------------------------------ ours
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from fastflashattention_b200 import _lib, fast_attention
    from fastflashattention_b200._kernel import fastflash_attn

    from fastflashattention_b200 import shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, H, S, D = args.B, args.H, args.S, args.D
    causal = True
    fwd_flops, step_flops = attn_flops(B, H, S, D, causal)

    def barrier():
        if world > 1:
            dist.barrier()

    def global_inputs(Bg, Hg, seed):
        """One global problem [Bg, Hg, S, D] drawn from one seed (every rank draws the same
        tensors) and this rank's contiguous block of (batch, head) slices of it, as views
        (shard.shard_heads); the global tensors are kept alive by the views."""
        gen = torch.Generator(device=dev).manual_seed(seed)
        full = [torch.randn(Bg, Hg, S, D, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(4)]
        return [shard.shard_heads(t, rank, world) for t in full]

    def make_step(q_, k_, v_, do_):
        qg_, kg_, vg_ = (t.detach().requires_grad_(True) for t in (q_, k_, v_))

        def step():
            o = fast_attention(qg_, kg_, vg_, is_causal=causal)
            return torch.autograd.grad(o, (qg_, kg_, vg_), do_)
        return step

    def timed(step, n):
        """Device ms per step over `n` steps on this rank, then the max over ranks."""
        e0_, e1_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0_.record(torch.cuda.current_stream(dev))
        for _ in range(n):
            step()
        e1_.record(torch.cuda.current_stream(dev))
        torch.cuda.synchronize()
        barrier()
        return shard.max_over_ranks(e0_.elapsed_time(e1_) / n)

    # Weak scaling (the headline line): a global batch of B*world sequences, H heads, one
    # seed; every rank owns B*H slices of it (world == 1: the whole B x H problem).
    q, k, v, do = (t.reshape(B, H, S, D) for t in global_inputs(B * world, H, 0))
    step = make_step(q, k, v, do)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    sampler = ClockSampler(pci_bus_string(torch.cuda.get_device_properties(dev)), local_rank)
    sampler.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    sampler.begin()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    sampler.end()
    barrier()
    ms_local = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop()
    ms = shard.max_over_ranks(ms_local)
    value = world * step_flops / (ms / 1e3) / 1e12

    # BASELINE configs[3] as stated: ONE global B8 H32 S8192 D128 causal problem split over
    # the ranks (strong scaling, whole-box TFLOP/s = total FLOP / max-rank time).
    box = None
    if not args.no_box:
        Bb, Hb = 8, 32
        bq, bk, bv, bdo = global_inputs(Bb, Hb, 3)
        bstep = make_step(bq, bk, bv, bdo)
        for _ in range(args.warmup):
            bstep()
        bms = timed(bstep, max(3, args.steps // 2))
        _, box_flops = attn_flops(Bb, Hb, S, D, causal)
        box = {"workload": f"B{Bb} H{Hb} S{S} D{D} causal fwd+bwd, one global problem split over {world} GPU(s) "
                           f"({bq.shape[1]} of {Bb * Hb} (batch, head) slices on rank 0)",
               "value": box_flops / (bms / 1e3) / 1e12, "unit": UNIT, "ms_per_step": bms, "scaling": "strong",
               "parallelism": f"dp{world} (shard.shard_heads of one global tensor, no collective)"}
        del bq, bk, bv, bdo, bstep
        torch.cuda.empty_cache()

    # ---- per-kernel times (same inputs, each kernel alone, CUDA events on this stream)
    lib = _lib.load()
    BH = B * H
    qf, kf, vf, dof = (t.reshape(BH, S, D) for t in (q, k, v, do))
    o, lse = fastflash_attn(q, k, v, causal, return_lse=True)
    of, lf = o.reshape(BH, S, D), lse.reshape(BH, S)
    delta = torch.empty(BH, S, device=dev, dtype=torch.float32)
    dq, dk, dv = (torch.empty_like(qf) for _ in range(3))
    sm = 1.0 / math.sqrt(D)
    sp = stream.cuda_stream
    st = D * 1, S * D
    kernels = {
        "fwd": lambda: lib.ffa_fwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), of.data_ptr(), lf.data_ptr(),
                                   BH, S, D, st[1], st[0], sm, 1, sp),
        "bwd_preprocess": lambda: lib.ffa_bwd_preprocess(of.data_ptr(), dof.data_ptr(), delta.data_ptr(), BH, S, D,
                                                         st[1], st[0], sp),
        "bwd_dkdv": lambda: lib.ffa_bwd_dkdv(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), dof.data_ptr(),
                                             lf.data_ptr(), delta.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                             BH, S, D, st[1], st[0], sm, 1, sp),
        "bwd_dq": lambda: lib.ffa_bwd_dq(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), dof.data_ptr(), lf.data_ptr(),
                                         delta.data_ptr(), dq.data_ptr(), BH, S, D, st[1], st[0], sm, 1, sp),
    }
    half = 0.5
    mm = 2.0 * BH * S * S * D * half  # one S x S x D contraction, causal half
    algo = {"fwd": (2 * mm, "flop"), "bwd_dkdv": (4 * mm, "flop"), "bwd_dq": (3 * mm, "flop"),
            "bwd_preprocess": (2.0 * BH * S * D * 2 + BH * S * 4, "byte")}
    kinfo = {}
    for name, fn in kernels.items():
        for _ in range(3):
            _lib.check(fn(), name)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(3, args.steps)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        kms = a.elapsed_time(b) / n
        amount, kind = algo[name]
        rate = amount / (kms / 1e3) / (1e12 if kind == "flop" else 1e9)
        kinfo[name] = {"ms": round(kms, 4), ("tflops" if kind == "flop" else "gbs"): round(rate, 1)}
    status = _lib.device_status()

    peaks, peak_kind = load_peaks()
    dk_ms = kinfo["bwd_dkdv"]["ms"]
    achieved = algo["bwd_dkdv"][0] / (dk_ms / 1e3) / 1e12
    peak = float(peaks["bf16_tflops"])
    traffic = None if DKDV_DRAM_BYTES_PER_SLICE is None else DKDV_DRAM_BYTES_PER_SLICE * BH
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": "ffa_bwd_dkdv_kernel",
                "peak_source": f"{peak_kind} bf16_tflops (burst; the kernel is timed alone)",
                "algorithmic": "4 contractions (S^T, dP^T, dV, dK) x 2*B*H*S^2*D x 1/2 causal per launch"}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # The step is split into head chunks on their own streams, so the upload of one
        # chunk and the download of another overlap the attention of a third (H2D and
        # D2H use separate copy engines).  Every byte still crosses PCIe every step.
        BHn = B * H
        flat = lambda t: t.reshape(1, BHn, S, D)  # noqa: E731
        hq, hk, hv, hdo = (flat(t).cpu().pin_memory() for t in (q, k, v, do))
        gq, gk, gv = (torch.empty(hq.shape, dtype=q.dtype, pin_memory=True) for _ in range(3))
        dq_in, dk_in, dv_in, ddo = (torch.empty((1, BHn, S, D), device=dev, dtype=q.dtype) for _ in range(4))
        n_chunks = max(1, min(args.e2e_chunks, BHn))
        bounds = [BHn * c // n_chunks for c in range(n_chunks + 1)]
        streams = [torch.cuda.Stream(device=dev) for _ in range(n_chunks)]

        def e2e_step():
            start = torch.cuda.Event()
            start.record(stream)
            done = []
            for c, cs in enumerate(streams):
                h0, h1 = bounds[c], bounds[c + 1]
                cs.wait_event(start)
                with torch.cuda.stream(cs):
                    with torch.no_grad():
                        for dst, src in ((dq_in, hq), (dk_in, hk), (dv_in, hv), (ddo, hdo)):
                            dst[:, h0:h1].copy_(src[:, h0:h1], non_blocking=True)
                    a_, b_, c_ = (t[:, h0:h1].detach().requires_grad_(True) for t in (dq_in, dk_in, dv_in))
                    o_ = fast_attention(a_, b_, c_, is_causal=causal)
                    g = torch.autograd.grad(o_, (a_, b_, c_), ddo[:, h0:h1])
                    for dst, src in ((gq, g[0]), (gk, g[1]), (gv, g[2])):
                        dst[:, h0:h1].copy_(src, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    done.append(ev)
            for ev in done:
                stream.wait_event(ev)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ems = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([ems], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        nbytes = q.numel() * q.element_size()
        e2e = {"value": world * step_flops / (ems / 1e3) / 1e12, "unit": UNIT, "ms_per_step": ems,
               "h2d_bytes_per_step": 4 * nbytes * world, "d2h_bytes_per_step": 3 * nbytes * world,
               "path": "pinned host q,k,v,dO -> fast_attention fwd + autograd bwd -> dq,dk,dv to pinned host",
               "pipelining": f"{n_chunks} head chunks on {n_chunks} streams (copies overlap compute)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        secs, threads = cpu_reference_sample(S, D, causal, heads=1, reps=2)
        _, flops_slice = attn_flops(1, 1, S, D, causal)
        cpu = {"value": flops_slice / secs / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"one (batch, head) slice of B{B} H{H} S{S} D{D} causal, fp32 math SDPA fwd+bwd, best of 2",
               "ms_per_slice": secs * 1e3}

    if rank == 0:
        spec = 2250.0
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1) bf16 inputs, seeded (no dataset)",
            "config": config_dict(args, world),
            "pct_peak": {"of_measured_bf16": round(100 * value / world / peak, 2),
                         "of_spec_2250": round(100 * value / world / spec, 2)},
            "roofline": roofline,
            "kernels": kinfo,
            "configs3_box": box,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": 4 * args.steps,
            "device_status": list(status),
        }
        print(json.dumps(line), flush=True)
    return 0


def run_ring(args, rank, world, local_rank):
    """Context-parallel ring: the sequence (B1 H32 S131072 D128 causal unless overridden)
    is split zig-zag over the ranks; value = whole-sequence fwd+bwd FLOPs / max-rank time."""
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from fastflashattention_b200 import _lib, ring

    B, H, S, D = 1, 32, 131072, 128
    if args.S != 8192:
        S = args.S
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    try:
        C2 = S // world
        gen = torch.Generator(device=dev).manual_seed(1000 + rank)
        mk = lambda: torch.randn(B, H, C2, D, device=dev, dtype=torch.bfloat16, generator=gen)  # noqa: E731
        q, k, v, do = mk(), mk(), mk(), mk()
        qg, kg, vg = (t.detach().requires_grad_(True) for t in (q, k, v))

        if world > 1:
            def step():
                o = ring.ring_attention(qg, kg, vg)
                return torch.autograd.grad(o, (qg, kg, vg), do)
        else:
            from fastflashattention_b200 import fast_attention

            def step():
                o = fast_attention(qg, kg, vg, is_causal=True)
                return torch.autograd.grad(o, (qg, kg, vg), do)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        sampler = ClockSampler(pci_bus_string(torch.cuda.get_device_properties(dev)), local_rank)
        sampler.start()
        time.sleep(0.1)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler.begin()
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        sampler.end()
        clocks = sampler.stop()
        ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        _, step_flops = attn_flops(B, H, S, D, True)
        if rank == 0:
            print(json.dumps({
                "metric": METRIC + " [context-parallel ring]", "value": step_flops / (ms / 1e3) / 1e12, "unit": UNIT,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic N(0,1) bf16 inputs, seeded",
                "config": {"workload": f"B{B} H{H} S{S} D{D} causal fwd+bwd, sequence split zig-zag over {world} GPUs",
                           "parallelism": f"cp{world} (ring: NCCL send/recv of K/V and dK/dV)"},
                "clocks": clocks, "device_status": list(_lib.device_status())}), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


def run_once(args):
    """A plain forward + backward of the library at --B --H --S --D causal, --warmup then
    --steps times, with no timing: the command profilers wrap (ncu launch lists and
    single-kernel captures on a case small enough to capture)."""
    import torch
    sys.path.insert(0, str(ROOT))
    from fastflashattention_b200 import _lib, fast_attention
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(args.B, args.H, args.S, args.D, device="cuda", dtype=torch.bfloat16, generator=gen)
                   for _ in range(4))
    qg, kg, vg = (t.requires_grad_(True) for t in (q, k, v))
    for _ in range(args.warmup + args.steps):
        o = fast_attention(qg, kg, vg, is_causal=not args.noncausal)
        torch.autograd.grad(o, (qg, kg, vg), do)
    torch.cuda.synchronize()
    print(json.dumps({"mode": "once", "B": args.B, "H": args.H, "S": args.S, "D": args.D,
                      "causal": not args.noncausal, "device_status": list(_lib.device_status())}))
    return 0


# ------------------------------------------------------------------ comparator sweep
SWEEP_S = [512, 1024, 2048, 4096, 8192, 16384]


def _comparators(causal):
    """name -> f(q, k, v) over [B,H,S,D] bf16 tensors, for every implementation that
    imports here.  Library kernels (cuDNN SDPA through torch, FlashAttention-2, the
    reference's Triton kernels from baseline/_ref) run as black boxes, as in the
    reference's bench/benchmark.py:25-41 (FA2 in [B,S,H,D] framing, transposed in and out)."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from fastflashattention_b200 import fast_attention

    impls = {"ours": lambda a, b, c: fast_attention(a, b, c, is_causal=causal)}
    notes = {}
    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "fastflash_attention" / "__init__.py").exists():
        sys.path.insert(0, str(ref_dir))
        try:
            import fastflash_attention as ref_mod
            impls["reference_triton"] = lambda a, b, c: ref_mod.fast_attention(a, b, c, is_causal=causal)
        except Exception as e:  # noqa: BLE001
            notes["reference_triton"] = f"import failed: {e!r}"[:200]
        finally:
            sys.path.remove(str(ref_dir))
    else:
        notes["reference_triton"] = "baseline/_ref not installed"

    def cudnn(a, b, c):
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            return F.scaled_dot_product_attention(a, b, c, is_causal=causal)
    impls["cudnn_sdpa"] = cudnn
    try:
        from flash_attn import flash_attn_func

        def fa2(a, b, c, det):
            q2, k2, v2 = (t.transpose(1, 2).contiguous() for t in (a, b, c))
            return flash_attn_func(q2, k2, v2, causal=causal, deterministic=det).transpose(1, 2)
        impls["fa2"] = lambda a, b, c: fa2(a, b, c, False)
        impls["fa2_det"] = lambda a, b, c: fa2(a, b, c, True)
    except Exception as e:  # noqa: BLE001
        notes["fa2"] = f"import failed: {e!r}"[:200]
    return impls, notes


def _event_ms(fn, warmup, iters):
    """Median CUDA-event time of fn() in ms (warm-up excluded), like bench/common.py:78-103."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = []
    for _ in range(iters):
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b))
    return statistics.median(out)


def run_sweep(args):
    """Forward / backward / step times of every comparator over the reference's S sweep
    (bench/benchmark.py: B4 H16, D in {64, 128}, causal and not).  One JSON line per
    (D, causal, S); an implementation that fails at a shape reports its error instead."""
    import torch
    sys.path.insert(0, str(ROOT))
    torch.cuda.set_device(0)
    peaks, peak_kind = load_peaks()
    peak = float(peaks["bf16_tflops"])
    blocks = [(128, True), (64, False), (128, False), (64, True)]
    if args.sweep_blocks:  # e.g. "128c,64n": head dim, then c(ausal) or n(on-causal)
        blocks = [(int(b[:-1]), b[-1] == "c") for b in args.sweep_blocks.split(",")]
    Ss = [int(x) for x in args.sweep_s.split(",")] if args.sweep_s else SWEEP_S
    for D, causal in blocks:
        impls, notes = _comparators(causal)
        for S in Ss:
            g = torch.Generator(device="cuda").manual_seed(0)
            mk = lambda: torch.randn(args.B, args.H, S, D, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
            q, k, v, do = mk(), mk(), mk(), mk()
            fwd, step = attn_flops(args.B, args.H, S, D, causal)
            row = {"mode": "sweep", "B": args.B, "H": args.H, "S": S, "D": D, "causal": causal,
                   "peak_tflops": peak, "peak_source": peak_kind, "impls": {}, "notes": notes}
            for name, fn in impls.items():
                try:
                    with torch.no_grad():
                        t_f = _event_ms(lambda: fn(q, k, v), args.warmup, args.steps)
                    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
                    out = fn(qg, kg, vg)
                    t_b = _event_ms(lambda: torch.autograd.grad(out, (qg, kg, vg), do, retain_graph=True),
                                    args.warmup, args.steps)
                    del out

                    def st():
                        o_ = fn(qg, kg, vg)
                        torch.autograd.grad(o_, (qg, kg, vg), do)
                    t_s = _event_ms(st, args.warmup, args.steps)
                    row["impls"][name] = {
                        "fwd_ms": round(t_f, 4), "bwd_ms": round(t_b, 4), "step_ms": round(t_s, 4),
                        "fwd_tflops": round(fwd / t_f / 1e9, 1), "bwd_tflops": round((step - fwd) / t_b / 1e9, 1),
                        "step_tflops": round(step / t_s / 1e9, 1),
                        "step_pct_measured_peak": round(100 * step / t_s / 1e9 / peak, 1)}
                except Exception as e:  # noqa: BLE001
                    row["impls"][name] = {"error": f"{type(e).__name__}: {e}"[:200]}
                torch.cuda.empty_cache()
            print(json.dumps(row), flush=True)
            del q, k, v, do
            torch.cuda.empty_cache()
    return 0


# ------------------------------------------------------------------------ peak memory
def _mem_worker(impl, S, regime, B, H, D):
    """Peak allocated MB of one (impl, S, regime) point in this fresh process (the
    reference's bench/mem.py:37-75 method: warm up, gc, reset the peak, one call)."""
    import gc
    import torch
    sys.path.insert(0, str(ROOT))
    torch.cuda.set_device(0)
    fn = _comparators(True)[0][impl]
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda: torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, do = mk(), mk(), mk(), mk()
    if regime == "fwd":
        def step():
            with torch.no_grad():
                fn(q, k, v)
    else:
        def step():
            qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
            out = fn(qg, kg, vg)
            torch.autograd.grad(out, (qg, kg, vg), do)
    for _ in range(6):
        step()
    torch.cuda.synchronize()
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    step()
    torch.cuda.synchronize()
    print(json.dumps({"impl": impl, "S": S, "regime": regime,
                      "peak_mb": round(torch.cuda.max_memory_allocated() / 1e6, 1)}), flush=True)
    return 0


def run_mem(args):
    """Peak allocated memory, forward-only and training step, B4 H16 D128 causal, each
    point in a fresh process; one JSON line per S with every implementation's MB."""
    Ss = [int(x) for x in args.sweep_s.split(",")] if args.sweep_s else SWEEP_S
    impls = ["ours", "reference_triton", "fa2", "cudnn_sdpa"]
    for S in Ss:
        row = {"mode": "mem", "B": args.B, "H": args.H, "S": S, "D": 128, "causal": True,
               "inputs_mb": round(4 * args.B * args.H * S * 128 * 2 / 1e6, 1), "fwd": {}, "train": {}}
        for regime in ("fwd", "train"):
            for impl in impls:
                cp = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--mode", "mem-worker",
                                     "--mem-impl", impl, "--S", str(S), "--mem-regime", regime,
                                     "--B", str(args.B), "--H", str(args.H)],
                                    capture_output=True, text=True)
                lines = [ln for ln in cp.stdout.splitlines() if ln.startswith("{")]
                row[regime][impl] = (json.loads(lines[-1])["peak_mb"] if lines and cp.returncode == 0
                                     else "error: " + (cp.stderr.strip().splitlines() or ["?"])[-1][:160])
        print(json.dumps(row), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--B", type=int, default=4)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--S", type=int, default=8192)
    ap.add_argument("--D", type=int, default=128)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=16, help="head chunks (streams) of the pipelined e2e step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-box", action="store_true", help="skip the B8 H32 global-problem (configs[3]) figure")
    ap.add_argument("--noncausal", action="store_true", help="--mode once: no causal mask")
    ap.add_argument("--mode", choices=["shard", "ring", "sweep", "mem", "mem-worker", "once"], default="shard",
                    help="shard: batch x head data parallel (default workload); ring: context-parallel ring "
                         "over the sequence (BASELINE configs[4]: B1 H32 S131072 D128); sweep: fwd/bwd/step "
                         "of this library beside cuDNN SDPA, FlashAttention-2 and the reference's Triton "
                         "kernels over S (one GPU); mem: peak memory of the same, fresh process per point; "
                         "once: untimed fwd+bwd at the given shape (for profilers)")
    ap.add_argument("--sweep-s", default="", help="comma-separated S list for --mode sweep/mem")
    ap.add_argument("--sweep-blocks", default="", help="--mode sweep blocks, e.g. 128c,64n (default: all four)")
    ap.add_argument("--mem-impl", default="ours")
    ap.add_argument("--mem-regime", choices=["fwd", "train"], default="train")
    args = ap.parse_args()
    if args.warmup < 3 and args.mode != "once":
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.mode == "ring":
        return run_ring(args, rank, world, local_rank)
    if args.mode == "sweep":
        return run_sweep(args)
    if args.mode == "mem":
        return run_mem(args)
    if args.mode == "once":
        return run_once(args)
    if args.mode == "mem-worker":
        return _mem_worker(args.mem_impl, args.S, args.mem_regime, args.B, args.H, args.D)
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
