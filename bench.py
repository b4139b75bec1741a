#!/usr/bin/env python
"""Benchmark of the FP4 fused attention path on B200 (one process per GPU).

Metric: fused FP4 attention TFLOPS = 4 * B * H * seq_q * seq_k * head_dim / t
(the reference's formula, tests/benchmark.cu:85-86), plus the fraction of the
mixed FP4/FP16 tensor roofline.  One step = one pass of the path over this
rank's shard: quantise Q and K (E2M1 + UE8M0/32) and run the attention kernel,
inputs resident in HBM.  Default workload: the prefill-sized single-GPU case,
batch 2, heads 32, seq_q = seq_k = 4096, head_dim 128, FP16 in/out.  Under
torchrun each rank runs that workload's 64 (batch x head) slices as its shard
of a job with 64*N slices (weak scaling, no collective on the data path; NCCL
only carries the barrier and the max-over-ranks of the timings).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --pass backward [--workload prefill_4k]   (the backward pass, one GPU)

The backward line (fp4attn_backward: dQ, dK, dV of the same workload) counts
10 * B * H * seq_q * seq_k * head_dim FLOPs per pass (S recomputed, dP, dV,
dK, dQ: 2.5x the forward's) against the mixed roofline with S at the FP4 rate
and the other four products at the FP16 rate.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 2**20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="prefill_4k")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--fuse-q", action="store_true",
                    help="quantise Q inside the attention kernel (fp4attn_forward_fused_q) in the timed step")
    ap.add_argument("--box-steps", type=int, default=5,
                    help="steps of this rank's share of the box-scale job (0: skip)")
    ap.add_argument("--pass", dest="direction", choices=["forward", "backward"], default="forward",
                    help="forward (the headline) or the backward pass of the workload")
    ap.add_argument("--causal", action="store_true",
                    help="bottom-right causal mask (not in the reference); FLOPs counted over the visible "
                         "(query, key) pairs")
    ap.add_argument("--in-dtype", choices=["float16", "float32"], default="float16",
                    help="backward pass: Q, K, V and dO in FP16 or FP32 (FP32 adds the FP16 conversion of V and dO)")
    return ap.parse_args()


def measured_peaks():
    """Dense bf16 TFLOP/s as a burst (a kernel timed alone, at full clock)
    and sustained (seconds-long back-to-back work at the power cap), HBM
    GB/s, and where they come from."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        burst = float(d["bf16_tflops"])
        return burst, float(d.get("bf16_tflops_sustained") or burst), float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def peak_basis(timed_s, reasons):
    """The bf16 figure a kernel timed over `timed_s` seconds under the
    sampled throttle `reasons` is held to: the sustained one only when the
    timed region is seconds long and the clocks were power-capped in it,
    otherwise the burst one."""
    return "sustained" if timed_s >= 2.0 and "sw_power_cap" in reasons else "burst"


def mixed_roofline(w, bf16_tflops):
    """Mixed FP4/FP16 tensor roofline for this workload's FLOPs: QK^T at the
    dense FP4 peak (4x the dense FP16 peak, NVIDIA's ratio for B200) and P.V at
    the dense FP16 peak, the FP16 peak being the measured bf16 GEMM figure.
    Returns the equivalent peak in TFLOP/s for the whole 4*B*H*sq*sk*d."""
    f_half = w.flops() / 2
    t = f_half / (4 * bf16_tflops) + f_half / bf16_tflops
    return w.flops() / t


def visible_fraction(seq_q, seq_k, causal):
    """The share of (query, key) pairs a query sees: 1 without a mask; with
    the bottom-right causal mask, query i sees keys j <= i + seq_k - seq_q."""
    if not causal:
        return 1.0
    off = seq_k - seq_q
    pairs = sum(max(0, min(seq_k, i + off + 1)) for i in range(seq_q))
    return pairs / (seq_q * seq_k)


class ClockSampler:
    """nvidia-smi samples (100 ms) of SM clock and throttle reasons."""
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [l for (t, l) in self.lines if t0 <= t <= t1]
        if not rows:  # region shorter than the sampling period: nearest samples
            rows = [l for (t, l) in sorted(self.lines, key=lambda x: abs(x[0] - (t0 + t1) / 2))[:2]]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [x.strip() for x in r.split(",")]
            if len(f) < 10:
                continue
            try:
                sm.append(float(f[2]))
                mx = float(f[3])
            except ValueError:
                continue
            for n, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def profile_traffic(workload, kernel):
    """DRAM bytes per attention launch from the committed ncu summary of this
    kernel on this workload, if any."""
    p = ROOT / "profiles" / f"{kernel.replace('_kernel', '')}_{workload}.md"
    if p.exists():
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
        if m:
            return float(m.group(1))
    return None


class CpuReference:
    """The reference's CPU path (oracle/_ref: its quantiser and cpu_attention,
    tests/test_attention.cu:33-54, one slice per std::thread) on a bounded
    sample of the workload: one slice per host thread, each with a prefix of
    its query rows against all seq_k keys.  Falls back to the oracle port when
    _ref was not built (kind "port")."""

    def __init__(self, w, threads=None):
        import numpy as np
        import oracle
        self.w = w
        self.oracle = oracle
        self.threads = threads or os.cpu_count() or 1
        self.kind = "reference" if oracle.ref_available() else "port"
        rng = np.random.default_rng(0)
        n = self.threads
        shape = (n, w.seq_k, w.head_dim)
        self.K = (rng.standard_normal(shape, dtype=np.float32) * w.std).astype(np.float16).astype(np.float32)
        self.V = (rng.standard_normal(shape, dtype=np.float32) * w.std).astype(np.float16).astype(np.float32)
        self.Qfull = (rng.standard_normal((n, w.seq_q, w.head_dim), dtype=np.float32) * w.std
                      ).astype(np.float16).astype(np.float32)
        self.rows = 1

    def run(self, rows):
        Q = self.Qfull[:, :rows].copy()
        t = time.perf_counter()
        if self.kind == "reference":
            self.oracle.ref_fp4_attention(Q, self.K, self.V, threads=self.threads)
        else:
            self.oracle.fp4_attention(Q, self.K, self.V, threads=self.threads)
        dt = time.perf_counter() - t
        return 4.0 * self.threads * rows * self.w.seq_k * self.w.head_dim / dt / 1e12, dt

    def calibrate(self, budget_s):
        _, t1 = self.run(2)
        self.rows = int(max(1, min(self.w.seq_q, 2 * budget_s / max(t1, 1e-6))))
        return self.rows

    def sample(self):
        return f"{self.threads} slices x {self.rows} query rows x {self.w.seq_k} keys x d{self.w.head_dim}"


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL prints a version banner on stdout while it sets up; keep stdout
        # for the single result line by pointing fd 1 at stderr meanwhile.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    return world, rank, local


def time_box_share(args, world, rank, dev):
    """Quantise + attend over this rank's share of the 512-slice box-scale
    job (B16 H32 8192^2 d128, FP32 out): (ms per step, attention-kernel ms,
    slices).  Inputs are drawn on the device and exceed the L2."""
    import torch
    import fp4attn_b200 as fa
    import fp4attn_b200.workloads as wl
    w = wl.WORKLOADS["box_sharded_8k"]
    lo, hi = fa.shard_range(w.slices, world, rank)
    n = hi - lo
    Q, K, V = (t[None] for t in wl.make_inputs(w, args.seed, slices=(lo, hi), device=dev))
    out = torch.empty((1, n, w.seq_q, w.head_dim), dtype=torch.float32, device=dev)
    ws = torch.empty(fa.workspace_size(1, n, w.seq_q, w.seq_k, w.head_dim), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.box_steps)]
    sv = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.box_steps)]
    for i in range(2):
        fa.prepare(Q, K, V, ws)
        fa.attend(V, out, ws, fa.F16, 1, n, w.seq_q, w.seq_k, w.head_dim)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    # Whole steps (the attention kernel the quantiser's dependent) alternate
    # with steps that time the attention kernel alone, so both see the same
    # clocks; a step lasts milliseconds, so its own events cost nothing.
    for i in range(args.box_steps):
        sv[i][0].record(stream)
        fa.prepare(Q, K, V, ws)
        fa.attend(V, out, ws, fa.F16, 1, n, w.seq_q, w.seq_k, w.head_dim)
        sv[i][1].record(stream)
        fa.prepare(Q, K, V, ws)
        ev[i][0].record(stream)
        fa.attend(V, out, ws, fa.F16, 1, n, w.seq_q, w.seq_k, w.head_dim)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    if fa.status_query() != fa.OK:
        raise SystemExit("box-scale share reported a device timeout")
    ms = sum(e[0].elapsed_time(e[1]) for e in sv) / args.box_steps
    kms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.box_steps
    del Q, K, V, out, ws
    torch.cuda.empty_cache()
    return ms, kms, n


def l2_note(io_bytes, l2_bytes=L2_BYTES):
    """Whether timed steps are preceded by an L2 flush (inputs + output
    smaller than twice the L2), and the sentence that says so."""
    flush = io_bytes < 2 * l2_bytes
    text = (f"inputs+output {io_bytes / 2**20:.0f} MiB < 2x L2: {2 * l2_bytes / 2**20:.0f} MiB written before "
            f"every step (L2 flush), outside the step time" if flush else
            f"inputs+output {io_bytes / 2**20:.0f} MiB > 2x {l2_bytes / 2**20:.0f} MiB L2; no flush")
    return flush, text


def job_config(args, world, rank):
    """The workload, this rank's slice range and the run's `config` (the same
    keys and values in both arms)."""
    import fp4attn_b200.workloads as wl
    from fp4attn_b200 import shard_range
    base = wl.WORKLOADS[args.workload]
    strong = args.workload == "box_sharded_8k"
    if strong:  # fixed 512-slice job split over the ranks
        job = base
        lo, hi = shard_range(job.slices, world, rank)
    else:  # weak scaling: each rank runs the workload as its shard of a world-times larger batch
        job = wl.Workload(base.name, base.batch * world, base.heads, base.seq_q, base.seq_k, base.head_dim,
                          base.std, base.outlier_frac, base.outlier_mult, base.out_dtype)
        lo, hi = rank * base.slices, (rank + 1) * base.slices
    n = hi - lo
    out_bytes = 2 if base.out_dtype == "float16" else 4
    io_bytes = n * (2 * (base.seq_q + 2 * base.seq_k) + out_bytes * base.seq_q) * base.head_dim
    _, l2 = l2_note(io_bytes)
    config = {"workload": base.name, "shape": base.describe(), "slices_per_gpu": n, "job_slices": job.slices,
              "parallelism": f"slice-shard x{world}", "l2": l2}
    if args.causal:
        config["mask"] = "causal (FLOPs over the visible pairs)"
    return base, job, strong, lo, hi, config


def reference_arm(args, world, rank):
    if rank != 0:
        return
    if args.causal:
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no causal mask"}), flush=True)
        return
    base, _, strong, _, _, config = job_config(args, world, rank)
    cpu = CpuReference(base)
    cpu.calibrate(max(0.02, 60.0 / max(1, args.steps + args.warmup)))
    rates = []
    for i in range(args.warmup + args.steps):
        r, _ = cpu.run(cpu.rows)
        if i >= args.warmup:
            rates.append(r)
    value = statistics.median(rates)
    cores, kind, sample = cpu.threads, cpu.kind, cpu.sample()
    line = {
        "impl": "reference", "metric": "fused FP4 attention TFLOPS", "value": value, "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32 (CPU, FP4-dequantised Q/K)",
        "data": "synthetic", "config": config,
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_backward(args, world, rank, local):
    """One backward pass (fp4attn_backward: quantise Q and K with their BF16
    dequantised copies, the per-row Dd / lse2 pass, and the backward kernel)
    per step, inputs and the forward's output and log-sum-exp resident in
    HBM; one JSON line.  Under torchrun each rank runs the workload's slices
    as its shard of a world-times larger batch (weak scaling; NCCL carries
    only the barriers and the max over ranks of the timings)."""
    import torch
    import fp4attn_b200 as fa
    import fp4attn_b200.workloads as wl
    w = wl.WORKLOADS[args.workload]
    if w.head_dim not in (32, 64, 96, 128):
        raise SystemExit("the backward pass covers head_dim 32 to 128")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    Q, K, V = (t[None] for t in wl.make_inputs(w, args.seed + rank, device=dev))
    n = w.slices
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    dO = torch.randn(Q.shape, device=dev, generator=g).half()
    idt = fa.F32 if args.in_dtype == "float32" else fa.F16
    if idt == fa.F32:  # the same values, widened
        Q, K, V, dO = (t.float() for t in (Q, K, V, dO))
    odt = torch.float16 if w.out_dtype == "float16" else torch.float32
    out, lse = fa.fused_fp4_attention_lse(Q, K, V, out_dtype=odt, causal=args.causal)
    ws = torch.empty(fa.backward_workspace_size(1, n, w.seq_q, w.seq_k, w.head_dim, idt), dtype=torch.uint8,
                     device=dev)
    dq, dk, dv = (torch.empty(t.shape, dtype=torch.float32, device=dev) for t in (Q, K, V))
    L = fa.lib()
    stream = torch.cuda.current_stream(dev)
    sh = (1, n, w.seq_q, w.seq_k, w.head_dim)
    mask = fa.MASK_CAUSAL if args.causal else fa.MASK_NONE

    def step(ev_a=None, ev_b=None):
        rc = L.fp4attn_backward_prepare(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), dO.data_ptr(),
                                        lse.data_ptr(), dq.data_ptr(), idt, fa._dtype_code(out), *sh,
                                        fa.SCALE_REFERENCE, ws.data_ptr(), ws.numel(), stream.cuda_stream)
        if ev_a is not None:
            ev_a.record(stream)
        rc = rc or L.fp4attn_backward_attend(V.data_ptr(), dO.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                             dv.data_ptr(), idt, *sh, 0.0, mask, ws.data_ptr(), ws.numel(),
                                             stream.cuda_stream)
        if ev_b is not None:
            ev_b.record(stream)
        if rc != fa.OK:
            raise SystemExit(f"fp4attn_backward failed: {fa.lib().fp4attn_last_error().decode()}")

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    io_bytes = sum(t.numel() * t.element_size() for t in (Q, K, V, out, dO, dq, dk, dv))
    flush, l2 = l2_note(io_bytes)
    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if flush else None
    props = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler(f"GPU-{props.uuid}" if getattr(props, "uuid", None) else "0")
    sampler.start()
    time.sleep(0.5)
    sev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    # Whole passes and passes that time the backward kernel alone run in
    # alternating blocks, so that both see the same clocks.
    nblk = max(1, min(4, args.steps))
    bounds = [args.steps * j // nblk for j in range(nblk + 1)]
    for j in range(nblk):
        for i in range(bounds[j], bounds[j + 1]):  # whole passes
            if flush:
                flush_buf.zero_()
            sev[i][0].record(stream)
            step()
            sev[i][1].record(stream)
        for i in range(bounds[j], bounds[j + 1]):  # the backward kernel alone
            if flush:
                flush_buf.zero_()
            step(*kev[i])
    torch.cuda.synchronize()
    barrier()
    t_wall1 = time.time()
    torch.cuda.synchronize()
    time.sleep(0.3)
    sampler.stop()
    status = fa.status_query()
    ms_step = sum(a.elapsed_time(b) for a, b in sev) / args.steps
    kern_ms = sum(a.elapsed_time(b) for a, b in kev) / args.steps
    times = torch.tensor([ms_step, kern_ms, float(status)], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_step, kern_ms, status = times.tolist()
    if rank != 0:
        return
    flops = 10.0 * n * w.seq_q * w.seq_k * w.head_dim * visible_fraction(w.seq_q, w.seq_k, args.causal)  # per rank
    value = world * flops / (ms_step * 1e-3) / 1e12
    burst, sustained, hbm, peak_src = measured_peaks()
    clocks = sampler.summary(t_wall0, t_wall1)
    basis = peak_basis(ms_step * args.steps * 1e-3, clocks["reasons"])
    bf16 = burst if basis == "burst" else sustained
    # S (2/10 of the FLOPs) at 4x the FP16 rate, the other 8/10 at 1x.
    peak = flops / (0.2 * flops / (4 * bf16) + 0.8 * flops / bf16)
    line = {
        "metric": "fused FP4 attention backward TFLOPS", "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e2m1 (S) + f16/bf16 (dP, dV, dK, dQ)",
        "data": "synthetic (seeded N(0,1) FP16 on device" + (", widened to FP32)" if idt == fa.F32 else ")"),
        "config": {"workload": w.name, "shape": w.describe(), "pass": "backward", "in_dtype": args.in_dtype, "l2": l2,
                   "slices_per_gpu": n, "job_slices": n * world, "parallelism": f"slice-shard x{world}",
                   **({"mask": "causal (FLOPs over the visible pairs)"} if args.causal else {})},
        "roofline": {"bound": "tensor", "achieved": flops / (kern_ms * 1e-3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": flops / (kern_ms * 1e-3) / 1e12 / peak, "traffic": profile_traffic(w.name, "fp4_attention_bwd_kernel"),
                     "peak_basis": f"mixed: S at 4x and dP, dV, dK, dQ at 1x the {peak_src} {basis} bf16 dense "
                                   f"{bf16:g} TFLOP/s",
                     "kernel": "fp4_attention_bwd_kernel", "kernel_ms": kern_ms},
        "frac_of_mixed_roofline_step": value / world / peak,
        # per pass: quantise, rows, backward kernel (plus one memset of dQ); FP32
        # input adds the FP16 conversion of V and dO; the timed region holds
        # the timed passes and, interleaved, as many that time the kernel
        "gpu_launches": 2 * (4 if idt == fa.F32 else 3) * args.steps,
        "clocks": clocks,
        "device_status": int(status),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.causal and args.fuse_q:
        raise SystemExit("--fuse-q has no causal variant")
    if args.direction == "backward" and args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no backward pass"}), flush=True)
        return
    world, rank, local = dist_setup(args)
    if args.direction == "backward":
        bench_backward(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.impl == "reference":
        reference_arm(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch
    import fp4attn_b200 as fa
    import fp4attn_b200.workloads as wl

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    base, job, strong, lo, hi, config = job_config(args, world, rank)
    n = hi - lo
    Q, K, V = wl.make_inputs(job, args.seed, slices=(lo, hi), device=dev)
    Q, K, V = Q[None], K[None], V[None]  # [1, n, seq, d]: batch x head slices flattened
    odt = torch.float16 if base.out_dtype == "float16" else torch.float32
    out = torch.empty((1, n, base.seq_q, base.head_dim), dtype=odt, device=dev)
    ws = torch.empty(fa.workspace_size(1, n, base.seq_q, base.seq_k, base.head_dim), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    shard = wl.Workload(base.name, 1, n, base.seq_q, base.seq_k, base.head_dim)
    flops_rank = shard.flops() * visible_fraction(base.seq_q, base.seq_k, args.causal)

    def step(ev_q=None, ev_a=None, ev_b=None):
        if args.fuse_q:
            # The fused forward is one public call: the attention kernel cannot
            # be separated from the K pre-pass by events, so its events bracket both.
            if ev_a is not None:
                ev_q.record(stream)
                ev_a.record(stream)
            fa.fused_fp4_attention_into(Q, K, V, out, ws, fuse_q=True)
            if ev_b is not None:
                ev_b.record(stream)
            return
        if ev_q is not None:
            ev_q.record(stream)
        fa.prepare(Q, K, V, ws)
        if ev_a is not None:
            ev_a.record(stream)
        fa.attend(V, out, ws, fa.F16, 1, n, base.seq_q, base.seq_k, base.head_dim, causal=args.causal)
        if ev_b is not None:
            ev_b.record(stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if fa.status_query() != fa.OK:
        raise SystemExit("warm-up reported a device timeout")

    props = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler(f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local))
    sampler.start()
    time.sleep(0.5)
    # The attention kernel's time (the dominant kernel): CUDA events around it
    # in a second set of steps.  An event between the two launches would end
    # the programmatic overlap of the attention kernel's launch with the
    # quantiser, so the steps that give `value` carry none; the two sets run
    # in alternating blocks, so that both see the same clocks (run one after
    # the other, the second set met a power-capped, slower clock: 0.400 ms
    # against 0.352 ms for the same kernel).  The quantiser's span in the
    # second set is recorded too, and the step time less it (the attention
    # kernel's share of a step) is printed beside the kernel's own time.
    kev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
    nblk = max(1, min(4, args.steps))
    bounds = [args.steps * j // nblk for j in range(nblk + 1)]
    blk = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nblk)]
    # Inputs smaller than twice the L2 would be served from it: then every
    # timed step is preceded by a write of twice the L2 size, and each step is
    # timed by its own events so the flush stays outside the step time.
    io_bytes = sum(t.numel() * t.element_size() for t in (Q, K, V, out))
    flush, _ = l2_note(io_bytes)
    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if flush else None
    sev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    for j in range(nblk):
        blk[j][0].record(stream)
        for i in range(bounds[j], bounds[j + 1]):
            if flush:
                flush_buf.zero_()
                sev[i][0].record(stream)
            step()
            if flush:
                sev[i][1].record(stream)
        blk[j][1].record(stream)
        for i in range(bounds[j], bounds[j + 1]):
            if flush:
                flush_buf.zero_()
            step(*kev[i])
    torch.cuda.synchronize()
    barrier()
    t_wall1 = time.time()
    time.sleep(0.3)
    sampler.stop()
    status = fa.status_query()
    ms_total = (sum(a.elapsed_time(b) for a, b in sev) if flush else
                sum(a.elapsed_time(b) for a, b in blk))
    quant_ms = sum(q.elapsed_time(a) for q, a, _ in kev) / args.steps
    kern_ms = sum(a.elapsed_time(b) for _, a, b in kev) / args.steps
    kern_share_ms = ms_total / args.steps - quant_ms

    # End to end through the public API with host buffers.  Every step copies
    # its Q, K, V in from pinned host memory, runs fp4attn_forward (quantise +
    # attend) and copies its output back, all inside the timed region.  As a
    # serving loop would, consecutive steps overlap on three streams (H2D of
    # step i+1 and D2H of step i-1 run while step i computes) with two sets of
    # device buffers; events keep each set's uses in order.
    hQ, hK, hV = (x.cpu().pin_memory() for x in (Q, K, V))
    hO = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    d_in = [tuple(torch.empty_like(x) for x in (Q, K, V)) for _ in range(2)]
    d_out = [torch.empty_like(out) for _ in range(2)]
    s_in, s_cp, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
    ev_in, ev_cp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def e2e_step(i):
        b = i & 1
        s_in.wait_event(ev_cp[b])      # step i-2's attention is done with d_in[b]
        with torch.cuda.stream(s_in):
            for d, h in zip(d_in[b], (hQ, hK, hV)):
                d.copy_(h, non_blocking=True)
        ev_in[b].record(s_in)
        s_cp.wait_event(ev_in[b])
        s_cp.wait_event(ev_out[b])     # step i-2's output has left d_out[b]
        fa.fused_fp4_attention_into(*d_in[b], d_out[b], ws, stream=s_cp, causal=args.causal)
        ev_cp[b].record(s_cp)
        s_out.wait_event(ev_cp[b])
        with torch.cuda.stream(s_out):
            hO[b].copy_(d_out[b], non_blocking=True)
        ev_out[b].record(s_out)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for s_ in (s_in, s_cp, s_out):
        s_.wait_event(x0)
    for i in range(args.e2e_steps):
        e2e_step(i)
    for s_ in (s_in, s_cp, s_out):
        stream.wait_stream(s_)
    x1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = x0.elapsed_time(x1) / args.e2e_steps
    h2d = sum(t.numel() * t.element_size() for t in (hQ, hK, hV))
    d2h = hO[0].numel() * hO[0].element_size()

    # This rank's share of the box-scale job (512 slices split over the
    # ranks), timed at every N so that one scaling run also gives the
    # strong-scaling curve of that job.
    del d_in, d_out, hQ, hK, hV, hO
    box_ms, box_kern_ms, box_n = (0.0, 0.0, 0) if args.box_steps <= 0 else time_box_share(args, world, rank, dev)

    times = torch.tensor([ms_total, kern_ms, e2e_ms, float(status), box_ms, box_kern_ms, quant_ms, kern_share_ms],
                         dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_total, kern_ms, e2e_ms, status_max, box_ms, box_kern_ms, quant_ms, kern_share_ms = times.tolist()
    ms_step = ms_total / args.steps
    total_flops = flops_rank * world
    value = total_flops / (ms_step * 1e-3) / 1e12
    e2e_value = total_flops / (e2e_ms * 1e-3) / 1e12

    if rank == 0:
        burst, sustained, hbm, peak_src = measured_peaks()
        clocks = sampler.summary(t_wall0, t_wall1)
        basis = peak_basis(ms_total * 1e-3, clocks["reasons"])
        w_shard = wl.Workload(base.name, 1, n, base.seq_q, base.seq_k, base.head_dim)
        peak_burst, peak_sust = mixed_roofline(w_shard, burst), mixed_roofline(w_shard, sustained)
        peak = peak_burst if basis == "burst" else peak_sust
        bf16 = burst if basis == "burst" else sustained
        achieved = flops_rank / (kern_ms * 1e-3) / 1e12
        kernel = "fp4_attention_pair_kernel" if base.head_dim <= 128 else "fp4_attention_fwd_kernel"
        if args.fuse_q:
            kernel += " (Q quantised in the kernel; kernel_ms includes the K pre-pass)"
        traffic = profile_traffic(args.workload, kernel)
        cpu = None
        if not args.no_cpu_baseline and world == 1 and not args.causal:  # the reference has no mask
            ref = CpuReference(base)
            ref.calibrate(10.0)
            r, _ = ref.run(ref.rows)
            cpu = {"value": r, "unit": "TFLOPS", "cores": ref.threads, "kind": ref.kind, "sample": ref.sample()}
        line = {
            "metric": "fused FP4 attention TFLOPS", "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "e2m1 (QK^T) + f16 (PV)",
            "data": "synthetic (seeded N(0,1) FP16 on device)",
            "config": config,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_basis": f"mixed: QK^T at 4x and PV at 1x the {peak_src} {basis} bf16 dense "
                                       f"{bf16:g} TFLOP/s ({basis}: timed region {ms_total * 1e-3:.3g} s, "
                                       f"throttle reasons {clocks['reasons'] or 'none'})",
                         "frac_burst": achieved / peak_burst, "frac_sustained": achieved / peak_sust,
                         "peak_burst": peak_burst, "peak_sustained": peak_sust,
                         "kernel": kernel, "kernel_ms": kern_ms,
                         "kernel_timing": ("CUDA events around the whole fused call" if args.fuse_q else
                                           "CUDA events around the attention launch, in steps interleaved in "
                                           f"{nblk} blocks with the timed ones"),
                         "quantise_ms": None if args.fuse_q else quant_ms,
                         "kernel_share_of_step_ms": None if args.fuse_q else kern_share_ms},
            "frac_of_mixed_roofline_step": value / world / peak,
            "e2e": {"value": e2e_value, "unit": "TFLOPS", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms,
                    "overlap": "H2D, compute and D2H of consecutive steps on three streams, two buffer sets"},
            # per step: one quantise launch (Q and K) + one attention launch, in
            # the timed steps and in the interleaved steps that time the kernel
            "gpu_launches": 4 * args.steps,
            "clocks": clocks,
            "device_status": int(status_max),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if box_n:
            box = wl.WORKLOADS["box_sharded_8k"]
            line["box_8k"] = {
                "job": box.describe(), "slices_per_gpu": box_n, "steps": args.box_steps,
                "ms_per_step": box_ms, "kernel_ms": box_kern_ms,
                "tflops_job": box.flops() / (box_ms * 1e-3) / 1e12,
                "timing": "quantise + attend over this rank's share, CUDA events, max over ranks"}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
