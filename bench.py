"""Benchmark of the B200 attention forward (one JSON line on rank 0).

Metric: attention TFLOP/s, algorithmic FLOPs = 4*Sq*Sk*d per
(batch, head) slice, halved when causal, as a fraction of the dense TF32
roofline.  A step is one forward over one batch of the workload with its
inputs resident in HBM.  Default workload
(32 heads x 4096 x 128, causal), TF32 tensor-core arithmetic, inputs from
BASELINE's generator: numpy default_rng(seed).standard_normal drawn in the
order Q, K, V, times the config's factor, then copied to the device.  Inputs
(268 MB) are larger than the 126 MB L2.  Smaller per-rank inputs (config 1, or
configs 2 and 3 over 4 or 8 GPUs) rotate over copies totalling more than twice
L2, so every step reads its inputs from HBM.

Multi-GPU: launched by torchrun, one process per GPU over NCCL.  The (batch,
head) slices are independent, so the FIXED workload is divided into
contiguous slice ranges, one per rank (strong scaling: 32/N heads per GPU for
config 2), with no data-path collective; the barrier and the max-over-ranks
of the CUDA-event times are the only communication.  Config 5 (one slice)
splits its keys over the ranks instead (fa_b200.kvsplit).

The line also carries: `parity` (rows of the timed output against the CPU
oracle), `precision_3xtf32` (the same workload in the library's default,
error-compensated mode), `e2e` (the crate-API host-slice call on ordinary
pageable buffers; pinned buffers as a sub-field), `roofline` and
`cpu_baseline`.

`--impl reference` times the CPU implementation of the same path (the C
restatement of the crate's v2 forward; the crate itself cannot be built here)
on the host cores, on a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flash-attention-cpu_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

CONFIGS = {
    # name: (bh, sq, sk, d, causal, seed, factor, description)
    "c1": (1, 512, 512, 64, False, 0, 1.0, "1 head x 512 x 64, non-causal"),
    "c2": (32, 4096, 4096, 128, True, 1, 0.5, "32 heads x 4096 x 128, causal prefill"),
    "c3": (256, 1024, 1024, 64, False, 2, 1.0, "16 batch x 16 heads x 1024 x 64, non-causal"),
    "c4": (64, 1, 32768, 128, False, 3, 1.0, "64 heads, Sq=1, Sk=32768, d128 decode"),
    "c5": (1, 131072, 131072, 128, True, 4, 0.3, "1 head x 131072 x 128, causal"),
}
PRECISION_NAMES = {"tf32": 0, "3xtf32": 1, "fp32": 2}


def flops_of(bh, sq, sk, d, causal):
    """Algorithmic FLOPs: 4*Sq*Sk*d per slice, halved when causal."""
    f = 4.0 * sq * sk * d * bh
    return f / 2 if causal else f


def bytes_of(bh, sq, sk, d):
    """Algorithmic bytes: one read of Q, K, V and one write of O (f32)."""
    return 4.0 * bh * (2 * sq * d + 2 * sk * d)


def tensor_peak(peaks, timed_s):
    """Dense TF32 peak (TFLOP/s) for a kernel timed back to back for `timed_s` seconds.

    Dense TF32 on B200 is half the dense bf16 rate.  A region of a second or more runs
    under the 1 kW power cap like the measured sustained GEMM loop, so it is held
    against the sustained figure; shorter regions against the burst figure.
    """
    if not peaks:
        return 1590.0 / 2, "dense TF32 = fallback bf16 1.59 PF/s / 2 (of fallback)"
    if timed_s >= 1.0 and "bf16_tflops_sustained" in peaks:
        return (peaks["bf16_tflops_sustained"] / 2,
                f"dense TF32 = measured bf16 sustained / 2 (timed region {timed_s:.2f} s)")
    return peaks["bf16_tflops"] / 2, f"dense TF32 = measured bf16 burst / 2 (timed region {timed_s:.2f} s)"


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""
    QUERY = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0=None, t1=None):
        """Median SM clock and active throttle reasons of the samples taken
        between wall times t0 and t1 (the timed region); if the region was too
        short to hold a sample, of all samples (warm-up included)."""
        import datetime
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        except OSError:
            pass
        finally:
            if self.path:
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def ts(r):
            try:
                return datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                return None
        window = "timed region"
        if t0 is not None:
            inside = [r for r in rows if ts(r) is not None and t0 <= ts(r) <= t1]
            if inside:
                rows = inside
            else:
                window = "warm-up + timed region (timed region shorter than one sample)"
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "window": window}


_CPU_SAMPLES = {}


def cpu_baseline(cfg, budget_s=12.0):
    """Times the oracle (the crate's v2 forward restated in C, all host cores) on
    whole heads of the workload, as many as fit in ~budget_s.  Returns a dict."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    bh, sq, sk, d, causal, seed, factor, _ = cfg
    cores = os.cpu_count() or 1

    def sample(nh):
        # seeded inputs, generated once per (config, size) and reused by later
        # calls (the reference arm times many short steps)
        key = (cfg, nh)
        if key not in _CPU_SAMPLES:
            rng = np.random.default_rng(seed)
            q = rng.standard_normal(nh * sq * d, dtype=np.float32) * np.float32(factor)
            k = rng.standard_normal(nh * sk * d, dtype=np.float32) * np.float32(factor)
            v = rng.standard_normal(nh * sk * d, dtype=np.float32) * np.float32(factor)
            _CPU_SAMPLES[key] = (q, k, v)
        return _CPU_SAMPLES[key]

    # C5 is one 4.4-TFLOP head: sample its query blocks instead of whole heads.
    if bh == 1 and sq * sk > 1 << 32:
        q, k, v = sample(1)
        n_items = (sq + 63) // 64
        take = max(cores, 64)
        t0 = time.perf_counter()
        O.flash_v2_multihead(q, k, v, 1, sq, sk, d, causal, nthreads=cores, max_items=take)
        dt = time.perf_counter() - t0
        # FLOPs of the first `take` 64-row blocks
        rows = range(min(sq, take * 64))
        fl = 4.0 * d * sum((min(sk, r + 1) if causal else sk) for r in rows)
        return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                "sample": f"first {take} of {n_items} 64-row query blocks of the head "
                          f"({fl / 1e9:.1f} GFLOP) in {dt:.2f} s",
                "tier": O.tier()}
    nh = 1
    if budget_s >= 1.0:  # size the sample by a one-slice probe
        q, k, v = sample(1)
        t0 = time.perf_counter()
        O.flash_v2_multihead(q, k, v, 1, sq, sk, d, causal, nthreads=cores)
        dt1 = time.perf_counter() - t0
        nh = int(max(1, min(bh, budget_s / max(dt1, 1e-6))))
    q, k, v = sample(nh)
    # repeat the sample until about budget_s of CPU time has been measured
    runs, dt = 0, 0.0
    while runs == 0 or (dt < budget_s and runs < 100):
        t0 = time.perf_counter()
        O.flash_v2_multihead(q, k, v, nh, sq, sk, d, causal, nthreads=cores)
        dt += time.perf_counter() - t0
        runs += 1
    fl = flops_of(nh, sq, sk, d, causal) * runs
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{nh} of {bh} slices, {runs} run(s) ({fl / 1e9:.1f} GFLOP) in {dt:.2f} s",
            "tier": O.tier()}


def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


REF_WALL_S = 120.0


def run_reference(args):
    """--impl reference: the CPU implementation of the path, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    bh, sq, sk, d, causal = cfg[:5]
    vals = []
    base = None
    # Each step is a bounded sample and the whole run stays within ~2 minutes:
    # the per-step budget shrinks with the step count, and once REF_WALL_S
    # have passed the remaining steps are not run (every step samples the same
    # workload and the line reports a rate; the steps actually timed are in
    # cpu_baseline).
    # (at least ~1 s per step, so that a step times whole batches of slices at
    # the rate a long run sees: one-slice samples of ~20 ms measured ~20 %
    # slower per FLOP)
    per_step = min(args.ref_budget, max(1.0, 120.0 / (args.warmup + args.steps)))
    t_start = time.perf_counter()
    for i in range(args.warmup + args.steps):
        b = cpu_baseline(cfg, budget_s=per_step)
        if i >= args.warmup:
            vals.append(b["value"])
            base = b
        if len(vals) >= 3 and time.perf_counter() - t_start > REF_WALL_S:
            break
    value = statistics.median(vals)
    base["value"] = value
    base["steps_timed"] = len(vals)
    # the time one whole step of the workload takes at the sampled rate
    full_ms = flops_of(bh, sq, sk, d, causal) / (value * 1e12) * 1e3
    line = {"metric": "attention TFLOP/s", "impl": "reference", "value": value,
            "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": full_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(args, cfg, world=1),
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0, "ms_per_step": full_ms}}
    print(json.dumps(line), flush=True)


def run_kv_split(args, cfg, rank, world, local, dev):
    """Config 5 across `world` GPUs: one 131072-long causal slice whose keys are
    split zig-zag over the ranks, partials merged after one all-to-all (NCCL).
    The total work is fixed, so this is strong scaling."""
    import torch
    import torch.distributed as dist
    import fa_b200
    from fa_b200.kvsplit import kv_split_forward, zigzag_chunks
    if world == 1 and not dist.is_initialized():
        dist.init_process_group("nccl", init_method="tcp://127.0.0.1:29533", rank=0,
                                world_size=1, device_id=dev)
    bh, sq, sk, d, causal, seed, factor, _ = cfg
    hq, hk, hv = seeded_inputs(cfg)
    q = torch.from_numpy(hq).to(dev).view(1, sq, d)
    k_meta = torch.empty(1, sk, d, device="meta")
    chunks = zigzag_chunks(sk, world, rank)
    kc = [torch.from_numpy(hk[c.start * d:c.stop * d]).to(dev).view(1, c.stop - c.start, d)
          for c in chunks]
    vc = [torch.from_numpy(hv[c.start * d:c.stop * d]).to(dev).view(1, c.stop - c.start, d)
          for c in chunks]

    def step():
        return kv_split_forward(q, k_meta, k_meta, causal, k_chunks=kc, v_chunks=vc)

    stream = torch.cuda.current_stream()
    clk = ClockSampler(local).__enter__()
    time.sleep(0.3)
    for _ in range(args.warmup):
        step()
    fa_b200.sync_status(stream)
    dist.barrier()
    torch.cuda.synchronize()
    launches0 = fa_b200.launch_count()
    wall0 = time.time()
    t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0e.record(stream)
    for _ in range(args.steps):
        out, lse, _rows = step()
    t1e.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    time.sleep(0.25)
    clk.__exit__(None, None, None)
    launches = fa_b200.launch_count() - launches0
    t = torch.tensor([t0e.elapsed_time(t1e) / args.steps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    fl = flops_of(1, sq, sk, d, causal)
    value = fl / (step_ms * 1e-3) / 1e12
    # end to end: Q and this rank's K/V chunks from pinned host memory, the
    # owned output rows back to pinned host memory, every step
    hq = torch.empty_like(q, device="cpu").pin_memory()
    hq.copy_(q)
    hk = [x.cpu().pin_memory() for x in kc]
    hv = [x.cpu().pin_memory() for x in vc]
    ho = torch.empty(sq // world, d).pin_memory()
    dist.barrier()
    te0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        q.copy_(hq, non_blocking=True)
        for a, b in zip(kc, hk):
            a.copy_(b, non_blocking=True)
        for a, b in zip(vc, hv):
            a.copy_(b, non_blocking=True)
        out, lse, _rows = step()
        ho.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
    te = torch.tensor([(time.perf_counter() - te0) / args.e2e_steps], device=dev,
                      dtype=torch.float64)
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())
    kv_bytes = sum(4 * 2 * (c.stop - c.start) * d for c in chunks)
    if rank == 0:
        peaks = measured_peaks()
        peak, peak_src = tensor_peak(peaks, step_ms * args.steps * 1e-3)
        peak *= world
        line = {"metric": "attention TFLOP/s", "value": value, "unit": "TFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "tf32", "data": "synthetic",
                "config": dict(config_dict(args, cfg, world),
                               parallelism=f"kv-split over {world} GPUs (zig-zag chunks, "
                                           "one all-to-all of partials, LSE merge)"),
                "clocks": clk.summary(wall0, wall1),
                "e2e": {"value": fl / e2e_s / 1e12, "unit": "TFLOP/s",
                        "h2d_bytes_per_step": 4 * sq * d + kv_bytes,
                        "d2h_bytes_per_step": 4 * (sq // world) * d, "ms_per_step": e2e_s * 1e3,
                        "api": "fa_b200.kvsplit.kv_split_forward"},
                "gpu_launches": launches,
                "roofline": {"bound": "tensor", "achieved": value, "peak": peak,
                             "unit": "TFLOP/s", "frac": value / peak, "traffic": None,
                             "peak_source": f"{world} x " + peak_src}}
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


def run_backward(args, cfg, q, k, v, out, lse, gen, rank, world, local, dev):
    """`--backward`: device time of fa_backward_device on the workload (forward
    output and LSE computed once beforehand).  FLOPs are the five matmuls of the
    gradient (S, dP, dV, dQ, dK: 2.5x the forward's count); both kernel families
    recompute S and dP once more for dQ (seven matmuls executed).  At TF32
    precision the tcgen05 kernels run; otherwise the exact f32 CUDA-core ones."""
    import torch
    import torch.distributed as dist
    import fa_b200
    bh, sq, sk, d, causal, seed, factor, _ = cfg
    nh = q.shape[0]  # this rank's slices of the fixed workload
    steps = args.steps if args.steps <= 200 else 40
    dout = torch.randn(nh, sq, d, device=dev, generator=gen) * factor
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    stream = torch.cuda.current_stream()
    fa_b200.forward_device(q, k, v, out, lse, causal=causal, stream=stream)
    clk = ClockSampler(local).__enter__()
    time.sleep(0.3)
    for _ in range(args.warmup):
        fa_b200.backward_device(q, k, v, out, lse, dout, dq, dk, dv, causal=causal, stream=stream)
    fa_b200.sync_status(stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = fa_b200.launch_count()
    wall0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fa_b200.backward_device(q, k, v, out, lse, dout, dq, dk, dv, causal=causal, stream=stream)
    e1.record()
    torch.cuda.synchronize()
    wall1 = time.time()
    time.sleep(0.25)
    clk.__exit__(None, None, None)
    launches = fa_b200.launch_count() - launches0
    fa_b200.sync_status(stream)
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    step_ms = float(t.item())
    fl = 2.5 * flops_of(bh, sq, sk, d, causal)
    if rank == 0:
        line = {"metric": "attention backward TFLOP/s", "value": fl / step_ms / 1e9,
                "unit": "TFLOP/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
                "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None,
                "dtype": "tf32" if fa_b200.last_path().startswith("tc_") else "f32",
                "data": "synthetic",
                "config": dict(config_dict(args, cfg, world),
                               precision=("tf32 (tcgen05)" if fa_b200.last_path().startswith("tc_")
                                          else "f32 (CUDA cores)")),
                "clocks": clk.summary(wall0, wall1), "gpu_launches": launches,
                "kernel": fa_b200.last_path()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def config_dict(args, cfg, world, h0=None, h1=None):
    bh, sq, sk, d, causal, seed, factor, desc = cfg
    per = f"{h1 - h0}" if h0 is not None else f"{bh}/{world}"
    nh_rank = (h1 - h0) if h0 is not None else max(1, bh // world)
    step_mb = bytes_of(nh_rank, sq, sk, d) / 1e6
    n_rot = rotation_sets(bytes_of(nh_rank, sq, sk, d))
    return {"workload": f"{args.config}: {desc}", "batch_heads": bh,
            "batch_heads_per_gpu": per, "seq_len_q": sq, "seq_len_k": sk, "d_head": d,
            "causal": causal, "seed": seed, "input_scale": factor,
            "generator": "numpy default_rng(seed).standard_normal, Q then K then V, x factor",
            "precision": args.precision,
            "parallelism": f"dp{world} (contiguous (batch, head) slice ranges of the fixed "
                           "workload per GPU, no collective)",
            "host_copy_threads": int(os.environ.get("FA_B200_COPY_THREADS", "0")) or "default",
            "l2": "inputs larger than L2 (no flush)" if n_rot == 1
            else f"each step's inputs ({step_mb:.0f} MB) rotate over {n_rot} copies "
                 f"({n_rot * step_mb:.0f} MB > 2x L2), so every step reads them from HBM"}


L2_BYTES = 126e6


def rotation_sets(step_bytes):
    """How many copies of a step's inputs the timed loop rotates over: one when
    they are larger than L2, else enough for more than twice L2 (at most 512)."""
    if step_bytes > L2_BYTES:
        return 1
    return int(min(512, -(-2 * L2_BYTES // step_bytes)))


def shard_range(bh, world, rank):
    """Contiguous (batch, head) slice range [h0, h1) of `rank` out of `world`."""
    return bh * rank // world, bh * (rank + 1) // world


def seeded_inputs(cfg, h0=0, h1=None):
    """Q, K, V of a config as flat float32 arrays, slices [h0, h1) only: the
    whole config is drawn from BASELINE's generator (so every rank sees the same
    numbers) and this rank's slices are cut out."""
    import numpy as np
    bh, sq, sk, d, causal, seed, factor, _ = cfg
    h1 = bh if h1 is None else h1
    rng = np.random.default_rng(seed)
    out = []
    for n in (sq, sk, sk):
        a = rng.standard_normal(bh * n * d, dtype=np.float32) * np.float32(factor)
        out.append(np.ascontiguousarray(a[h0 * n * d:h1 * n * d]))
    return out


def parity_items(nh, sq, block=64):
    """(head, 64-row query block) items of the oracle spread over nh slices:
    first, middle and last blocks of the first and last slice."""
    nb = (sq + block - 1) // block
    pick = sorted({0, nb // 2, nb - 1})
    return sorted({h * nb + b for h in {0, nh - 1} for b in pick})


def parity_check(q, k, v, out, lse, nh, sq, sk, d, causal, tol, h0=0):
    """Max abs error of sampled output rows and their LSE against the oracle
    (the crate's v2 forward restated in C), on whole query blocks of run_v2."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    items = parity_items(nh, sq)
    want, wlse = O.flash_v2_items(q, k, v, nh, sq, sk, d, causal, items)
    rows = O.item_rows(items, sq)
    err = float(np.max(np.abs(out.reshape(-1, d)[rows].astype(np.float64) -
                              want.reshape(-1, d)[rows])))
    lerr = float(np.max(np.abs(lse[rows].astype(np.float64) - wlse[rows])))
    return {"max_abs_err": err, "lse_max_abs_err": lerr, "tol": tol,
            "pass": bool(err <= tol and lerr <= tol), "rows_checked": int(len(rows)),
            "oracle": "oracle/fa_oracle.c (crate v2 forward restated), whole 64-row query "
                      f"blocks {items} of slices [{h0}, {h0 + nh})"}


def time_device(fa_b200, step, steps, stream, world):
    """Device time per step (CUDA events on the launching stream; max over
    ranks), and kernels launched per step."""
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = fa_b200.launch_count()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    launches = fa_b200.launch_count() - launches0
    fa_b200.sync_status(stream)
    t = torch.tensor([t0.elapsed_time(t1) / steps], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), launches


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=6000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--precision", default="tf32", choices=sorted(PRECISION_NAMES))
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the parity check, the 3xTF32 leg and the e2e legs (profiling)")
    ap.add_argument("--ref-budget", type=float, default=8.0)
    ap.add_argument("--kv-split", action="store_true",
                    help="config 5 through the key-range split even on one GPU")
    ap.add_argument("--bh", type=int, default=0,
                    help="override the slice count (smaller cases for profiler captures)")
    ap.add_argument("--backward", action="store_true",
                    help="time the backward pass (dQ, dK, dV) of the workload instead")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    args.e2e_steps = max(1, args.e2e_steps)
    if args.impl == "reference":
        return run_reference(args)

    # One process per GPU shares the host: each rank's copy pool (the staged
    # host-slice calls) gets its share of the cores.
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    if world_env > 1 and "FA_B200_COPY_THREADS" not in os.environ:
        try:
            cores = len(os.sched_getaffinity(0))  # the CPUs this process may run on
        except AttributeError:
            cores = os.cpu_count() or 16
        os.environ["FA_B200_COPY_THREADS"] = str(max(2, min(16, cores // world_env)))
    import numpy as np
    import torch
    import torch.distributed as dist
    import fa_b200

    rank, world, local = dist_setup(args.gpus)
    fa_b200.set_device(torch.cuda.current_device())
    fa_b200.set_precision(PRECISION_NAMES[args.precision])
    cfg = CONFIGS[args.config]
    if args.bh > 0:
        cfg = (args.bh,) + cfg[1:]
    bh, sq, sk, d, causal, seed, factor, _ = cfg
    dev = torch.device("cuda", torch.cuda.current_device())
    if args.config == "c5" and (world > 1 or args.kv_split):
        return run_kv_split(args, cfg, rank, world, local, dev)

    # this rank's contiguous slice range of the fixed workload
    h0, h1 = shard_range(bh, world, rank)
    nh = h1 - h0
    hq, hk, hv = seeded_inputs(cfg, h0, h1)
    q = torch.from_numpy(hq).to(dev).view(nh, sq, d)
    k = torch.from_numpy(hk).to(dev).view(nh, sk, d)
    v = torch.from_numpy(hv).to(dev).view(nh, sk, d)
    out = torch.empty_like(q)
    lse = torch.empty(nh, sq, device=dev)
    if args.backward:
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed * 1000 + rank)
        return run_backward(args, cfg, q, k, v, out, lse, gen, rank, world, local, dev)
    # Inputs smaller than L2 (126 MB): the step rotates over copies of them
    # whose total is more than twice L2, so each step's Q/K/V come from HBM as
    # in a pipeline of different layers' data, and steps run back to back.
    n_sets = rotation_sets(bytes_of(nh, sq, sk, d))
    sets = [(q, k, v, out, lse)] + [
        (q.clone(), k.clone(), v.clone(), torch.empty_like(out), torch.empty_like(lse))
        for _ in range(n_sets - 1)]
    stream = torch.cuda.current_stream()
    it_box = [0]

    def step():
        qs, ks, vs, os_, ls = sets[it_box[0] % n_sets]
        it_box[0] += 1
        fa_b200.forward_device(qs, ks, vs, os_, ls, causal=causal, stream=stream)

    clk = ClockSampler(local).__enter__()
    time.sleep(0.3)  # let nvidia-smi take its first sample
    for _ in range(args.warmup):
        step()
    fa_b200.sync_status(stream)

    # device-timed region: every launch of the step on `stream`
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = fa_b200.launch_count()
    wall0 = time.time()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        step()
    t_end.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    time.sleep(0.25)
    clk.__exit__(None, None, None)
    launches = fa_b200.launch_count() - launches0
    fa_b200.sync_status(stream)
    path = fa_b200.last_path()
    step_ms = t_start.elapsed_time(t_end) / args.steps
    # the parity check below reads set 0's output: recompute it
    fa_b200.forward_device(q, k, v, out, lse, causal=causal, stream=stream)
    torch.cuda.synchronize()
    t = torch.tensor([step_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    step_ms = float(t.item())
    fl_all = flops_of(bh, sq, sk, d, causal)   # the whole job (all ranks)
    fl_rank = flops_of(nh, sq, sk, d, causal)  # this rank's share
    value = fl_all / (step_ms * 1e-3) / 1e12
    clocks = clk.summary(wall0, wall1)
    tol_main = 2e-3 if args.precision == "tf32" else 2e-5

    parity = None
    extra = {}
    if not args.no_extras:
        # parity of the timed output (its last step) against the oracle
        o_h = out.cpu().numpy().ravel()
        l_h = lse.cpu().numpy().ravel()
        if not path.startswith(("tcgen05", "simt")):
            tol_main = 2e-5  # the exact-f32 decode path
        parity = parity_check(hq, hk, hv, o_h, l_h, nh, sq, sk, d, causal, tol_main, h0)
        # the library's default precision (error-compensated 3xTF32) on the same inputs
        if args.precision == "tf32" and path.startswith("tcgen05"):
            fa_b200.set_precision(fa_b200.PREC_3XTF32)
            for _ in range(3):
                step()
            steps3 = max(20, min(args.steps // 3, 2000))
            ms3, l3 = time_device(fa_b200, step, steps3, stream, world)
            path3 = fa_b200.last_path()
            fa_b200.forward_device(q, k, v, out, lse, causal=causal, stream=stream)  # set 0
            torch.cuda.synchronize()
            p3 = parity_check(hq, hk, hv, out.cpu().numpy().ravel(), lse.cpu().numpy().ravel(),
                              nh, sq, sk, d, causal, 2e-5, h0)
            fa_b200.set_precision(PRECISION_NAMES[args.precision])
            v3 = fl_all / (ms3 * 1e-3) / 1e12
            extra["precision_3xtf32"] = {
                "value": v3, "unit": "TFLOP/s", "ms_per_step": ms3, "steps": steps3,
                "kernel": path3, "launches_per_step": l3 / steps3,
                "note": "attention TFLOP/s; the tensor pipe executes 3x these FLOPs "
                        "(hi*hi + hi*lo + lo*hi)",
                "parity": p3}
        # the backward pass (dQ, dK, dV; beyond the crate) on the same inputs,
        # at TF32 (the tcgen05 kernels); its parity is in tests/test_backward.py
        if args.precision == "tf32" and path.startswith("tcgen05") and d in (32, 64, 96, 128):
            gen_b = np.random.default_rng(cfg[5] + 1000)
            dout_b = torch.from_numpy(
                gen_b.standard_normal(nh * sq * d, dtype=np.float32)).to(dev).view(nh, sq, d)
            grads = [torch.empty_like(t) for t in (q, k, v)]

            def bstep():
                fa_b200.backward_device(q, k, v, out, lse, dout_b, *grads, causal=causal,
                                        stream=stream)
            for _ in range(3):
                bstep()
            steps_b = max(10, min(args.steps // 20, 200))
            ms_b, l_b = time_device(fa_b200, bstep, steps_b, stream, world)
            vb = 2.5 * fl_all / (ms_b * 1e-3) / 1e12
            pk_b, pk_src_b = tensor_peak(measured_peaks(), ms_b * steps_b * 1e-3)
            pk_b *= world
            extra["backward"] = {
                "value": vb, "unit": "TFLOP/s",
                "ms_per_step": ms_b, "steps": steps_b, "kernel": fa_b200.last_path(),
                "launches_per_step": l_b / steps_b,
                "note": "gradient FLOPs (5 matmuls, 2.5x the forward); 7 executed",
                "roofline": {"bound": "tensor", "achieved": vb, "peak": pk_b, "unit": "TFLOP/s",
                             "frac": vb / pk_b, "frac_executed": 1.4 * vb / pk_b,
                             "peak_source": pk_src_b},
                "parity": "tests/test_backward.py (f64 oracle, 2e-3 relative at TF32)"}
            del grads, dout_b

    # end-to-end through the crate API (host slices, synchronous): the call a
    # crate user makes, on this rank's slices; copies inside the timed region
    e2e = None
    if not args.no_extras:
        cfgc = fa_b200.FlashAttentionConfig(64, 128, causal)
        po = np.empty(nh * sq * d, np.float32)

        def timed_call(qa, ka, va, oa):
            fa_b200.flash_attention_multihead_v2(qa, ka, va, 1, nh, sq, sk, d, cfgc, oa)
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            for _ in range(args.e2e_steps):
                fa_b200.flash_attention_multihead_v2(qa, ka, va, 1, nh, sq, sk, d, cfgc, oa)
            te = torch.tensor([(time.perf_counter() - t0) / args.e2e_steps], device=dev,
                              dtype=torch.float64)
            if world > 1:
                dist.all_reduce(te, op=dist.ReduceOp.MAX)
            return float(te.item())

        # ordinary pageable buffers: what a caller of the crate API passes
        pg_s = timed_call(hq, hk, hv, po)
        # pinned buffers (fa_pin_host): the host-link floor
        pq = torch.empty(nh * sq * d, dtype=torch.float32, pin_memory=True)
        pk = torch.empty(nh * sk * d, dtype=torch.float32, pin_memory=True)
        pv = torch.empty(nh * sk * d, dtype=torch.float32, pin_memory=True)
        pout = torch.empty(nh * sq * d, dtype=torch.float32, pin_memory=True)
        pq.numpy()[:] = hq
        pk.numpy()[:] = hk
        pv.numpy()[:] = hv
        pin_s = timed_call(pq.numpy(), pk.numpy(), pv.numpy(), pout.numpy())
        e2e = {"value": fl_all / pg_s / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 4 * (bh * sq * d + 2 * bh * sk * d),
               "d2h_bytes_per_step": 4 * bh * sq * d, "ms_per_step": pg_s * 1e3,
               "api": "fa_flash_attention_multihead_v2 (host slices, synchronous) on "
                      "pageable numpy buffers, each rank its slice range",
               "pinned": {"value": fl_all / pin_s / 1e12, "ms_per_step": pin_s * 1e3,
                          "note": "same call on page-locked host buffers"}}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks = measured_peaks()
    if path.startswith("decode"):
        bound, unit = "hbm", "GB/s"
        achieved = bytes_of(nh, sq, sk, d) / (step_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"] if peaks else 6650.0
        peak_src = "measured hbm_gbs (of measured)" if peaks else "fallback 6.65 TB/s (of fallback)"
    else:
        bound, unit = "tensor", "TFLOP/s"
        achieved = fl_rank / (step_ms * 1e-3) / 1e12
        peak, peak_src = tensor_peak(peaks, step_ms * args.steps * 1e-3)
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            tr = json.load(f).get(f"{args.config}/{args.precision}")
            if tr and world == 1:
                traffic = tr["bytes_per_launch"]
    except OSError:
        pass
    roof = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
            "kernel": path, "launches_per_step": launches / args.steps,
            "per": "rank 0's launch (its slice range), device time"}
    line = {"metric": "attention TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "tf32" if args.precision == "tf32" and not path.startswith(("decode", "simt"))
            else ("3xtf32" if args.precision == "3xtf32" and path.startswith("tcgen05") else "f32"),
            "data": "synthetic (BASELINE generator)",
            "config": config_dict(args, cfg, world, h0, h1),
            "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "roofline": roof,
            "parity": parity}
    line.update(extra)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
