"""Quick timing of the crate-API variants on this library, for a regression history.

The counterpart of the crate's ``examples/bench_quick.rs``: the same shapes
((256, 64), (512, 64), (1024, 64), (2048, 64), (1024, 128)), the same
variants (v1, v2, v3, non-causal and causal, through the host-slice calls),
one untimed warm-up call, then the median over 20-30 calls (the crate takes
the mean of 3-10 calls; GPU calls this short need more to be stable).  On the GPU the
three variants run the same kernels, so their rows differ only by noise; the
``device`` variant times the same work through ``fa_forward_device`` on
resident tensors (no PCIe), which is what the kernels alone cost.  The crate's
``naive`` row has no counterpart here: naive attention is the crate's CPU code.

    python -m fa_b200.bench_quick            # table
    python -m fa_b200.bench_quick --csv      # CSV rows for benches/history.csv

CSV schema (one header line, then one row per measurement)::

    timestamp,commit,os,arch,device,gpus,precision,variant,causal,seq_len,d_head,time_ms

Every column except ``timestamp`` and ``time_ms`` is part of the comparison
key used by ``fa_b200.bench_compare``, so rows from different devices, GPU
counts or precisions are never compared with each other.
"""
from __future__ import annotations

import os
import platform
import subprocess
import sys
import time

HEADER = ("timestamp,commit,os,arch,device,gpus,precision,variant,causal,seq_len,d_head,"
          "time_ms")
SHAPES = [(256, 64), (512, 64), (1024, 64), (2048, 64), (1024, 128)]
VARIANTS = ("v1", "v2", "v3")
PRECISIONS = {0: "tf32", 1: "3xtf32", 2: "fp32"}


def resolve_commit() -> str:
    """``BENCH_COMMIT`` if set, else ``git rev-parse --short HEAD``, else "unknown"."""
    c = os.environ.get("BENCH_COMMIT")
    if c:
        return c
    try:
        r = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True,
                           text=True, timeout=10)
        if r.returncode == 0 and r.stdout.strip():
            return r.stdout.strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return "unknown"


def random_vec(n: int, seed: int):
    import numpy as np
    return np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32)


def time_it(fn, iters: int) -> float:
    """Median seconds per call over `iters` timed calls after one warm-up call.
    (The median, since single calls of a few hundred microseconds see
    scheduling noise that a mean over a handful of calls would keep.)"""
    fn()  # warm-up (first-touch, caches) outside the timed loop
    ts = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    ts.sort()
    return ts[len(ts) // 2]


def measure(fa, iters_small: int = 30, iters_large: int = 20):
    """Rows (variant, causal, seq_len, d_head, time_ms) for the current precision."""
    import numpy as np
    import torch
    rows = []
    fns = {"v1": fa.flash_attention_v1, "v2": fa.flash_attention_v2,
           "v3": fa.flash_attention_v3}
    for s, d in SHAPES:
        q, k, v = random_vec(s * d, 1), random_vec(s * d, 2), random_vec(s * d, 3)
        out = np.zeros(s * d, np.float32)
        iters = iters_small if s <= 512 else iters_large
        dq, dk, dv = (torch.from_numpy(x).cuda().view(1, s, d) for x in (q, k, v))
        dout = torch.empty_like(dq)
        for causal in (False, True):
            cfg = fa.FlashAttentionConfig(64, 128, causal)
            for name in VARIANTS:
                t = time_it(lambda: fns[name](q, k, v, s, s, d, cfg, out), iters)
                rows.append((name, causal, s, d, t * 1e3))

            def dev_call():
                fa.forward_device(dq, dk, dv, dout, None, causal=causal)
                torch.cuda.synchronize()
            t = time_it(dev_call, max(iters, 20))
            rows.append(("device", causal, s, d, t * 1e3))
    return rows


def csv_lines(rows, commit: str, device: str, gpus: int, precision: str, timestamp: int):
    out = [HEADER]
    osn, arch = sys.platform, platform.machine()
    for variant, causal, s, d, ms in rows:
        out.append(f"{timestamp},{commit},{osn},{arch},{device},{gpus},{precision},{variant},"
                   f"{str(causal).lower()},{s},{d},{ms:.4f}")
    return out


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    csv_mode = "--csv" in argv
    import torch
    import fa_b200 as fa
    prec = fa.get_precision()
    rows = measure(fa)
    if csv_mode:
        dev = torch.cuda.get_device_name().replace(",", " ")
        for line in csv_lines(rows, resolve_commit(), dev, 1, PRECISIONS.get(prec, str(prec)),
                              int(time.time())):
            print(line)
        return 0
    print(f"precision {PRECISIONS.get(prec, prec)}  (ms per call; v1/v2/v3 through host "
          "slices, device = resident tensors)")
    print(f"{'seq':>7} {'d':>5} | {'v1_ms':>8} {'v2_ms':>8} {'v3_ms':>8} {'dev_ms':>8} | "
          f"{'v1c_ms':>8} {'v2c_ms':>8} {'v3c_ms':>8} {'devc_ms':>8}")
    by = {(r[0], r[1], r[2], r[3]): r[4] for r in rows}
    for s, d in SHAPES:
        a = [by[(n, False, s, d)] for n in VARIANTS + ("device",)]
        b = [by[(n, True, s, d)] for n in VARIANTS + ("device",)]
        print(f"{s:>7} {d:>5} | " + " ".join(f"{x:>8.3f}" for x in a) + " | " +
              " ".join(f"{x:>8.3f}" for x in b))
    return 0


if __name__ == "__main__":
    sys.exit(main())
