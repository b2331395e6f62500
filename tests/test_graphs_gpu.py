"""The device entry points under CUDA graph capture.

A caller that launches many short attention calls (decode steps, prefill
chunks) captures them once in a CUDA graph and replays the graph, which takes
the host's per-call launch work out of the loop.  Every device path is
capturable: the split workspaces come from cudaMallocAsync / cudaFreeAsync on
the caller's stream (graph allocation nodes), the tensor maps are kernel
parameters, and nothing synchronises.  A replay must give exactly the eager
call's result on the same inputs, and the oracle's on new inputs copied into
the captured buffers.
"""
import numpy as np
import pytest

import oracle as O
from fa_cases import max_abs_diff, random_vec

pytestmark = pytest.mark.gpu

TOL = {0: 2e-3, 1: 2e-5, 2: 2e-5}

# (bh, sq, sk, d, causal, precision): the pair kernel with and without
# key-range parts, the single-CTA kernel with parts, split-KV decode, the
# 3xTF32 pair kernel with and without parts (its split_lo prepass included),
# the single-CTA kernels at d = 32 and 96, and the CUDA-core f32 kernel.
CASES = [
    (2, 512, 512, 128, True, 0),
    (1, 1024, 4096, 128, False, 0),
    (1, 100, 8192, 128, False, 0),
    (4, 1, 8192, 128, False, 0),
    (1, 512, 4096, 64, True, 1),
    (12, 1024, 1024, 128, True, 1),
    (2, 300, 700, 96, False, 1),
    (2, 300, 300, 32, True, 0),
    (2, 200, 300, 96, True, 2),
]


@pytest.fixture
def fa(gpu_lib):
    old = gpu_lib.get_precision()
    yield gpu_lib
    gpu_lib.set_precision(old)


def _inputs(bh, sq, sk, d, seed):
    return (random_vec(bh * sq * d, seed), random_vec(bh * sk * d, seed + 1),
            random_vec(bh * sk * d, seed + 2))


@pytest.mark.parametrize("case", CASES)
def test_forward_replay_matches_eager_and_oracle(fa, case):
    import torch
    bh, sq, sk, d, causal, prec = case
    fa.set_precision(prec)
    q, k, v = _inputs(bh, sq, sk, d, 300)
    dq = torch.from_numpy(q).cuda().view(bh, sq, d)
    dk = torch.from_numpy(k).cuda().view(bh, sk, d)
    dv = torch.from_numpy(v).cuda().view(bh, sk, d)
    out = torch.full((bh, sq, d), float("nan"), device="cuda")
    lse = torch.full((bh, sq), float("nan"), device="cuda")

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # eager warm-up: attributes, device state
        fa.forward_device(dq, dk, dv, out, lse, causal=causal)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    eager_o, eager_l = out.clone(), lse.clone()

    g = torch.cuda.CUDAGraph()
    out.fill_(float("nan"))
    lse.fill_(float("nan"))
    with torch.cuda.graph(g):
        fa.forward_device(dq, dk, dv, out, lse, causal=causal)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager_o) and torch.equal(lse, eager_l)

    q2, k2, v2 = _inputs(bh, sq, sk, d, 400)
    for dst, src in ((dq, q2), (dk, k2), (dv, v2)):
        dst.view(-1).copy_(torch.from_numpy(src))
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    want, wlse, _ = O.flash_v2_multihead(q2, k2, v2, bh, sq, sk, d, causal)
    assert max_abs_diff(out.cpu().numpy().ravel(), want) < TOL[prec]
    assert max_abs_diff(lse.cpu().numpy().ravel(), wlse) < TOL[prec]


def test_many_calls_in_one_graph(fa):
    # A decode-like loop: 16 calls over different key lengths captured once.
    import torch
    fa.set_precision(0)
    bh, d, sk_max = 2, 128, 4096
    q, k, v = _inputs(bh, 1, sk_max, d, 500)
    dq = torch.from_numpy(q).cuda().view(bh, 1, d)
    dk = torch.from_numpy(k).cuda().view(bh, sk_max, d)
    dv = torch.from_numpy(v).cuda().view(bh, sk_max, d)
    lens = [256 * (i + 1) for i in range(16)]
    keys = [dk[:, :n].contiguous() for n in lens]
    vals = [dv[:, :n].contiguous() for n in lens]
    outs = [torch.empty(bh, 1, d, device="cuda") for _ in lens]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for kk, vv, oo in zip(keys, vals, outs):
            fa.forward_device(dq, kk, vv, oo)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for kk, vv, oo in zip(keys, vals, outs):
            fa.forward_device(dq, kk, vv, oo)
    for oo in outs:
        oo.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    for n, kk, vv, oo in zip(lens, keys, vals, outs):
        want, _, _ = O.flash_v2_multihead(q, kk.cpu().numpy().ravel(), vv.cpu().numpy().ravel(),
                                          bh, 1, n, d, False)
        assert max_abs_diff(oo.cpu().numpy().ravel(), want) < TOL[0]


@pytest.mark.parametrize("prec", [1, 0])  # CUDA-core and tensor-core backward
def test_backward_replay_matches_eager(fa, prec):
    import torch
    bh, sq, sk, d = 2, 192, 256, 64
    q, k, v = _inputs(bh, sq, sk, d, 600)
    dq_in = torch.from_numpy(q).cuda().view(bh, sq, d)
    dk_in = torch.from_numpy(k).cuda().view(bh, sk, d)
    dv_in = torch.from_numpy(v).cuda().view(bh, sk, d)
    dout = torch.from_numpy(random_vec(bh * sq * d, 603)).cuda().view(bh, sq, d)
    o = torch.empty(bh, sq, d, device="cuda")
    lse = torch.empty(bh, sq, device="cuda")
    grads = [torch.empty_like(t) for t in (dq_in, dk_in, dv_in)]
    fa.set_precision(prec)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fa.forward_device(dq_in, dk_in, dv_in, o, lse, causal=True)
        fa.backward_device(dq_in, dk_in, dv_in, o, lse, dout, *grads, causal=True)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    eager = [t.clone() for t in grads]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fa.forward_device(dq_in, dk_in, dv_in, o, lse, causal=True)
        fa.backward_device(dq_in, dk_in, dv_in, o, lse, dout, *grads, causal=True)
    for t in grads:
        t.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(grads, eager):
        assert torch.equal(a, b)
