"""The bounded-wait failure path of the tensor-core kernels, made to happen.

Every mbarrier wait in the tcgen05 kernels has a time limit; when one runs out
the CTA raises its abort flag and the device error word, every role leaves its
loop, copies and MMAs in flight are drained, tensor memory is freed, and the
call reports FA_ERR_TIMEOUT.  The test hook fa_test_stall makes one softmax
warp withhold its "P ready" arrive on one key block (a software arrive only:
no copy or MMA completion is skipped) and shortens the limit to 20 ms, so the
MMA issuer's wait for P runs out.  The GPU context must stay usable: a normal
call right after gives the oracle's result.
"""
import numpy as np
import pytest

import oracle as O
from fa_cases import max_abs_diff, random_vec

pytestmark = pytest.mark.gpu

TOL = {0: 2e-3, 1: 2e-5}


@pytest.fixture
def fa(gpu_lib):
    old = gpu_lib.get_precision()
    yield gpu_lib
    gpu_lib.test_stall(-1)
    gpu_lib.set_precision(old)


@pytest.mark.parametrize("prec,shape,kernel", [
    (0, (1, 100, 1000, 128, False), "single CTA, TF32"),
    (0, (2, 512, 1024, 128, True), "CTA pair, TF32, d 128"),
    (0, (2, 512, 1024, 64, False), "CTA pair, TF32, d 64"),
    (1, (1, 100, 1000, 128, False), "3xTF32, single CTA"),
    (1, (2, 512, 1024, 128, True), "3xTF32, CTA pair"),
])
def test_withheld_arrive_times_out_and_the_gpu_recovers(fa, prec, shape, kernel):
    bh, sq, sk, d, causal = shape
    fa.set_precision(prec)
    q, k, v = random_vec(bh * sq * d, 1), random_vec(bh * sk * d, 2), random_vec(bh * sk * d, 3)
    fa.test_stall(0, 20_000_000)
    try:
        with pytest.raises(fa.FaError, match="FA_ERR_TIMEOUT"):
            fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    finally:
        fa.test_stall(-1)
    # the error word was cleared by the failed call: the next call runs in full
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    assert fa.last_path() == ("tcgen05_tf32" if prec == 0 else "tcgen05_3xtf32"), kernel
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    assert max_abs_diff(out, want) < TOL[prec]
    assert max_abs_diff(lse, wlse) < TOL[prec]


def test_device_call_reports_the_timeout_through_sync_status(fa):
    import torch
    fa.set_precision(0)
    bh, sq, sk, d = 2, 512, 1024, 128
    q, k, v = (torch.from_numpy(random_vec(bh * n * d, s)).cuda().view(bh, n, d)
               for n, s in ((sq, 4), (sk, 5), (sk, 6)))
    out = torch.empty(bh, sq, d, device="cuda")
    fa.test_stall(0, 20_000_000)
    try:
        fa.forward_device(q, k, v, out, None, causal=True)
        with pytest.raises(fa.FaError, match="FA_ERR_TIMEOUT"):
            fa.sync_status()
    finally:
        fa.test_stall(-1)
    fa.sync_status()  # cleared
    fa.forward_device(q, k, v, out, None, causal=True)
    fa.sync_status()
    want, _, _ = O.flash_v2_multihead(q.cpu().numpy().ravel(), k.cpu().numpy().ravel(),
                                      v.cpu().numpy().ravel(), bh, sq, sk, d, True)
    assert max_abs_diff(out.cpu().numpy().ravel(), want) < 2e-3


@pytest.mark.parametrize("d", [64, 128])
def test_backward_withheld_arrive_times_out_and_the_gpu_recovers(fa, d):
    # The tensor-core backward: a softmax thread of the first dK/dV CTA
    # withholds its "P ready" arrive on query block 0, the MMA issuer's wait
    # for it runs out, and the host call reports FA_ERR_TIMEOUT; the next call
    # gives the oracle's gradients.
    bh, sq, sk = 2, 300, 400
    q, k, v = random_vec(bh * sq * d, 31), random_vec(bh * sk * d, 32), random_vec(bh * sk * d, 33)
    dout = random_vec(bh * sq * d, 34)
    fa.set_precision(fa.PREC_FP32)
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, True)
    fa.set_precision(fa.PREC_TF32)
    fa.test_stall(0, 20_000_000)
    try:
        with pytest.raises(fa.FaError, match="FA_ERR_TIMEOUT"):
            fa.flash_attention_backward(q, k, v, out, lse, dout, bh, sq, sk, d, True)
    finally:
        fa.test_stall(-1)
    dq, dk, dv = fa.flash_attention_backward(q, k, v, out, lse, dout, bh, sq, sk, d, True)
    assert fa.last_path() == "tc_tf32_backward"
    for h in range(bh):
        sl_q, sl_k = slice(h * sq * d, (h + 1) * sq * d), slice(h * sk * d, (h + 1) * sk * d)
        rq, rk, rv = O.attention_backward_f64(q[sl_q], k[sl_k], v[sl_k], dout[sl_q], sq, sk, d, True)
        for g, r in ((dq[sl_q], rq), (dk[sl_k], rk), (dv[sl_k], rv)):
            assert np.max(np.abs(g - r)) < 2e-3 * (1.0 + np.max(np.abs(r)))
