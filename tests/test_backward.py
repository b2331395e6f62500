"""Backward pass (gradients of the forward; the crate itself is forward-only).

Parity oracle: oracle.attention_backward_f64, the f64 calculus of the crate's
forward (parity unpinned against the reference, which has no backward).  The
oracle is first checked here against central finite differences of an f64
forward, then the GPU kernels against the oracle."""
import numpy as np
import pytest

import oracle as O
from fa_cases import random_vec


def forward_f64(q, k, v, sq, sk, d, causal):
    Q, K, V = (np.asarray(x, np.float64).reshape(n, d) for x, n in ((q, sq), (k, sk), (v, sk)))
    S = (Q @ K.T) * float(1.0 / np.sqrt(np.float32(d)))
    if causal:
        S = np.where(np.arange(sk)[None, :] <= np.arange(sq)[:, None], S, -np.inf)
    m = S.max(axis=1, keepdims=True)
    E = np.exp(S - np.where(np.isfinite(m), m, 0.0))
    l = E.sum(axis=1, keepdims=True)
    return (np.where(l > 0, E / np.where(l > 0, l, 1.0), 0.0) @ V).ravel()


@pytest.mark.parametrize("sq,sk,d,causal", [(3, 4, 2, False), (4, 3, 3, True), (5, 5, 4, True)])
def test_oracle_backward_matches_finite_differences(sq, sk, d, causal):
    rng = np.random.default_rng(sq * 100 + sk * 10 + d)
    q, k, v = (rng.uniform(-1, 1, n) for n in (sq * d, sk * d, sk * d))
    dout = rng.uniform(-1, 1, sq * d)
    dq, dk, dv = O.attention_backward_f64(q, k, v, dout, sq, sk, d, causal)
    h = 1e-6
    for x, g in ((q, dq), (k, dk), (v, dv)):
        num = np.zeros_like(x)
        for i in range(x.size):
            xp, xm = x.copy(), x.copy()
            xp[i] += h
            xm[i] -= h
            args = [q, k, v]
            idx = 0 if x is q else (1 if x is k else 2)
            args[idx] = xp
            fp = forward_f64(*args, sq, sk, d, causal) @ dout
            args[idx] = xm
            fm = forward_f64(*args, sq, sk, d, causal) @ dout
            num[i] = (fp - fm) / (2 * h)
        assert np.max(np.abs(num - g)) < 1e-7


def test_backward_host_api_checks_shapes():
    import fa_b200
    q = random_vec(4 * 8, 1)
    with pytest.raises(fa_b200.Panic, match="k shape mismatch"):
        fa_b200.flash_attention_backward(q, q[:-1], q, q, np.zeros(4, np.float32), q, 1, 4, 4, 8)


BWD_CASES = [(1, 1, 4, False), (37, 50, 16, True), (64, 64, 64, False), (100, 300, 128, True),
             (300, 100, 128, True), (129, 257, 32, False), (65, 65, 7, True),
             (200, 200, 96, False), (33, 17, 128, True)]


@pytest.mark.gpu
@pytest.mark.parametrize("sq,sk,d,causal", BWD_CASES)
def test_backward_matches_f64_oracle(gpu_lib, sq, sk, d, causal):
    fa = gpu_lib
    old = fa.get_precision()
    fa.set_precision(fa.PREC_FP32)  # exact forward, so O and LSE match the oracle's P
    try:
        q, k, v = random_vec(sq * d, 11), random_vec(sk * d, 12), random_vec(sk * d, 13)
        dout = random_vec(sq * d, 14)
        out, lse = fa.multihead_lse(q, k, v, 1, sq, sk, d, causal)
        dq, dk, dv = fa.flash_attention_backward(q, k, v, out, lse, dout, 1, sq, sk, d, causal)
    finally:
        fa.set_precision(old)
    rq, rk, rv = O.attention_backward_f64(q, k, v, dout, sq, sk, d, causal)
    for g, r in ((dq, rq), (dk, rk), (dv, rv)):
        assert np.all(np.isfinite(g))
        assert np.max(np.abs(g - r)) < 2e-5 * (1.0 + np.max(np.abs(r)))


@pytest.mark.gpu
def test_backward_device_api_multihead_matches_host_api(gpu_lib):
    import torch
    fa = gpu_lib
    bh, sq, sk, d = 3, 150, 200, 64
    old = fa.get_precision()
    fa.set_precision(fa.PREC_FP32)
    try:
        q, k, v = random_vec(bh * sq * d, 21), random_vec(bh * sk * d, 22), random_vec(bh * sk * d, 23)
        dout = random_vec(bh * sq * d, 24)
        out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, True)
        hq, hk, hv = fa.flash_attention_backward(q, k, v, out, lse, dout, bh, sq, sk, d, True)
        t = lambda x, n: torch.from_numpy(np.ascontiguousarray(x)).cuda().view(bh, n, -1)
        dq, dk, dv = (torch.empty(bh, n, d, device="cuda") for n in (sq, sk, sk))
        fa.backward_device(t(q, sq), t(k, sk), t(v, sk), t(out, sq),
                           torch.from_numpy(lse).cuda().view(bh, sq), t(dout, sq), dq, dk, dv,
                           causal=True)
        fa.sync_status()
        assert fa.last_path() == "simt_backward"
    finally:
        fa.set_precision(old)
    assert np.array_equal(dq.cpu().numpy().ravel(), hq)
    assert np.array_equal(dk.cpu().numpy().ravel(), hk)
    assert np.array_equal(dv.cpu().numpy().ravel(), hv)
    for h in range(bh):
        sl_q, sl_k = slice(h * sq * d, (h + 1) * sq * d), slice(h * sk * d, (h + 1) * sk * d)
        rq, rk, rv = O.attention_backward_f64(q[sl_q], k[sl_k], v[sl_k], dout[sl_q], sq, sk, d, True)
        assert np.max(np.abs(hq[sl_q] - rq)) < 2e-5 * (1 + np.abs(rq).max())
        assert np.max(np.abs(hk[sl_k] - rk)) < 2e-5 * (1 + np.abs(rk).max())
        assert np.max(np.abs(hv[sl_k] - rv)) < 2e-5 * (1 + np.abs(rv).max())


# Tensor-core backward (TF32 precision, d in {32, 64, 96, 128}): the same f64
# oracle, within the TF32 bound of the forward's parity bar, 2e-3 relative to
# the gradient's magnitude (measured: at most 6e-4 on these cases).
TC_TOL = 2e-3
TC_BWD_CASES = [(1, 64, 64, 64, False), (1, 128, 128, 128, True), (2, 300, 200, 128, True),
                (1, 200, 300, 128, True), (3, 129, 257, 32, False), (1, 1000, 1000, 96, True),
                (2, 517, 517, 64, True), (1, 33, 17, 128, True), (1, 1, 5, 64, False),
                (1, 700, 900, 128, False), (2, 2048, 2048, 128, True), (4, 1024, 1024, 64, False)]


def _tc_grads(fa, bh, sq, sk, d, causal, seed=0):
    q, k, v = (random_vec(bh * n * d, seed + i) for i, n in enumerate((sq, sk, sk)))
    dout = random_vec(bh * sq * d, seed + 3)
    old = fa.get_precision()
    try:
        fa.set_precision(fa.PREC_FP32)  # exact forward: O and LSE as the oracle's
        out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
        fa.set_precision(fa.PREC_TF32)
        grads = fa.flash_attention_backward(q, k, v, out, lse, dout, bh, sq, sk, d, causal)
        path = fa.last_path()
    finally:
        fa.set_precision(old)
    return (q, k, v, dout), grads, path


@pytest.mark.gpu
@pytest.mark.parametrize("bh,sq,sk,d,causal", TC_BWD_CASES)
def test_tc_backward_matches_f64_oracle(gpu_lib, bh, sq, sk, d, causal):
    (q, k, v, dout), (dq, dk, dv), path = _tc_grads(gpu_lib, bh, sq, sk, d, causal)
    assert path == "tc_tf32_backward"
    for h in range(bh):
        sl_q, sl_k = slice(h * sq * d, (h + 1) * sq * d), slice(h * sk * d, (h + 1) * sk * d)
        rq, rk, rv = O.attention_backward_f64(q[sl_q], k[sl_k], v[sl_k], dout[sl_q], sq, sk, d,
                                              causal)
        for g, r in ((dq[sl_q], rq), (dk[sl_k], rk), (dv[sl_k], rv)):
            assert np.all(np.isfinite(g))
            assert np.max(np.abs(g - r)) < TC_TOL * (1.0 + np.max(np.abs(r)))


@pytest.mark.gpu
def test_tc_backward_keys_no_row_sees_are_zero(gpu_lib):
    # Causal with seq_len_k > seq_len_q: keys past the last row get exactly
    # zero dK and dV (their key blocks have no query block at all).
    bh, sq, sk, d = 2, 100, 700, 64
    _, (dq, dk, dv), path = _tc_grads(gpu_lib, bh, sq, sk, d, True, seed=40)
    assert path == "tc_tf32_backward"
    dk, dv = dk.reshape(bh, sk, d), dv.reshape(bh, sk, d)
    assert np.all(dk[:, sq:] == 0) and np.all(dv[:, sq:] == 0)
    assert np.any(dk[:, :sq] != 0)


@pytest.mark.gpu
def test_tc_backward_device_api_and_unaligned_fallback(gpu_lib):
    # The device entry point runs the tensor-core kernels on 16-byte aligned
    # tensors and the exact f32 kernels on a view at an odd float offset; both
    # match the oracle.
    import torch
    fa = gpu_lib
    bh, sq, sk, d = 3, 150, 200, 64
    q, k, v = random_vec(bh * sq * d, 51), random_vec(bh * sk * d, 52), random_vec(bh * sk * d, 53)
    dout = random_vec(bh * sq * d, 54)
    old = fa.get_precision()
    try:
        fa.set_precision(fa.PREC_FP32)
        out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, True)
        fa.set_precision(fa.PREC_TF32)
        for shift, want_path in ((0, "tc_tf32_backward"), (1, "simt_backward")):
            def t(x, n):
                buf = torch.zeros(x.size + shift, device="cuda")
                buf[shift:] = torch.from_numpy(np.ascontiguousarray(x)).cuda()
                return buf[shift:].view(bh, n, -1)
            grads = [t(np.zeros(bh * n * d, np.float32), n) for n in (sq, sk, sk)]
            fa.backward_device(t(q, sq), t(k, sk), t(v, sk), t(out, sq),
                               torch.from_numpy(lse).cuda().view(bh, sq), t(dout, sq), *grads,
                               causal=True)
            fa.sync_status()
            assert fa.last_path() == want_path
            dq, dk, dv = (g.cpu().numpy().ravel() for g in grads)
            for h in range(bh):
                sl_q, sl_k = slice(h * sq * d, (h + 1) * sq * d), slice(h * sk * d, (h + 1) * sk * d)
                rq, rk, rv = O.attention_backward_f64(q[sl_q], k[sl_k], v[sl_k], dout[sl_q], sq,
                                                      sk, d, True)
                for g, r in ((dq[sl_q], rq), (dk[sl_k], rk), (dv[sl_k], rv)):
                    assert np.max(np.abs(g - r)) < TC_TOL * (1.0 + np.max(np.abs(r)))
    finally:
        fa.set_precision(old)
