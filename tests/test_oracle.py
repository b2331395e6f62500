"""Pins the CPU oracle (oracle/fa_oracle.c) to what the reference's own tests hold.

The reference has no golden vectors; its tests pin behaviour by known answers
and by agreement with its naive oracle.  Each test below restates one of those
checks against the oracle, so the oracle is trusted before it checks the GPU.
"""
import math

import numpy as np
import pytest

import oracle as O
from fa_cases import AGREEMENT_CASES, REFERENCE_CASES, max_abs_diff, random_vec


def test_exp_matches_libm():
    # avx512.rs:596-620: exp over [-80, 80) step 0.1, rel err < 1e-5 where exp > 1e-30.
    worst = 0.0
    for i in range(-800, 800):
        x = i * 0.1
        want = math.exp(np.float32(x))
        if want > 1e-30 and math.isfinite(want):
            got = O.exp_cephes(np.float32(x))
            worst = max(worst, abs(got - want) / want)
    assert worst < 1e-5, worst


def test_exp_of_neg_inf_is_zero():
    assert O.exp_cephes(float("-inf")) == 0.0


@pytest.mark.parametrize("case", REFERENCE_CASES)
def test_flash_matches_naive(case):
    # tests/correctness.rs:74-113 (run_case): flash vs naive, max abs < 1e-3.
    sq, sk, d, br, bc, causal = case
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    out, lse = O.flash_v2(q, k, v, sq, sk, d, causal, br, bc)
    naive = O.naive_f32(q, k, v, sq, sk, d, causal)
    assert max_abs_diff(out, naive) < 1e-3
    # and against f64 (bounds the oracle's own rounding error; LSE included)
    n64, l64 = O.naive_f64(q, k, v, sq, sk, d, causal)
    assert max_abs_diff(out, n64) < 2e-6
    assert max_abs_diff(lse, l64) < 2e-6


def test_multihead_matches_per_head_naive():
    # tests/correctness.rs:204-238
    b, h, sq, sk, d = 2, 3, 37, 50, 16
    q = random_vec(b * h * sq * d, 21)
    k = random_vec(b * h * sk * d, 22)
    v = random_vec(b * h * sk * d, 23)
    out, _, _ = O.flash_v2_multihead(q, k, v, b * h, sq, sk, d, True, 8, 12, nthreads=3)
    for bh in range(b * h):
        want = O.naive_f32(q[bh * sq * d:(bh + 1) * sq * d], k[bh * sk * d:(bh + 1) * sk * d],
                           v[bh * sk * d:(bh + 1) * sk * d], sq, sk, d, True)
        assert max_abs_diff(out[bh * sq * d:(bh + 1) * sq * d], want) < 1e-3


@pytest.mark.parametrize("br,bc", [(64, 128), (32, 32), (1024, 1024), (1, 1)])
def test_causal_first_query_equals_first_value_row(br, bc):
    # tests/correctness.rs:240-263: known answer, within 1e-5.
    s, d = 256, 64
    q, k, v = random_vec(s * d, 30), random_vec(s * d, 31), random_vec(s * d, 32)
    out, _ = O.flash_v2(q, k, v, s, s, d, True, br, bc)
    assert max_abs_diff(out[:d], v[:d]) < 1e-5


@pytest.mark.parametrize("case", AGREEMENT_CASES)
def test_block_sizes_agree(case):
    # The crate's v1/v2/v3 agreement (:295-375) in its v2-only form: different
    # tilings of the same math agree to 1e-5.
    sq, sk, d, br, bc, causal = case
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    a, _ = O.flash_v2(q, k, v, sq, sk, d, causal, br, bc)
    b, _ = O.flash_v2(q, k, v, sq, sk, d, causal, 64, 128)
    assert max_abs_diff(a, b) < 1e-5


def test_zero_sized_dimensions_leave_out_untouched():
    # tests/correctness.rs:461-504
    d = 8
    out = np.full(4 * d, 12.5, np.float32)
    O.flash_v2(random_vec(4 * d, 4), np.zeros(0, np.float32), np.zeros(0, np.float32),
               4, 0, d, False, out=out)
    assert np.all(out == 12.5)


def test_zero_block_size_is_clamped():
    # tests/correctness.rs:506-537
    sq, sk, d = 23, 29, 16
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    for causal in (False, True):
        out, _ = O.flash_v2(q, k, v, sq, sk, d, causal, 0, 0)
        assert max_abs_diff(out, O.naive_f32(q, k, v, sq, sk, d, causal)) < 1e-3


def test_multithreaded_driver_matches_single_thread():
    bh, sq, sk, d = 3, 70, 90, 32
    q, k, v = random_vec(bh * sq * d, 5), random_vec(bh * sk * d, 6), random_vec(bh * sk * d, 7)
    a, la, items = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, True, nthreads=4)
    assert items == bh * ((sq + 63) // 64)
    for h in range(bh):
        o, l = O.flash_v2(q[h * sq * d:(h + 1) * sq * d], k[h * sk * d:(h + 1) * sk * d],
                          v[h * sk * d:(h + 1) * sk * d], sq, sk, d, True)
        assert np.array_equal(a[h * sq * d:(h + 1) * sq * d], o)
        assert np.array_equal(la[h * sq:(h + 1) * sq], l)


@pytest.mark.parametrize("sq,sk,d,causal", [(70, 90, 32, True), (90, 70, 64, False),
                                            (128, 300, 16, True), (1, 257, 8, False)])
def test_lse_matches_f64_logsumexp(sq, sk, d, causal):
    # the row log-sum-exp the restatement adds (m_i + ln l_i of the scaled
    # scores, the value the GPU kernels return beside O) against float64
    q, k, v = random_vec(sq * d, 11), random_vec(sk * d, 12), random_vec(sk * d, 13)
    _, lse = O.flash_v2(q, k, v, sq, sk, d, causal)
    s = (q.reshape(sq, d).astype(np.float64) @ k.reshape(sk, d).astype(np.float64).T) / np.sqrt(d)
    if causal:
        s = np.where(np.arange(sk)[None, :] <= np.arange(sq)[:, None], s, -np.inf)
    mx = s.max(axis=1, keepdims=True)
    want = (mx + np.log(np.exp(s - mx).sum(axis=1, keepdims=True))).ravel()
    assert np.max(np.abs(lse - want)) < 1e-5 * (1 + np.max(np.abs(want)))


def test_partial_run_matches_full_run_on_its_rows():
    # max_items limits the driver to the first 64-row query blocks (bench.py
    # samples the config-5 head this way); those rows equal a full run's
    bh, sq, sk, d = 1, 300, 300, 32
    q, k, v = random_vec(sq * d, 21), random_vec(sk * d, 22), random_vec(sk * d, 23)
    full, lf, n_full = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, True, nthreads=2)
    part, lp, n_part = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, True, nthreads=2,
                                            max_items=2)
    assert n_full == (sq + 63) // 64 and n_part == 2
    assert np.array_equal(part[:128 * d], full[:128 * d])
    assert np.array_equal(lp[:128], lf[:128])


@pytest.mark.parametrize("causal", [False, True])
def test_listed_query_blocks_equal_the_full_run(causal):
    # oracle_flash_v2_items computes single query blocks of run_v2 (used to
    # check a 131072-row head on sampled blocks): each listed block's rows must
    # be bit-identical to the same rows of a full multihead run.
    bh, sq, sk, d = 3, 300, 200, 64
    q, k, v = random_vec(bh * sq * d, 5), random_vec(bh * sk * d, 6), random_vec(bh * sk * d, 7)
    full, flse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    items = [0, 4, 7, 14]
    part, plse = O.flash_v2_items(q, k, v, bh, sq, sk, d, causal, items)
    rows = O.item_rows(items, sq)
    assert len(rows) == 64 + 44 + 64 + 44
    assert np.array_equal(full.reshape(-1, d)[rows], part.reshape(-1, d)[rows])
    assert np.array_equal(flse[rows], plse[rows])
    with pytest.raises(ValueError):
        O.flash_v2_items(q, k, v, bh, sq, sk, d, causal, [15])
