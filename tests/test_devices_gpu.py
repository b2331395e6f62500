"""The host-slice calls over a list of devices (fa_set_devices).

The crate fans its (batch, head) slices out over all cores
(src/common.rs:72-101); with a device list the library fans them out over
GPUs (contiguous slice ranges, no collective), and splits a single long slice's
keys over the GPUs with an LSE merge after peer copies of the partials.

A device may be listed more than once, so the whole multi-device logic (slice
ranges, zig-zag key chunks, row ownership, peer copies, merges) runs on one
GPU; the tests on several distinct GPUs run where the box has them.
"""
import numpy as np
import pytest

import oracle as O
from fa_cases import baseline_inputs, max_abs_diff, random_vec

pytestmark = pytest.mark.gpu

TOL = {0: 2e-3, 1: 2e-5}


@pytest.fixture
def fa(gpu_lib):
    old = gpu_lib.get_precision()
    yield gpu_lib
    gpu_lib.set_devices([])
    gpu_lib.set_precision(old)


def _one_device(fa, q, k, v, bh, sq, sk, d, causal):
    fa.set_devices([])
    return fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)


@pytest.mark.parametrize("devs", [[0, 0], [0, 0, 0], [0, 0, 0, 0, 0, 0, 0, 0]])
@pytest.mark.parametrize("prec", [0, 1])
def test_slice_ranges_over_listed_devices(fa, devs, prec):
    fa.set_precision(prec)
    bh, sq, sk, d = 7, 600, 700, 128
    q, k, v = random_vec(bh * sq * d, 1), random_vec(bh * sk * d, 2), random_vec(bh * sk * d, 3)
    want, wlse = _one_device(fa, q, k, v, bh, sq, sk, d, True)
    fa.set_devices(devs)
    assert fa.get_devices() == devs
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, True)
    # each range runs the same kernels as the whole call; only the key-range
    # split of small launches may differ, to rounding
    assert max_abs_diff(out, want) < 1e-5
    assert max_abs_diff(lse, wlse) < 1e-5
    ref, rlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, True)
    assert max_abs_diff(out, ref) < TOL[prec]
    assert max_abs_diff(lse, rlse) < TOL[prec]


@pytest.mark.parametrize("devs", [[0, 0], [0, 0, 0, 0]])
@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("shape", [(1, 16384, 16384, 128, True), (1, 12000, 12000, 64, False),
                                   (1, 5000, 20000, 128, True), (2, 9000, 9000, 128, True)])
def test_key_range_split_over_listed_devices(fa, devs, prec, shape):
    # Fewer slices than devices on long sequences: zig-zag key chunks, partial
    # rows copied to their owners, LSE merge.  Compared with the oracle on
    # whole query blocks of run_v2 spread over the slices.
    bh, sq, sk, d, causal = shape
    fa.set_precision(prec)
    q, k, v = (random_vec(bh * sq * d, 11), random_vec(bh * sk * d, 12),
               random_vec(bh * sk * d, 13))
    fa.set_devices(devs)
    out = np.full(bh * sq * d, np.nan, np.float32)
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal, out=out)
    assert np.all(np.isfinite(out))
    nb = (sq + 63) // 64
    items = sorted({h * nb + b for h in range(bh) for b in (0, 1, nb // 3, nb // 2, nb - 2, nb - 1)})
    want, wlse = O.flash_v2_items(q, k, v, bh, sq, sk, d, causal, items)
    rows = O.item_rows(items, sq)
    assert max_abs_diff(out.reshape(-1, d)[rows], want.reshape(-1, d)[rows]) < TOL[prec]
    assert max_abs_diff(lse[rows], wlse[rows]) < TOL[prec]


def test_c5_over_listed_devices_matches_one_device(fa):
    # BASELINE config 5 (one 131072-row causal head) split over four entries
    # of the device list against the one-device call, TF32.
    fa.set_precision(0)
    q, k, v, (bh, sq, sk, d, causal) = baseline_inputs("c5")
    want, wlse = _one_device(fa, q, k, v, bh, sq, sk, d, causal)
    fa.set_devices([0, 0, 0, 0])
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    assert max_abs_diff(out, want) < 2e-3
    assert max_abs_diff(lse, wlse) < 2e-3


@pytest.mark.parametrize("prec", [0, 1])
def test_several_gpus(fa, prec):
    # Distinct GPUs (peer copies between devices), where the box has them.
    # Checked against the oracle: the one-device result is itself a TF32
    # approximation, so two such results may differ by twice the tolerance.
    n = fa.device_count()
    if n < 2:
        pytest.skip("one GPU")
    devs = list(range(min(n, 8)))
    fa.set_precision(prec)
    for bh, sq, sk, d, causal in ((32, 2048, 2048, 128, True), (1, 32768, 32768, 128, True)):
        q, k, v = (random_vec(bh * sq * d, 21), random_vec(bh * sk * d, 22),
                   random_vec(bh * sk * d, 23))
        fa.set_devices(devs)
        out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
        nb = (sq + 63) // 64
        items = sorted({h * nb + b for h in {0, bh - 1} for b in (0, 1, nb // 2, nb - 2, nb - 1)})
        want, wlse = O.flash_v2_items(q, k, v, bh, sq, sk, d, causal, items)
        rows = O.item_rows(items, sq)
        assert max_abs_diff(out.reshape(-1, d)[rows], want.reshape(-1, d)[rows]) < TOL[prec]
        assert max_abs_diff(lse[rows], wlse[rows]) < TOL[prec]
