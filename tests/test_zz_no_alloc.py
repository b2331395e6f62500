"""The allocation-free decode entry point (fa_forward_decode_noalloc).

Some callers cannot allocate device memory while they run (an allocator that
forbids new device allocations, or a runtime that owns all device memory).
This entry point serves them: its split partials live in a fixed device array
of the library.  The tests call it through the C ABI on several calls in a
row and check each result against the CPU oracle (the crate's v2 forward
restated) and against the regular device entry point (fa_forward_device),
within the tolerance of the exact-f32 decode path.  This file is collected
last, and passes alone or after the rest.

The array holds 2^20 floats.  A call needs splits * rows * (d + 1) of them,
and the split count keeps every CTA of the launch in one wave (at most 8
resident CTAs per SM), so on a 148-SM B200 the largest need is about
8 * 148 * 257 floats (1.2 MB): the size refusal cannot trigger there.  The
CPU tests (tests/test_abi.py) cover the refusals that can.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-5


def _inputs(bh, sq, sk, d, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(bh * n * d, dtype=np.float32) for n in (sq, sk, sk)]


def _run(fa, torch, host, bh, sq, sk, d, causal):
    q, k, v = (torch.from_numpy(a).cuda().view(bh, -1, d) for a in host)
    want = torch.empty(bh, sq, d, device="cuda")
    want_lse = torch.empty(bh, sq, device="cuda")
    fa.forward_device(q, k, v, want, want_lse, causal=causal)
    got = torch.full((bh, sq, d), float("nan"), device="cuda")
    got_lse = torch.full((bh, sq), float("nan"), device="cuda")
    fa.forward_decode_noalloc(q, k, v, got, got_lse, causal=causal)
    fa.sync_status()
    assert fa.last_path() == "decode_splitkv_noalloc"
    return got.cpu().numpy().ravel(), got_lse.cpu().numpy().ravel(), want, want_lse


@pytest.mark.parametrize("shapes", [
    # two calls in a row on different shapes (the second reuses the array
    # the first left behind)
    ((64, 1, 32768, 128, False, 3), (6, 4, 5000, 64, True, 7)),
    # d = 256, one slice (the most key splits) then enough rows for one split
    ((1, 1, 70000, 256, False, 11), (64, 16, 600, 128, False, 12)),
])
def test_noalloc_matches_oracle_and_device_entry(gpu_lib, shapes):
    import torch
    fa = gpu_lib
    for (bh, sq, sk, d, causal, seed) in shapes:
        host = _inputs(bh, sq, sk, d, seed)
        got, got_lse, want, want_lse = _run(fa, torch, host, bh, sq, sk, d, causal)
        ref, ref_lse, _ = O.flash_v2_multihead(*host, bh, sq, sk, d, causal)
        assert float(np.abs(got - ref).max()) < TOL
        assert float(np.abs(got_lse - ref_lse).max()) < TOL
        assert float(np.abs(got - want.cpu().numpy().ravel()).max()) < TOL
        assert float(np.abs(got_lse - want_lse.cpu().numpy().ravel()).max()) < TOL


def test_noalloc_uses_the_device_set_by_fa_set_device(gpu_lib):
    # After fa_set_device the call runs on that device even when another one
    # is current (here: the same device, made current again by the library).
    import torch
    fa = gpu_lib
    fa.set_device(0)
    bh, sq, sk, d = 4, 1, 4096, 128
    host = _inputs(bh, sq, sk, d, 5)
    got, got_lse, _, _ = _run(fa, torch, host, bh, sq, sk, d, False)
    ref, ref_lse, _ = O.flash_v2_multihead(*host, bh, sq, sk, d, False)
    assert float(np.abs(got - ref).max()) < TOL
    assert float(np.abs(got_lse - ref_lse).max()) < TOL
