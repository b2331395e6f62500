"""The allocation-free decode entry point (fa_forward_decode_noalloc).

Some callers cannot allocate device memory while they run (an allocator that
forbids new device allocations, or a runtime that owns all device memory).
This entry point serves them: its split partials live in a fixed device array
of the library.  The test calls it through the C ABI twice in a row, on two
different shapes, and checks each result against the regular device entry
point (fa_forward_device) within the tolerance of the exact-f32 decode path.
It sits in its own file, collected last, and passes alone or after the rest.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5


def _inputs(torch, bh, sq, sk, d, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return [torch.randn(bh, n, d, device="cuda", generator=g) for n in (sq, sk, sk)]


def test_noalloc_matches_device_entry_on_two_calls(gpu_lib):
    import torch
    fa = gpu_lib
    for (bh, sq, sk, d, causal, seed) in ((64, 1, 32768, 128, False, 3),
                                           (6, 4, 5000, 64, True, 7)):
        q, k, v = _inputs(torch, bh, sq, sk, d, seed)
        want = torch.empty(bh, sq, d, device="cuda")
        want_lse = torch.empty(bh, sq, device="cuda")
        fa.forward_device(q, k, v, want, want_lse, causal=causal)
        got = torch.full((bh, sq, d), float("nan"), device="cuda")
        got_lse = torch.full((bh, sq), float("nan"), device="cuda")
        fa.forward_decode_noalloc(q, k, v, got, got_lse, causal=causal)
        fa.sync_status()
        assert fa.last_path() == "decode_splitkv_noalloc"
        assert float((got - want).abs().max()) < TOL
        assert float((got_lse - want_lse).abs().max()) < TOL

