"""GPU parity: the C ABI on a B200 against the CPU oracle on identical inputs.

Tolerances (max abs error vs the oracle, output and row LSE):
  TF32   (tcgen05 kind::tf32)         2e-3
  3xTF32 (error-compensated default)  2e-5
  FP32   (CUDA-core f32)              2e-5
plus the crate's own assertion of every case against its naive oracle, 1e-3
(tests/correctness.rs:109-112).
"""
import numpy as np
import pytest

import oracle as O
from fa_cases import (AGREEMENT_CASES, BASELINE_CONFIGS, REFERENCE_CASES, TC_CASES,
                      baseline_inputs, max_abs_diff, random_vec)

pytestmark = pytest.mark.gpu

TOL = {0: 2e-3, 1: 2e-5, 2: 2e-5}
PRECISIONS = [0, 1, 2]


@pytest.fixture
def fa(gpu_lib):
    old = gpu_lib.get_precision()
    yield gpu_lib
    gpu_lib.set_precision(old)


def run_single(fa, q, k, v, sq, sk, d, br, bc, causal, fn=None):
    out = np.zeros(sq * d, np.float32)
    (fn or fa.flash_attention_v2)(q, k, v, sq, sk, d,
                                  fa.FlashAttentionConfig(br, bc, causal), out)
    return out


@pytest.mark.parametrize("prec", PRECISIONS)
@pytest.mark.parametrize("case", REFERENCE_CASES)
def test_reference_matrix(fa, prec, case):
    sq, sk, d, br, bc, causal = case
    fa.set_precision(prec)
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    out = run_single(fa, q, k, v, sq, sk, d, br, bc, causal)
    want, _ = O.flash_v2(q, k, v, sq, sk, d, causal, br, bc)
    assert max_abs_diff(out, want) < TOL[prec], fa.last_path()
    assert max_abs_diff(out, O.naive_f32(q, k, v, sq, sk, d, causal)) < 1e-3


@pytest.mark.parametrize("prec", PRECISIONS)
@pytest.mark.parametrize("case", TC_CASES)
def test_tensor_core_shapes_with_lse(fa, prec, case):
    # the crate's input distribution, uniform(-1, 1) (tests/correctness.rs:63-66)
    sq, sk, d, causal = case
    fa.set_precision(prec)
    q, k, v = random_vec(sq * d, sq), random_vec(sk * d, sk + 1), random_vec(sk * d, d + 2)
    out, lse = fa.multihead_lse(q, k, v, 1, sq, sk, d, causal)
    path = fa.last_path()
    want, wlse = O.flash_v2(q, k, v, sq, sk, d, causal)
    assert max_abs_diff(out, want) < TOL[prec], path
    assert max_abs_diff(lse, wlse) < TOL[prec], path
    if prec == 0 and sq > 16:
        assert path == "tcgen05_tf32"
    if prec == 1 and sq > 16:
        assert path == "tcgen05_3xtf32"


@pytest.mark.parametrize("case", TC_CASES[:8])
def test_tf32_error_model_on_gaussian_inputs(fa, case):
    # N(0,1) inputs: the tensor core reads K and V truncated to TF32 (relative
    # error < 2^-10 each), Q is rounded to nearest when staged; the output error
    # stays within 2^-10 * max|V| + 5e-4, which is the TF32 bound this mode
    # documents (the 2e-3 contract holds for the benchmark configs).
    sq, sk, d, causal = case
    fa.set_precision(fa.PREC_TF32)
    rng = np.random.default_rng(sq * 7919 + sk * 31 + d)
    q = rng.standard_normal(sq * d, dtype=np.float32)
    k = rng.standard_normal(sk * d, dtype=np.float32)
    v = rng.standard_normal(sk * d, dtype=np.float32)
    out, lse = fa.multihead_lse(q, k, v, 1, sq, sk, d, causal)
    want, wlse = O.flash_v2(q, k, v, sq, sk, d, causal)
    bound = 2.0 ** -10 * float(np.abs(v).max()) + 5e-4
    assert max_abs_diff(out, want) < bound
    assert max_abs_diff(lse, wlse) < 2e-3


@pytest.mark.parametrize("prec", PRECISIONS)
def test_multihead_matches_per_head_naive(fa, prec):
    fa.set_precision(prec)
    b, h, sq, sk, d = 2, 3, 37, 50, 16
    q = random_vec(b * h * sq * d, 21)
    k = random_vec(b * h * sk * d, 22)
    v = random_vec(b * h * sk * d, 23)
    cfg = fa.FlashAttentionConfig(8, 12, True)
    for fn in (fa.flash_attention_multihead_v1, fa.flash_attention_multihead_v2,
               fa.flash_attention_multihead_v3, fa.flash_attention_multihead):
        out = np.zeros(b * h * sq * d, np.float32)
        fn(q, k, v, b, h, sq, sk, d, cfg, out)
        for bh in range(b * h):
            sl_q = slice(bh * sq * d, (bh + 1) * sq * d)
            sl_k = slice(bh * sk * d, (bh + 1) * sk * d)
            want = O.naive_f32(q[sl_q], k[sl_k], v[sl_k], sq, sk, d, True)
            assert max_abs_diff(out[sl_q], want) < 1e-3


@pytest.mark.parametrize("br,bc", [(64, 128), (32, 32), (1024, 1024), (1, 1)])
def test_causal_first_query_equals_first_value_row(fa, br, bc):
    # tests/correctness.rs:240-263 at the library's default precision (3xTF32): 1e-5.
    fa.set_precision(fa.PREC_3XTF32)
    s, d = 256, 64
    q, k, v = random_vec(s * d, 30), random_vec(s * d, 31), random_vec(s * d, 32)
    for fn in (fa.flash_attention_v1, fa.flash_attention_v2, fa.flash_attention_v3):
        out = run_single(fa, q, k, v, s, s, d, br, bc, True, fn)
        assert max_abs_diff(out[:d], v[:d]) < 1e-5


def test_causal_first_query_tf32_within_tf32_rounding(fa):
    # In TF32 mode V is rounded to 10 mantissa bits, so row 0 equals V[0] only
    # to TF32 precision (the reason the default precision is 3xTF32).
    fa.set_precision(fa.PREC_TF32)
    s, d = 256, 64
    q, k, v = random_vec(s * d, 30), random_vec(s * d, 31), random_vec(s * d, 32)
    out = run_single(fa, q, k, v, s, s, d, 64, 128, True)
    assert max_abs_diff(out[:d], v[:d]) < 2e-3


@pytest.mark.parametrize("prec", PRECISIONS)
def test_output_is_finite(fa, prec):
    fa.set_precision(prec)
    sq, sk, d = 40, 40, 32
    out = run_single(fa, random_vec(sq * d, 10), random_vec(sk * d, 11), random_vec(sk * d, 12),
                     sq, sk, d, 64, 128, True)
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("case", AGREEMENT_CASES)
def test_v1_v2_v3_agree(fa, case):
    # tests/correctness.rs:295-375 demands v2 == v3 within 1e-5; on the GPU the
    # three run the same kernels, so they agree bit for bit.
    sq, sk, d, br, bc, causal = case
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    outs = [run_single(fa, q, k, v, sq, sk, d, br, bc, causal, fn)
            for fn in (fa.flash_attention_v1, fa.flash_attention_v2, fa.flash_attention_v3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


def test_zero_block_size_is_clamped(fa):
    sq, sk, d = 23, 29, 16
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    for causal in (False, True):
        out = run_single(fa, q, k, v, sq, sk, d, 0, 0, causal)
        assert max_abs_diff(out, O.naive_f32(q, k, v, sq, sk, d, causal)) < 1e-3


def test_block_size_does_not_change_results(fa):
    sq, sk, d = 200, 200, 128
    q, k, v = random_vec(sq * d, 1), random_vec(sk * d, 2), random_vec(sk * d, 3)
    a = run_single(fa, q, k, v, sq, sk, d, 64, 128, True)
    for br, bc in ((1, 1), (7, 3), (1024, 1024)):
        assert np.array_equal(a, run_single(fa, q, k, v, sq, sk, d, br, bc, True))


@pytest.mark.parametrize("sq,sk,d,causal", [
    (1, 32768, 128, False), (1, 5000, 64, True), (4, 3000, 128, True), (16, 2049, 256, False),
    (3, 1000, 36, False), (8, 100000, 128, False), (2, 7, 128, False)])
def test_decode_split_kv(fa, sq, sk, d, causal):
    bh = 3
    rng = np.random.default_rng(sq + sk + d)
    q = rng.standard_normal(bh * sq * d, dtype=np.float32)
    k = rng.standard_normal(bh * sk * d, dtype=np.float32)
    v = rng.standard_normal(bh * sk * d, dtype=np.float32)
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    assert fa.last_path() == "decode_splitkv"
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    assert max_abs_diff(out, want) < 2e-5
    assert max_abs_diff(lse, wlse) < 2e-5


# ---- the five benchmark configs, both tensor-core modes ------
# Every row of C1-C4 is compared with the oracle (the crate's v2 forward
# restated); C5 (one 131072-row causal head, 4.4 TFLOP) on whole 64-row query
# blocks of run_v2 spread over the head, each equal to the same block of a
# full oracle run, plus rows against the f64 naive.

@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4"])
def test_baseline_configs_every_row(fa, prec, name):
    fa.set_precision(prec)
    q, k, v, (bh, sq, sk, d, causal) = baseline_inputs(name)
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    tol = 2e-5 if name == "c4" else TOL[prec]  # c4 runs the exact-f32 decode kernel
    assert max_abs_diff(out, want) < tol
    assert max_abs_diff(lse, wlse) < tol


C5_BLOCKS = [0, 1, 2, 63, 64, 511, 1023, 1024, 1500, 2046, 2047]


@pytest.mark.parametrize("prec", [0, 1])
def test_baseline_c5_query_blocks_against_v2_oracle(fa, prec):
    fa.set_precision(prec)
    q, k, v, (bh, sq, sk, d, causal) = baseline_inputs("c5")
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    assert np.all(np.isfinite(out))
    assert fa.last_path() == ("tcgen05_tf32" if prec == 0 else "tcgen05_3xtf32")
    want, wlse = O.flash_v2_items(q, k, v, bh, sq, sk, d, causal, C5_BLOCKS)
    rows = O.item_rows(C5_BLOCKS, sq)
    got = out.reshape(-1, d)[rows]
    assert max_abs_diff(got, want.reshape(-1, d)[rows]) < TOL[prec]
    assert max_abs_diff(lse[rows], wlse[rows]) < TOL[prec]
    for r in (0, 127, 4097, 65535, 100000, sq - 1):
        w, wl = O.naive_f64(q, k, v, sq, sk, d, causal, r, r + 1)
        assert max_abs_diff(out[r * d:(r + 1) * d], w) < TOL[prec]
        assert abs(float(lse[r]) - float(wl[0])) < TOL[prec]


def test_device_api_matches_host_api(fa):
    import torch
    fa.set_precision(fa.PREC_TF32)
    bh, sq, sk, d = 4, 300, 500, 128
    q, k, v = (random_vec(bh * sq * d, 1), random_vec(bh * sk * d, 2),
               random_vec(bh * sk * d, 3))
    host, hlse = fa.multihead_lse(q, k, v, bh, sq, sk, d, True)
    dq = torch.from_numpy(q).cuda().view(bh, sq, d)
    dk = torch.from_numpy(k).cuda().view(bh, sk, d)
    dv = torch.from_numpy(v).cuda().view(bh, sk, d)
    out = torch.empty_like(dq)
    lse = torch.empty(bh, sq, device="cuda")
    n0 = fa.launch_count()
    fa.forward_device(dq, dk, dv, out, lse, causal=True)
    fa.sync_status()
    assert fa.launch_count() > n0
    assert np.array_equal(out.cpu().numpy().ravel(), host)
    assert np.array_equal(lse.cpu().numpy().ravel(), hlse)


@pytest.mark.parametrize("prec", [0, 2])
def test_partial_ranges_and_lse_combine(fa, prec):
    # The KV-range split used across GPUs, emulated on one GPU: three key
    # ranges (one entirely in some rows' future), merged by the LSE combine.
    import torch
    fa.set_precision(prec)
    bh, s, d = 2, 700, 128
    q, k, v = random_vec(bh * s * d, 4), random_vec(bh * s * d, 5), random_vec(bh * s * d, 6)
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, s, s, d, True)
    dq = torch.from_numpy(q).cuda().view(bh, s, d)
    dk = torch.from_numpy(k).cuda().view(bh, s, d)
    dv = torch.from_numpy(v).cuda().view(bh, s, d)
    bounds = [0, 256, 400, s]
    parts_o = torch.empty(len(bounds) - 1, bh, s, d, device="cuda")
    parts_l = torch.empty(len(bounds) - 1, bh, s, device="cuda")
    for i in range(len(bounds) - 1):
        a, b = bounds[i], bounds[i + 1]
        fa.forward_partial_device(dq, dk[:, a:b].contiguous(), dv[:, a:b].contiguous(),
                                  parts_o[i], parts_l[i], True, 0, a)
    out = torch.empty(bh * s, d, device="cuda")
    lse = torch.empty(bh * s, device="cuda")
    fa.lse_combine_device(parts_o.view(len(bounds) - 1, bh * s, d),
                          parts_l.view(len(bounds) - 1, bh * s), out, lse)
    fa.sync_status()
    tol = TOL[prec]
    assert max_abs_diff(out.cpu().numpy().ravel(), want) < tol
    assert max_abs_diff(lse.cpu().numpy().ravel(), wlse) < tol


def test_kv_split_one_rank_nccl(fa):
    # The multi-GPU key-range split through the real kernels and NCCL with one
    # rank (zig-zag chunks, partial kernels, all-to-all, LSE merge).
    import torch
    import torch.distributed as dist
    from fa_b200.kvsplit import kv_split_forward
    fa.set_precision(fa.PREC_TF32)
    rows, d = 1000, 128
    q, k, v = (random_vec(rows * d, s) for s in (41, 42, 43))
    want, wlse = O.flash_v2(q, k, v, rows, rows, d, True)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:29541", rank=0, world_size=1,
                            device_id=dev)
    try:
        t = [torch.from_numpy(x).to(dev).view(1, rows, d) for x in (q, k, v)]
        out, lse, (a, b) = kv_split_forward(t[0], t[1], t[2], True)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    assert (a, b) == (0, rows)
    assert max_abs_diff(out.cpu().numpy().ravel(), want) < 2e-3
    assert max_abs_diff(lse.cpu().numpy(), wlse) < 2e-3


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("shape", [(6, 4096, 4096, 128, True), (24, 1024, 1024, 64, False),
                                   (5, 2560, 2000, 128, True), (9, 3000, 3000, 64, True),
                                   (7, 300, 1100, 128, False)])
def test_persistent_schedule_many_tiles_per_cluster(fa, prec, shape):
    # More 256-row work tiles than SM pairs, so every cluster runs several tiles
    # back to back (next-tile Q staging, the cross-tile MMA order, epilogues).
    # Outputs start as NaN so a row the kernel skips cannot pass on stale memory.
    import torch
    bh, sq, sk, d, causal = shape
    fa.set_precision(prec)
    q, k, v = (random_vec(bh * sq * d, 51), random_vec(bh * sk * d, 52),
               random_vec(bh * sk * d, 53))
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.full((bh, sq, d), float("nan"), device="cuda")
    lse = torch.full((bh, sq), float("nan"), device="cuda")
    fa.forward_device(dq.view(bh, sq, d), dk.view(bh, sk, d), dv.view(bh, sk, d), out, lse,
                      causal=causal)
    fa.sync_status()
    assert fa.last_path() == ("tcgen05_tf32" if prec == 0 else "tcgen05_3xtf32")
    assert max_abs_diff(out.cpu().numpy().ravel(), want) < TOL[prec]
    assert max_abs_diff(lse.cpu().numpy().ravel(), wlse) < TOL[prec]


@pytest.mark.parametrize("prec", [0, 1])
def test_partial_ranges_with_keyless_tiles(fa, prec):
    # Key range [2048, 4096) of a causal 4096-row slice: the first 2048 rows see
    # no key (O = 0, lse = -inf), so the persistent kernel meets work tiles with
    # no key block between tiles with keys.  Merged with [0, 2048) by LSE.
    import torch
    fa.set_precision(prec)
    bh, s, d = 6, 4096, 128
    q, k, v = random_vec(bh * s * d, 61), random_vec(bh * s * d, 62), random_vec(bh * s * d, 63)
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, s, s, d, True)
    dq, dk, dv = (torch.from_numpy(x).cuda().view(bh, s, d) for x in (q, k, v))
    parts_o = torch.full((2, bh, s, d), float("nan"), device="cuda")
    parts_l = torch.full((2, bh, s), float("nan"), device="cuda")
    for i, (a, b) in enumerate([(0, 2048), (2048, s)]):
        fa.forward_partial_device(dq, dk[:, a:b].contiguous(), dv[:, a:b].contiguous(),
                                  parts_o[i], parts_l[i], True, 0, a)
        fa.sync_status()
        assert fa.last_path() == ("tcgen05_tf32" if prec == 0 else "tcgen05_3xtf32")
    late = parts_o[1][:, :2048].cpu().numpy()
    assert np.all(late == 0.0)
    assert np.all(np.isneginf(parts_l[1][:, :2048].cpu().numpy()))
    out = torch.empty(bh * s, d, device="cuda")
    lse = torch.empty(bh * s, device="cuda")
    fa.lse_combine_device(parts_o.view(2, bh * s, d), parts_l.view(2, bh * s), out, lse)
    fa.sync_status()
    assert max_abs_diff(out.cpu().numpy().ravel(), want) < TOL[prec]
    assert max_abs_diff(lse.cpu().numpy().ravel(), wlse) < TOL[prec]


@pytest.mark.parametrize("prec", [0, 1])
def test_pageable_host_buffers_go_through_pinned_staging(fa, prec):
    # A call this large with ordinary (pageable) numpy buffers takes the pinned
    # staging path; it must give exactly what the device API gives.
    import torch
    fa.set_precision(prec)
    bh, s, d = 12, 1024, 128
    q, k, v = (random_vec(bh * s * d, 71), random_vec(bh * s * d, 72),
               random_vec(bh * s * d, 73))
    out, lse = fa.multihead_lse(q, k, v, bh, s, s, d, True)
    dq, dk, dv = (torch.from_numpy(x).cuda().view(bh, s, d) for x in (q, k, v))
    dout = torch.empty_like(dq)
    dlse = torch.empty(bh, s, device="cuda")
    fa.forward_device(dq, dk, dv, dout, dlse, causal=True)
    fa.sync_status()
    # (the staged call runs in chunks of slices, whose launches may split key
    # ranges differently from one launch over all slices: equal to rounding)
    assert max_abs_diff(out, dout.cpu().numpy().ravel()) < 1e-5
    assert max_abs_diff(lse, dlse.cpu().numpy().ravel()) < 1e-5
    out2 = np.zeros(bh * s * d, np.float32)
    fa.flash_attention_multihead_v2(q, k, v, 1, bh, s, s, d, fa.FlashAttentionConfig(64, 128, True),
                                    out2)
    assert np.array_equal(out2, out)


def test_pinned_host_buffers_via_fa_pin_host(fa):
    # Buffers pinned through the library take the direct copy path and give the
    # same result as the staged path on the same data.
    fa.set_precision(fa.PREC_TF32)
    bh, s, d = 12, 1024, 128
    q, k, v = (random_vec(bh * s * d, 81), random_vec(bh * s * d, 82),
               random_vec(bh * s * d, 83))
    cfg = fa.FlashAttentionConfig(64, 128, True)
    staged = np.zeros(bh * s * d, np.float32)
    fa.flash_attention_multihead_v2(q, k, v, 1, bh, s, s, d, cfg, staged)
    out = np.zeros(bh * s * d, np.float32)
    for a in (q, k, v, out):
        fa.pin_host(a)
    fa.pin_host(q)  # pinning twice is accepted
    try:
        fa.flash_attention_multihead_v2(q, k, v, 1, bh, s, s, d, cfg, out)
    finally:
        for a in (q, k, v, out):
            fa.unpin_host(a)
    assert max_abs_diff(out, staged) < 1e-5


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("shape", [(1, 4096, 4096, 128, True), (1, 4096, 4096, 128, False),
                                   (1, 512, 512, 64, False), (2, 1000, 3000, 128, True),
                                   (3, 700, 700, 64, True), (1, 2048, 2048, 64, False),
                                   (1, 100, 20000, 128, False), (2, 128, 8192, 64, False),
                                   (1, 77, 9000, 128, True), (1, 96, 32768, 128, False)])
def test_key_range_split_of_small_launches(fa, prec, shape):
    # Few tiles: the tcgen05 kernels divide each tile's key blocks over several
    # work units (TF32) or CTAs (3xTF32) and merge their partials by LSE.
    bh, sq, sk, d, causal = shape
    fa.set_precision(prec)
    q, k, v = (random_vec(bh * sq * d, 91), random_vec(bh * sk * d, 92),
               random_vec(bh * sk * d, 93))
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    assert fa.last_path() == ("tcgen05_tf32" if prec == 0 else "tcgen05_3xtf32")
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    assert max_abs_diff(out, want) < TOL[prec]
    assert max_abs_diff(lse, wlse) < TOL[prec]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("shape", [(2, 300, 300, 128, True), (3, 1, 2000, 64, False),
                                   (2, 100, 700, 64, False)])
def test_device_api_pointers_off_16_bytes(fa, prec, shape):
    # Views one float into a buffer: the tensor-map and vector-load kernels need
    # 16-byte aligned bases, so the call runs the CUDA-core f32 kernel.
    import torch
    bh, sq, sk, d, causal = shape
    fa.set_precision(prec)
    q, k, v = (random_vec(bh * sq * d, 71), random_vec(bh * sk * d, 72),
               random_vec(bh * sk * d, 73))

    def shifted(a, rows):
        buf = torch.zeros(a.size + 1, device="cuda")
        buf[1:].copy_(torch.from_numpy(a))
        return buf[1:].view(bh, rows, d)

    dq, dk, dv = shifted(q, sq), shifted(k, sk), shifted(v, sk)
    dout = torch.full((bh * sq * d + 1,), float("nan"), device="cuda")[1:].view(bh, sq, d)
    lse = torch.empty(bh, sq, device="cuda")
    assert dq.data_ptr() % 16 != 0
    fa.forward_device(dq, dk, dv, dout, lse, causal=causal)
    torch.cuda.synchronize()
    assert fa.last_path() == "simt_fp32"
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    assert max_abs_diff(dout.cpu().numpy().ravel(), want) < TOL[2]
    assert max_abs_diff(lse.cpu().numpy().ravel(), wlse) < TOL[2]


def test_calls_after_fa_shutdown(fa):
    # fa_shutdown frees the staging rings and the calling thread's streams,
    # events and status word; the next calls create them again.
    import ctypes
    L = fa._load()
    L.fa_shutdown.restype = None
    fa.set_precision(0)
    for bh, s, d in ((2, 300, 64), (8, 1024, 128)):  # the small path, then the staged one
        q, k, v = (random_vec(bh * s * d, 81 + i) for i in range(3))
        cfg = fa.FlashAttentionConfig(64, 128, True)
        a = np.zeros(bh * s * d, np.float32)
        fa.flash_attention_multihead_v2(q, k, v, 1, bh, s, s, d, cfg, a)
        L.fa_shutdown()
        b = np.full(bh * s * d, np.nan, np.float32)
        fa.flash_attention_multihead_v2(q, k, v, 1, bh, s, s, d, cfg, b)
        assert np.array_equal(a, b)
        L.fa_shutdown()


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("causal", [False, True])
def test_rising_scores_rescale_every_block(fa, prec, causal):
    # Q all ones and K rows j/64 (exact in TF32): the score of key j is j / 8
    # before scaling, so every 128-key block raises the row maximum by ~23
    # log2 units and takes the rescale path of O and l (P recomputed against
    # the new maximum).  The output is a weighted mean of the last few V rows.
    bh, sq, sk, d = 2, 300, 1024, 64
    fa.set_precision(prec)
    q = np.ones(bh * sq * d, np.float32)
    kr = (np.arange(sk, dtype=np.float32) / 64.0)[:, None] * np.ones((1, d), np.float32)
    k = np.tile(kr.ravel(), bh).astype(np.float32)
    v = random_vec(bh * sk * d, 97)
    out, lse = fa.multihead_lse(q, k, v, bh, sq, sk, d, causal)
    want, wlse, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal)
    assert np.all(np.isfinite(out))
    assert max_abs_diff(out, want) < TOL[prec]
    # the LSE carries the rounding of the prescaled Q (TF32: 2^-12 relative)
    # times scores near 40 log2 units; 3xTF32 is compensated
    rel = 2.0 ** -10 if prec == 0 else 1e-4
    assert max_abs_diff(lse, wlse) < rel * (1 + np.max(np.abs(wlse)))
