"""CPU-side checks of the C ABI: the library loads, exports every function the
header declares, and applies the crate's argument semantics (shape panics,
zero-dimension early return) before touching any device.  No compute call is
made here; without a GPU the compute calls must fail loudly (no CPU path)."""
import ctypes
import os
import re

import numpy as np
import pytest

import fa_b200
from fa_cases import random_vec

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fa_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FA_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(", text)))


def test_header_declares_the_crate_api():
    names = declared_functions()
    for n in ("fa_flash_attention_v1", "fa_flash_attention_v2", "fa_flash_attention_v3",
              "fa_flash_attention", "fa_flash_attention_multihead_v1",
              "fa_flash_attention_multihead_v2", "fa_flash_attention_multihead_v3",
              "fa_flash_attention_multihead", "fa_config_default"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(fa_b200.lib_path())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_config_default_mirrors_crate():
    c = fa_b200._load().fa_config_default()
    assert (c.block_size_q, c.block_size_kv, c.causal) == (64, 128, 0)
    py = fa_b200.FlashAttentionConfig()
    assert (py.block_size_q, py.block_size_kv, py.causal) == (64, 128, False)


@pytest.mark.parametrize("which", ["q", "k", "v", "out"])
@pytest.mark.parametrize("fn", [fa_b200.flash_attention_v1, fa_b200.flash_attention_v2,
                                fa_b200.flash_attention_v3, fa_b200.flash_attention])
def test_shape_mismatch_panics(fn, which):
    # tests/correctness.rs:396-433: each of q/k/v/out one element short panics.
    sq, sk, d = 4, 4, 8
    bufs = {"q": random_vec(sq * d, 1), "k": random_vec(sk * d, 2), "v": random_vec(sk * d, 3),
            "out": np.zeros(sq * d, np.float32)}
    bufs[which] = np.ascontiguousarray(bufs[which][:-1])
    with pytest.raises(fa_b200.Panic, match=f"{which} shape mismatch"):
        fn(bufs["q"], bufs["k"], bufs["v"], sq, sk, d, fa_b200.FlashAttentionConfig(), bufs["out"])


@pytest.mark.parametrize("fn", [fa_b200.flash_attention_multihead_v1,
                                fa_b200.flash_attention_multihead_v2,
                                fa_b200.flash_attention_multihead_v3,
                                fa_b200.flash_attention_multihead])
def test_multihead_shape_mismatch_panics(fn):
    # tests/correctness.rs:435-459
    b, h, sq, sk, d = 2, 2, 4, 4, 8
    q = random_vec(b * h * sq * d, 1)[:-1].copy()
    k, v = random_vec(b * h * sk * d, 2), random_vec(b * h * sk * d, 3)
    out = np.zeros(b * h * sq * d, np.float32)
    with pytest.raises(fa_b200.Panic):
        fn(q, k, v, b, h, sq, sk, d, fa_b200.FlashAttentionConfig(), out)


def test_zero_sized_dimensions_leave_out_untouched():
    # tests/correctness.rs:461-504 -- returns before any device is needed.
    d = 8
    cfg = fa_b200.FlashAttentionConfig()
    e = np.zeros(0, np.float32)
    out = np.zeros(0, np.float32)
    fa_b200.flash_attention_v2(e, random_vec(4 * d, 2), random_vec(4 * d, 3), 0, 4, d, cfg, out)
    out2 = np.full(4 * d, 12.5, np.float32)
    fa_b200.flash_attention_v2(random_vec(4 * d, 4), e, e, 4, 0, d, cfg, out2)
    assert np.all(out2 == 12.5)
    fa_b200.flash_attention_v2(e, e, e, 4, 4, 0, cfg, out)


def test_no_device_fails_loudly():
    if fa_b200.device_count() > 0:
        pytest.skip("a GPU is present")
    d = 8
    out = np.zeros(4 * d, np.float32)
    with pytest.raises(fa_b200.FaError, match="FA_ERR_NO_DEVICE"):
        fa_b200.flash_attention_v2(random_vec(4 * d, 1), random_vec(4 * d, 2),
                                   random_vec(4 * d, 3), 4, 4, d,
                                   fa_b200.FlashAttentionConfig(), out)


def test_precision_control():
    old = fa_b200.get_precision()
    try:
        for p in (fa_b200.PREC_TF32, fa_b200.PREC_3XTF32, fa_b200.PREC_FP32):
            fa_b200.set_precision(p)
            assert fa_b200.get_precision() == p
        with pytest.raises(fa_b200.FaError):
            fa_b200.set_precision(7)
    finally:
        fa_b200.set_precision(old)


def test_device_entry_points_validate_before_any_device_call():
    # fa_forward_device / fa_backward_device check their arguments first, the
    # same on a host without a GPU: zero sizes return at once, null buffers
    # and d_head > 256 are argument errors.
    L = fa_b200._load()
    buf = (ctypes.c_float * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    FA_OK, FA_ERR_ARG, FA_ERR_UNSUPPORTED = 0, 2, 6
    assert L.fa_forward_device(p, p, p, p, None, 0, 4, 4, 8, 0, None) == FA_OK
    assert L.fa_forward_device(p, p, p, p, None, 1, 0, 4, 8, 0, None) == FA_OK
    assert L.fa_forward_device(None, p, p, p, None, 1, 4, 4, 8, 0, None) == FA_ERR_ARG
    assert L.fa_forward_device(p, p, p, None, None, 1, 4, 4, 8, 0, None) == FA_ERR_ARG
    assert L.fa_forward_device(p, p, p, p, None, 1, 4, 4, 257, 0, None) == FA_ERR_UNSUPPORTED
    L.fa_backward_device.restype = ctypes.c_int
    assert L.fa_backward_device(p, p, p, p, p, p, p, p, p, 0, 4, 4, 8, 0, None) == FA_OK
    assert L.fa_backward_device(p, p, p, p, None, p, p, p, p, 1, 4, 4, 8, 0, None) == FA_ERR_ARG
    assert L.fa_backward_device(p, p, p, p, p, p, p, p, p, 1, 4, 4, 129, 0,
                                None) == FA_ERR_UNSUPPORTED


def test_python_device_api_checks_tensors():
    torch = pytest.importorskip("torch")
    q = torch.zeros(2, 4, 8)
    k = torch.zeros(2, 6, 8)
    with pytest.raises(fa_b200.Panic):  # out shaped like k, not like q
        fa_b200.forward_device(q, k, k, torch.zeros(2, 6, 8))
    with pytest.raises(TypeError, match="CUDA tensor"):  # host tensors
        fa_b200.forward_device(q, k, k, torch.zeros(2, 4, 8))


def test_noalloc_refuses_before_any_device_call():
    # fa_forward_decode_noalloc checks sizes on their size_t values and the
    # 16-byte alignment its vector loads need before it touches a device, so
    # these refusals are the same on a host without a GPU, and launch nothing.
    L = fa_b200._load()
    buf = (ctypes.c_float * 1024)()
    base = ctypes.addressof(buf)
    a16 = (base + 15) & ~15
    p = ctypes.c_void_p(a16)
    odd = ctypes.c_void_p(a16 + 4)  # one float into the buffer
    FA_OK, FA_ERR_UNSUPPORTED = 0, 6
    n0 = fa_b200.launch_count()
    assert L.fa_forward_decode_noalloc(p, p, p, p, None, 0, 1, 4, 8, 0, None) == FA_OK
    for args in ((odd, p, p, p), (p, odd, p, p), (p, p, odd, p), (p, p, p, odd)):
        assert L.fa_forward_decode_noalloc(*args, None, 1, 1, 4, 8, 0, None) == FA_ERR_UNSUPPORTED
        assert b"16-byte aligned" in L.fa_last_error()
    # d_head beyond 32 bits must not wrap to an accepted value
    assert L.fa_forward_decode_noalloc(p, p, p, p, None, 1, 1, 4, (1 << 32) + 8, 0,
                                       None) == FA_ERR_UNSUPPORTED
    assert L.fa_forward_decode_noalloc(p, p, p, p, None, 1, 17, 4, 8, 0,
                                       None) == FA_ERR_UNSUPPORTED
    assert L.fa_forward_decode_noalloc(p, p, p, p, None, 65536, 1, 4, 8, 0,
                                       None) == FA_ERR_UNSUPPORTED
    assert b"batch_heads" in L.fa_last_error()
    assert L.fa_forward_decode_noalloc(p, p, p, p, None, 1, 1, 1 << 31, 8, 0,
                                       None) == FA_ERR_UNSUPPORTED
    assert b"seq_len_k" in L.fa_last_error()
    assert fa_b200.launch_count() == n0


def test_device_list_control_without_a_gpu():
    if fa_b200.device_count() > 0:
        pytest.skip("a GPU is present")
    fa_b200.set_devices([])  # returning to one device needs no GPU
    assert fa_b200.get_devices() == []
    with pytest.raises(fa_b200.FaError, match="FA_ERR_NO_DEVICE"):
        fa_b200.set_devices([0, 1])
