"""Python mirror of the `flash-attention-cpu` crate's public API over the B200 C ABI.

Same names, argument order and meaning as the crate (src/lib.rs:78-87):

    FlashAttentionConfig(block_size_q=64, block_size_kv=128, causal=False)
    flash_attention_v1 / _v2 / _v3(q, k, v, seq_len_q, seq_len_k, d_head, config, out)
    flash_attention_multihead_v1 / _v2 / _v3(q, k, v, batch, heads, seq_len_q,
                                             seq_len_k, d_head, config, out)
    flash_attention = flash_attention_v2
    flash_attention_multihead = flash_attention_multihead_v2

Buffers are flat float32 numpy arrays (the crate's `&[f32]` / `&mut [f32]`);
`out` is written in place.  Where the crate panics (a shape mismatch,
src/common.rs:51-54, 87-90) these functions raise `Panic` (an AssertionError)
with the same message; a zero dimension returns without touching `out`
(src/common.rs:56).  Every call runs on the GPU through lib/libfa_b200.so; if
the library or a GPU is missing the call raises -- there is no CPU path.

Beyond the crate: `multihead_lse` (output plus row log-sum-exp), the
device-resident calls on torch CUDA tensors (`forward_device`,
`forward_partial_device`, `lse_combine_device`), and library control
(`set_precision`, `launch_count`, `last_path`, `sync_status`).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

__all__ = [
    "FlashAttentionConfig", "Panic", "FaError",
    "flash_attention_v1", "flash_attention_v2", "flash_attention_v3", "flash_attention",
    "flash_attention_multihead_v1", "flash_attention_multihead_v2",
    "flash_attention_multihead_v3", "flash_attention_multihead",
    "multihead_lse", "forward_device", "forward_decode_noalloc", "forward_partial_device", "lse_combine_device",
    "set_precision", "get_precision", "launch_count", "last_path", "sync_status",
    "device_count", "set_device", "set_devices", "get_devices", "lib_path", "PREC_TF32", "PREC_3XTF32", "PREC_FP32",
]

PREC_TF32, PREC_3XTF32, PREC_FP32 = 0, 1, 2
_STATUS = {0: "FA_OK", 1: "FA_ERR_SHAPE", 2: "FA_ERR_ARG", 3: "FA_ERR_CUDA",
           4: "FA_ERR_TIMEOUT", 5: "FA_ERR_NO_DEVICE", 6: "FA_ERR_UNSUPPORTED"}

_PKG = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(os.path.dirname(_PKG), "lib", "libfa_b200.so")


class Panic(AssertionError):
    """Raised where the crate would panic (shape-contract violations)."""


class FaError(RuntimeError):
    """A non-shape failure reported by the C ABI (no device, CUDA error, timeout)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS.get(status, status)}: {message}")
        self.status = status


@dataclass
class FlashAttentionConfig:
    """Mirrors FlashAttentionConfig (src/common.rs:16-36); Default = 64 / 128 / False."""
    block_size_q: int = 64
    block_size_kv: int = 128
    causal: bool = False


class _CConfig(ctypes.Structure):
    _fields_ = [("block_size_q", ctypes.c_size_t), ("block_size_kv", ctypes.c_size_t),
                ("causal", ctypes.c_uint8)]


_lib = None
_SZ = ctypes.c_size_t
_P = ctypes.c_void_p


def lib_path() -> str:
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise FaError(5, f"{_LIB_PATH} is not built (run __graft_entry__.build()); "
                         "there is no CPU fallback")
    L = ctypes.CDLL(_LIB_PATH)
    single = [_P, _SZ, _P, _SZ, _P, _SZ, _SZ, _SZ, _SZ, ctypes.POINTER(_CConfig), _P, _SZ]
    multi = [_P, _SZ, _P, _SZ, _P, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, ctypes.POINTER(_CConfig), _P,
             _SZ]
    for n in ("fa_flash_attention_v1", "fa_flash_attention_v2", "fa_flash_attention_v3",
              "fa_flash_attention"):
        getattr(L, n).argtypes = single
        getattr(L, n).restype = ctypes.c_int
    for n in ("fa_flash_attention_multihead_v1", "fa_flash_attention_multihead_v2",
              "fa_flash_attention_multihead_v3", "fa_flash_attention_multihead"):
        getattr(L, n).argtypes = multi
        getattr(L, n).restype = ctypes.c_int
    L.fa_flash_attention_multihead_lse.argtypes = [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_int,
                                                   _P, _P]
    L.fa_flash_attention_multihead_lse.restype = ctypes.c_int
    L.fa_forward_device.argtypes = [_P, _P, _P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_int, _P]
    L.fa_forward_device.restype = ctypes.c_int
    L.fa_forward_partial_device.argtypes = [_P, _P, _P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_int,
                                            _SZ, _SZ, _P]
    L.fa_forward_partial_device.restype = ctypes.c_int
    L.fa_forward_decode_noalloc.argtypes = [_P, _P, _P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_int, _P]
    L.fa_forward_decode_noalloc.restype = ctypes.c_int
    L.fa_lse_combine_device.argtypes = [_P, _P, _SZ, _SZ, _SZ, _P, _P, _P]
    L.fa_lse_combine_device.restype = ctypes.c_int
    L.fa_sync_status.argtypes = [_P]
    L.fa_sync_status.restype = ctypes.c_int
    L.fa_set_precision.argtypes = [ctypes.c_int]
    L.fa_set_precision.restype = ctypes.c_int
    L.fa_get_precision.restype = ctypes.c_int
    L.fa_set_device.argtypes = [ctypes.c_int]
    L.fa_set_device.restype = ctypes.c_int
    L.fa_device_count.restype = ctypes.c_int
    L.fa_set_devices.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    L.fa_set_devices.restype = ctypes.c_int
    L.fa_get_devices.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    L.fa_get_devices.restype = ctypes.c_int
    L.fa_last_error.restype = ctypes.c_char_p
    L.fa_last_path.restype = ctypes.c_char_p
    L.fa_launch_count.restype = ctypes.c_uint64
    L.fa_config_default.restype = _CConfig
    L.fa_backward_device.argtypes = [_P] * 9 + [_SZ, _SZ, _SZ, _SZ, ctypes.c_int, _P]
    L.fa_backward_device.restype = ctypes.c_int
    L.fa_flash_attention_backward.argtypes = [_P] * 9 + [_SZ, _SZ, _SZ, _SZ, ctypes.c_int]
    L.fa_flash_attention_backward.restype = ctypes.c_int
    L.fa_test_stall.argtypes = [ctypes.c_int, ctypes.c_ulonglong]
    L.fa_test_stall.restype = ctypes.c_int
    L.fa_pin_host.argtypes = [_P, _SZ]
    L.fa_pin_host.restype = ctypes.c_int
    L.fa_unpin_host.argtypes = [_P]
    L.fa_unpin_host.restype = ctypes.c_int
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc == 0:
        return
    msg = _load().fa_last_error().decode()
    if rc == 1:
        raise Panic(msg)
    raise FaError(rc, msg)


def _buf(a, name: str, writable: bool = False):
    """Pointer and length of a flat float32 buffer (the crate's &[f32])."""
    if not isinstance(a, np.ndarray) or a.dtype != np.float32:
        raise TypeError(f"{name} must be a float32 numpy array")
    if not a.flags.c_contiguous:
        raise TypeError(f"{name} must be C-contiguous")
    if writable and not a.flags.writeable:
        raise TypeError(f"{name} must be writable")
    return (a.ctypes.data if a.size else None), a.size


def _cfg(config):
    config = config or FlashAttentionConfig()
    return _CConfig(int(config.block_size_q), int(config.block_size_kv), 1 if config.causal else 0)


def _single(name):
    def fn(q, k, v, seq_len_q, seq_len_k, d_head, config, out):
        L = _load()
        qp, ql = _buf(q, "q")
        kp, kl = _buf(k, "k")
        vp, vl = _buf(v, "v")
        op, ol = _buf(out, "out", True)
        c = _cfg(config)
        _check(getattr(L, name)(qp, ql, kp, kl, vp, vl, seq_len_q, seq_len_k, d_head,
                                ctypes.byref(c), op, ol))
    fn.__name__ = name[3:]
    fn.__doc__ = (f"Drop-in for the crate's `{name[3:]}` (single head, host slices); "
                  "writes `out` in place.")
    return fn


def _multi(name):
    def fn(q, k, v, batch, heads, seq_len_q, seq_len_k, d_head, config, out):
        L = _load()
        qp, ql = _buf(q, "q")
        kp, kl = _buf(k, "k")
        vp, vl = _buf(v, "v")
        op, ol = _buf(out, "out", True)
        c = _cfg(config)
        _check(getattr(L, name)(qp, ql, kp, kl, vp, vl, batch, heads, seq_len_q, seq_len_k,
                                d_head, ctypes.byref(c), op, ol))
    fn.__name__ = name[3:]
    fn.__doc__ = (f"Drop-in for the crate's `{name[3:]}` ([batch, heads, seq, d] host slices); "
                  "writes `out` in place.")
    return fn


flash_attention_v1 = _single("fa_flash_attention_v1")
flash_attention_v2 = _single("fa_flash_attention_v2")
flash_attention_v3 = _single("fa_flash_attention_v3")
flash_attention = _single("fa_flash_attention")
flash_attention_multihead_v1 = _multi("fa_flash_attention_multihead_v1")
flash_attention_multihead_v2 = _multi("fa_flash_attention_multihead_v2")
flash_attention_multihead_v3 = _multi("fa_flash_attention_multihead_v3")
flash_attention_multihead = _multi("fa_flash_attention_multihead")


def multihead_lse(q, k, v, batch_heads, seq_len_q, seq_len_k, d_head, causal, out=None):
    """Host-slice multihead forward that also returns the row LSE: (out, lse)."""
    L = _load()
    if out is None:
        out = np.zeros(batch_heads * seq_len_q * d_head, np.float32)
    lse = np.full(max(batch_heads * seq_len_q, 1), -np.inf, np.float32)
    qp, _ = _buf(q, "q")
    kp, _ = _buf(k, "k")
    vp, _ = _buf(v, "v")
    op, _ = _buf(out, "out", True)
    for name, a, n in (("q", q, batch_heads * seq_len_q * d_head),
                       ("k", k, batch_heads * seq_len_k * d_head),
                       ("v", v, batch_heads * seq_len_k * d_head),
                       ("out", out, batch_heads * seq_len_q * d_head)):
        if a.size != n:
            raise Panic(f"multihead {name} shape mismatch")
    _check(L.fa_flash_attention_multihead_lse(qp, kp, vp, batch_heads, seq_len_q, seq_len_k,
                                              d_head, int(bool(causal)), op, lse.ctypes.data))
    return out, lse[: batch_heads * seq_len_q]


# ---- device-resident calls on torch CUDA tensors -----------------------------

def _dptr(t, name):
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32:
        raise TypeError(f"{name} must be a float32 CUDA tensor")
    if not t.is_contiguous():
        raise TypeError(f"{name} must be contiguous")
    return t.data_ptr()


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def forward_device(q, k, v, out, lse=None, causal=False, stream=None):
    """Enqueue the forward on device tensors q,out [bh, sq, d], k,v [bh, sk, d]."""
    bh, sq, d = q.shape
    sk = k.shape[1]
    if tuple(k.shape) != (bh, sk, d) or tuple(v.shape) != (bh, sk, d) or \
            tuple(out.shape) != (bh, sq, d):
        raise Panic("device shape mismatch")
    _check(_load().fa_forward_device(_dptr(q, "q"), _dptr(k, "k"), _dptr(v, "v"),
                                     _dptr(out, "out"),
                                     _dptr(lse, "lse") if lse is not None else None,
                                     bh, sq, sk, d, int(bool(causal)), _stream(stream)))


def forward_partial_device(q, k, v, out, lse, causal, q_offset, k_offset, stream=None):
    """Partial forward over the key range in k/v starting at global key k_offset."""
    bh, sq, d = q.shape
    sk = k.shape[1]
    _check(_load().fa_forward_partial_device(
        _dptr(q, "q"), _dptr(k, "k"), _dptr(v, "v"), _dptr(out, "out"), _dptr(lse, "lse"),
        bh, sq, sk, d, int(bool(causal)), int(q_offset), int(k_offset), _stream(stream)))


def forward_decode_noalloc(q, k, v, out, lse=None, causal=False, stream=None):
    """Decode forward (seq_len_q <= 16) that allocates no device memory: the
    split partials use the library's fixed device array.  For callers that may
    not allocate while running; calls that overlap on one GPU race."""
    bh, sq, d = q.shape
    sk = k.shape[1]
    if tuple(k.shape) != (bh, sk, d) or tuple(v.shape) != (bh, sk, d) or \
            tuple(out.shape) != (bh, sq, d):
        raise Panic("device shape mismatch")
    _check(_load().fa_forward_decode_noalloc(
        _dptr(q, "q"), _dptr(k, "k"), _dptr(v, "v"), _dptr(out, "out"),
        _dptr(lse, "lse") if lse is not None else None, bh, sq, sk, d, int(bool(causal)),
        _stream(stream)))


def lse_combine_device(o_parts, lse_parts, out, lse_out=None, stream=None):
    """Merge partials o_parts [n, rows, d], lse_parts [n, rows] into out [rows, d]."""
    n, rows, d = o_parts.shape
    _check(_load().fa_lse_combine_device(
        _dptr(o_parts, "o_parts"), _dptr(lse_parts, "lse_parts"), n, rows, d,
        _dptr(out, "out"), _dptr(lse_out, "lse_out") if lse_out is not None else None,
        _stream(stream)))


# ---- library control ---------------------------------------------------------

def set_precision(p: int) -> None:
    _check(_load().fa_set_precision(int(p)))


def get_precision() -> int:
    return _load().fa_get_precision()


def set_device(dev: int) -> None:
    _check(_load().fa_set_device(int(dev)))


def set_devices(devices) -> None:
    """Devices the host-slice calls spread over (fa_set_devices): a list of
    device indices (repeats allowed), [] for one device."""
    devs = [int(x) for x in devices]
    arr = (ctypes.c_int * max(1, len(devs)))(*devs)
    _check(_load().fa_set_devices(arr, len(devs)))


def get_devices() -> list:
    L = _load()
    n = L.fa_get_devices(None, 0)
    arr = (ctypes.c_int * max(1, n))()
    L.fa_get_devices(arr, n)
    return [arr[i] for i in range(n)]


def device_count() -> int:
    return _load().fa_device_count()


def launch_count() -> int:
    return int(_load().fa_launch_count())


def backward_device(q, k, v, out, lse, dout, dq, dk, dv, causal=False, stream=None):
    """Gradients dq, dk, dv of the forward (device tensors; q/out/dout/dq [bh, sq, d],
    k/v/dk/dv [bh, sk, d], lse [bh, sq] from the forward).  Asynchronous."""
    bh, sq, d = q.shape
    sk = k.shape[1]
    for name, t, shape in (("k", k, (bh, sk, d)), ("v", v, (bh, sk, d)), ("out", out, (bh, sq, d)),
                           ("dout", dout, (bh, sq, d)), ("dq", dq, (bh, sq, d)),
                           ("dk", dk, (bh, sk, d)), ("dv", dv, (bh, sk, d))):
        if tuple(t.shape) != shape:
            raise Panic(f"{name} shape mismatch")
    _check(_load().fa_backward_device(
        _dptr(q, "q"), _dptr(k, "k"), _dptr(v, "v"), _dptr(out, "out"), _dptr(lse, "lse"),
        _dptr(dout, "dout"), _dptr(dq, "dq"), _dptr(dk, "dk"), _dptr(dv, "dv"),
        bh, sq, sk, d, int(bool(causal)), _stream(stream)))


def flash_attention_backward(q, k, v, out, lse, dout, batch_heads, seq_len_q, seq_len_k, d_head,
                             causal=False):
    """Host-buffer backward: returns (dq, dk, dv) as new float32 arrays."""
    import numpy as np
    nq, nk = batch_heads * seq_len_q * d_head, batch_heads * seq_len_k * d_head
    arrs = [np.ascontiguousarray(a, np.float32) for a in (q, k, v, out, lse, dout)]
    want = (nq, nk, nk, nq, batch_heads * seq_len_q, nq)
    for name, a, n in zip(("q", "k", "v", "out", "lse", "dout"), arrs, want):
        if a.size != n:
            raise Panic(f"{name} shape mismatch")
    dq, dk, dv = np.zeros(nq, np.float32), np.zeros(nk, np.float32), np.zeros(nk, np.float32)
    _check(_load().fa_flash_attention_backward(
        *(a.ctypes.data for a in arrs), dq.ctypes.data, dk.ctypes.data, dv.ctypes.data,
        batch_heads, seq_len_q, seq_len_k, d_head, int(bool(causal))))
    return dq, dk, dv


def pin_host(arr) -> None:
    """Page-lock a numpy array's memory (fa_pin_host) for fast host-slice calls."""
    _check(_load().fa_pin_host(arr.ctypes.data, arr.nbytes))


def unpin_host(arr) -> None:
    """Undo pin_host for the same array."""
    _check(_load().fa_unpin_host(arr.ctypes.data))


def test_stall(skip_block: int, wait_ns: int = 0) -> None:
    """Failure-path test hook (fa_test_stall): with skip_block >= 0 the next
    tensor-core launches withhold one softmax arrive on that key block, so
    their bounded wait runs out after wait_ns (0: the default 2 s) and the
    call reports FA_ERR_TIMEOUT.  test_stall(-1) restores normal operation."""
    _check(_load().fa_test_stall(int(skip_block), int(wait_ns)))


def last_path() -> str:
    return _load().fa_last_path().decode()


def sync_status(stream=None) -> None:
    """Wait for `stream` and raise if a kernel hit its bounded-wait limit."""
    _check(_load().fa_sync_status(_stream(stream)))
