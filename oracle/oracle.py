"""TEST INFRASTRUCTURE ONLY: ctypes loader for the C restatement in fa_oracle.c.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module, and only as the checker or the timed CPU baseline.  The product library
never calls it.  See fa_oracle.c for what it restates (reference
src/v2.rs:160-385, src/naive.rs:14-75, src/avx512.rs:113-375).

Parity pinning of this oracle: pinned to the reference's known-answer tests and
to its naive oracle; not to outputs of the reference itself (no Rust toolchain).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_BUILD = os.path.join(_HERE, "_build")
_LIB = None
_F = ctypes.POINTER(ctypes.c_float)
_D = ctypes.POINTER(ctypes.c_double)
_SZ = ctypes.c_size_t


def host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return " avx512f" in line
    except OSError:
        pass
    return False


def build() -> None:
    """Compile the restatement (both ISA tiers) into oracle/_build/."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def tier() -> str:
    return "avx512" if host_has_avx512() else "avx2"


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_BUILD, f"liboracle_{tier()}.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.oracle_exp_cephes.restype = ctypes.c_float
        L.oracle_exp_cephes.argtypes = [ctypes.c_float]
        L.oracle_flash_v2.restype = ctypes.c_int
        L.oracle_flash_v2.argtypes = [_F, _F, _F, _SZ, _SZ, _SZ, _SZ, _SZ, ctypes.c_int, _F, _F]
        L.oracle_flash_v2_multihead.restype = ctypes.c_long
        L.oracle_flash_v2_multihead.argtypes = [_F, _F, _F, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ,
                                                ctypes.c_int, _F, _F, ctypes.c_int, _SZ]
        L.oracle_flash_v2_items.restype = ctypes.c_long
        L.oracle_flash_v2_items.argtypes = [_F, _F, _F, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ,
                                            ctypes.c_int, _F, _F, ctypes.c_int,
                                            ctypes.POINTER(_SZ), _SZ]
        L.oracle_naive_f32.restype = None
        L.oracle_naive_f32.argtypes = [_F, _F, _F, _SZ, _SZ, _SZ, ctypes.c_int, _F]
        L.oracle_naive_f64_rows.restype = None
        L.oracle_naive_f64_rows.argtypes = [_F, _F, _F, _SZ, _SZ, _SZ, ctypes.c_int,
                                            _SZ, _SZ, _D, _D]
        _LIB = L
    return _LIB


def _fp(a):
    return a.ctypes.data_as(_F) if a is not None and a.size else None


def _c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def exp_cephes(x: float) -> float:
    return lib().oracle_exp_cephes(float(x))


def flash_v2(q, k, v, sq, sk, d, causal, block_q=64, block_kv=128, out=None):
    """Single-head v2 forward.  Returns (out, lse); out untouched on a zero dim."""
    q, k, v = _c32(q), _c32(k), _c32(v)
    if out is None:
        out = np.zeros(sq * d, np.float32)
    lse = np.full(max(sq, 1), -np.inf, np.float32)
    lib().oracle_flash_v2(_fp(q), _fp(k), _fp(v), sq, sk, d, block_q, block_kv,
                          int(causal), out.ctypes.data_as(_F), lse.ctypes.data_as(_F))
    return out, lse[:sq]


def flash_v2_multihead(q, k, v, bh, sq, sk, d, causal, block_q=64, block_kv=128,
                       nthreads=None, max_items=0, out=None, lse=None):
    """Multihead v2 forward over bh contiguous slices.  Returns (out, lse, items)."""
    q, k, v = _c32(q), _c32(k), _c32(v)
    if out is None:
        out = np.zeros(bh * sq * d, np.float32)
    if lse is None:
        lse = np.full(max(bh * sq, 1), -np.inf, np.float32)
    nthreads = nthreads or os.cpu_count() or 1
    items = lib().oracle_flash_v2_multihead(
        _fp(q), _fp(k), _fp(v), bh, sq, sk, d, block_q, block_kv, int(causal),
        out.ctypes.data_as(_F), lse.ctypes.data_as(_F), int(nthreads), int(max_items))
    return out, lse[: bh * sq], items


def flash_v2_items(q, k, v, bh, sq, sk, d, causal, items, block_q=64, block_kv=128,
                   nthreads=None):
    """v2 forward of the listed (head, query block) items only.

    `items` are indices head * ceil(sq / block_q) + block.  Returns (out, lse)
    as full-size arrays in which only the rows of the listed items are written
    (out zeros, lse -inf elsewhere); each computed row equals the row a full
    run produces.
    """
    q, k, v = _c32(q), _c32(k), _c32(v)
    out = np.zeros(bh * sq * d, np.float32)
    lse = np.full(max(bh * sq, 1), -np.inf, np.float32)
    it = np.ascontiguousarray(np.asarray(items, dtype=np.uint64))
    n = lib().oracle_flash_v2_items(
        _fp(q), _fp(k), _fp(v), bh, sq, sk, d, block_q, block_kv, int(causal),
        out.ctypes.data_as(_F), lse.ctypes.data_as(_F), int(nthreads or os.cpu_count() or 1),
        it.ctypes.data_as(ctypes.POINTER(_SZ)), it.size)
    if n < 0:
        raise ValueError("item out of range")
    return out, lse[: bh * sq]


def item_rows(items, sq, block_q=64):
    """Global row indices (head * sq + row) covered by the listed items."""
    nb = (sq + block_q - 1) // block_q
    rows = []
    for it in items:
        h, b = divmod(int(it), nb)
        r0 = b * block_q
        rows.extend(h * sq + r for r in range(r0, min(sq, r0 + block_q)))
    return np.asarray(rows, dtype=np.int64)


def naive_f32(q, k, v, sq, sk, d, causal):
    q, k, v = _c32(q), _c32(k), _c32(v)
    out = np.zeros(max(sq * d, 1), np.float32)
    lib().oracle_naive_f32(_fp(q), _fp(k), _fp(v), sq, sk, d, int(causal),
                           out.ctypes.data_as(_F))
    return out[: sq * d]


def naive_f64(q, k, v, sq, sk, d, causal, row0=0, row1=None):
    """f64 naive attention for rows [row0, row1).  Returns (out[rows*d], lse[rows])."""
    row1 = sq if row1 is None else row1
    q, k, v = _c32(q), _c32(k), _c32(v)
    n = row1 - row0
    out = np.zeros(max(n * d, 1), np.float64)
    lse = np.zeros(max(n, 1), np.float64)
    lib().oracle_naive_f64_rows(_fp(q), _fp(k), _fp(v), sq, sk, d, int(causal), row0,
                                row1, out.ctypes.data_as(_D), lse.ctypes.data_as(_D))
    return out[: n * d], lse[:n]


def attention_backward_f64(q, k, v, dout, sq, sk, d, causal):
    """f64 gradients (dq, dk, dv) of softmax(scale Q K^T) V for one slice.

    The reference crate has no backward pass, so this restates the calculus
    of its forward (``src/naive.rs:14-75``: scale 1/sqrt(d), top-left causal
    mask) directly: P = softmax(S), dV = P^T dO, dP = dO V^T,
    dS = P * (dP - rowsum(dO * O)), dQ = scale dS K, dK = scale dS^T Q.
    Rows that see no key have P = 0 and zero gradients.
    """
    Q = np.asarray(q, np.float64).reshape(sq, d)
    K = np.asarray(k, np.float64).reshape(sk, d)
    V = np.asarray(v, np.float64).reshape(sk, d)
    dO = np.asarray(dout, np.float64).reshape(sq, d)
    scale = 1.0 / np.sqrt(np.float32(d))
    S = (Q @ K.T) * float(scale)
    if causal:
        S = np.where(np.arange(sk)[None, :] <= np.arange(sq)[:, None], S, -np.inf)
    m = S.max(axis=1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    E = np.exp(S - m)
    l = E.sum(axis=1, keepdims=True)
    P = np.where(l > 0, E / np.where(l > 0, l, 1.0), 0.0)
    O = P @ V
    dV = P.T @ dO
    dP = dO @ V.T
    Dv = (dO * O).sum(axis=1, keepdims=True)
    dS = P * (dP - Dv)
    dQ = (dS @ K) * float(scale)
    dK = (dS.T @ Q) * float(scale)
    return dQ.ravel(), dK.ravel(), dV.ravel()
