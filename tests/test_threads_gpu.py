"""The crate's functions are pure and callable from many threads at once
(src/v2.rs:175, src/common.rs:92); so are this library's.  Host-slice calls
from several Python threads (ctypes releases the GIL) must give exactly the
results of the same calls made one at a time."""
import threading

import numpy as np
import pytest

from fa_cases import random_vec

pytestmark = pytest.mark.gpu

# (batch_heads, seq_len_q, seq_len_k, d_head, causal): tcgen05 pair and single
# kernels, the f32 CUDA-core kernel (d = 40), split-KV decode, and one call large
# enough for the pinned staging path
SHAPES = [(2, 300, 300, 128, True), (3, 200, 100, 64, False), (1, 500, 700, 40, True),
          (4, 1, 5000, 128, False), (6, 1024, 1024, 128, True)]


def call(fa, shape, seed):
    bh, sq, sk, d, causal = shape
    q, k, v = random_vec(bh * sq * d, seed), random_vec(bh * sk * d, seed + 1), \
        random_vec(bh * sk * d, seed + 2)
    out = np.zeros(bh * sq * d, np.float32)
    fa.flash_attention_multihead_v2(q, k, v, 1, bh, sq, sk, d,
                                    fa.FlashAttentionConfig(64, 128, causal), out)
    return out


def test_concurrent_host_calls_match_serial_calls(gpu_lib):
    fa = gpu_lib
    old = fa.get_precision()
    fa.set_precision(fa.PREC_TF32)
    try:
        want = [call(fa, sh, 100 + 10 * i) for i, sh in enumerate(SHAPES)]
        got = [[None] * 3 for _ in SHAPES]
        errors = []

        def worker(i):
            try:
                for rep in range(3):
                    got[i][rep] = call(fa, SHAPES[i], 100 + 10 * i)
            except Exception as e:  # reported below
                errors.append(e)

        threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(SHAPES))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
    finally:
        fa.set_precision(old)
    assert not errors, errors
    for i in range(len(SHAPES)):
        for rep in range(3):
            assert np.array_equal(got[i][rep], want[i]), (SHAPES[i], rep)
