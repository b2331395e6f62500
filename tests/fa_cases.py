"""Test inputs shared by the CPU and GPU suites.

`REFERENCE_CASES` is the shape matrix of the crate's integration tests
(tests/correctness.rs:115-237): (seq_q, seq_k, d, block_q, block_kv, causal).
The crate draws uniform(-1, 1) values from Rust's StdRng, a stream that cannot
be reproduced without Rust; these tests draw the same distribution from numpy
with fixed seeds (no reference test pins exact values).

`BASELINE_CONFIGS` are the five workloads of the benchmark: numpy
default_rng(seed).standard_normal drawn in the order Q, K, V, times a factor.
"""
import numpy as np

REFERENCE_CASES = [
    # matches_naive_exact_block_multiples (:115-121)
    (64, 64, 64, 32, 32, False), (128, 128, 64, 64, 64, False),
    # matches_naive_ragged_sizes (:123-135)
    (17, 23, 32, 8, 8, False), (1, 1, 16, 8, 8, False), (1, 50, 33, 16, 16, False),
    (50, 1, 33, 16, 16, False), (97, 131, 17, 32, 40, False), (200, 200, 128, 64, 128, False),
    # block_size_q_not_a_multiple_of_four (:137-152)
    *[(23, 29, 24, br, 12, c) for br in (3, 5, 6, 7) for c in (False, True)],
    # block_size_kv_not_a_multiple_of_four (:154-171)
    *[(29, 23, 24, 12, bc, c) for bc in (3, 5, 6, 7) for c in (False, True)],
    # matches_naive_causal (:173-181)
    (64, 64, 64, 32, 32, True), (97, 97, 33, 16, 24, True), (1, 1, 16, 8, 8, True),
    (5, 5, 8, 64, 64, True),
    # matches_naive_causal_asymmetric_seq_lens (:183-194)
    (10, 40, 32, 4, 8, True),
    # single_block_bigger_than_everything (:196-202)
    (10, 10, 8, 1024, 1024, False), (10, 10, 8, 1024, 1024, True),
]

# v1_v2_v3_mutually_agree (:295-375)
AGREEMENT_CASES = [
    (64, 64, 64, 32, 32, False), (97, 131, 17, 32, 40, True), (5, 5, 8, 64, 64, True),
    (200, 200, 128, 64, 128, True),
]

# Shapes the tensor-core kernels tile (d = 32, 64, 96, 128), ragged and causal, incl. Sq != Sk.
TC_CASES = [
    (128, 128, 64, True), (128, 128, 128, True), (200, 200, 128, True), (200, 200, 128, False),
    (300, 77, 64, False), (77, 300, 64, True), (77, 300, 128, True), (513, 1000, 128, True),
    (1000, 513, 64, True), (256, 4096, 128, False), (4096, 256, 64, True), (130, 130, 64, False),
    (33, 700, 128, True), (700, 33, 128, False), (129, 129, 128, True),
    # d = 32 and 96 (the crate's tests use 32; 96 is a common head size): the
    # single-CTA tcgen05 kernels at every length
    (128, 128, 32, True), (513, 1000, 32, True), (77, 300, 32, False), (300, 77, 96, False),
    (200, 200, 96, True), (1000, 513, 96, True), (2048, 2048, 96, False), (100, 5000, 96, True),
]


def random_vec(n, seed):
    """uniform(-1, 1) float32, like the crate's random_vec (tests/correctness.rs:63-66)."""
    return np.random.default_rng(0xC0FFEE ^ seed).uniform(-1.0, 1.0, n).astype(np.float32)


# name: (bh, sq, sk, d, causal, seed, factor)
BASELINE_CONFIGS = {
    "c1": (1, 512, 512, 64, False, 0, 1.0),
    "c2": (32, 4096, 4096, 128, True, 1, 0.5),
    "c3": (256, 1024, 1024, 64, False, 2, 1.0),
    "c4": (64, 1, 32768, 128, False, 3, 1.0),
    "c5": (1, 131072, 131072, 128, True, 4, 0.3),
}


def baseline_inputs(name, bh=None):
    """Q, K, V (flat float32) of a benchmark config; `bh` overrides the slice count."""
    cbh, sq, sk, d, causal, seed, factor = BASELINE_CONFIGS[name]
    bh = cbh if bh is None else bh
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal(bh * sq * d, dtype=np.float32) * np.float32(factor))
    k = (rng.standard_normal(bh * sk * d, dtype=np.float32) * np.float32(factor))
    v = (rng.standard_normal(bh * sk * d, dtype=np.float32) * np.float32(factor))
    return q, k, v, (bh, sq, sk, d, causal)


def max_abs_diff(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0
