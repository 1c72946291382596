"""Seeded synthetic inputs standing in for the benchmark data.

The reference's benchmark data (real Qwen3-Bonsai / qwen3-zh-5k checkpoints,
MNIST) is not available offline; these generators produce data of the same
shapes and value distributions, seeded per configuration
(numpy.random.default_rng(20261201 + config_index)):
  * weights: Bernoulli(0.5) sign bits, one binary16 scale per 128 weights
    drawn from U[0.005, 0.05];
  * activations: N(0, 1) with 1% of entries multiplied by 20.
"""
import numpy as np

SEED_BASE = 20261201
GROUP = 128

# Qwen3-1.7B linear shapes (in x out) of the single-op sweep.
SWEEP_SHAPES = [(2048, 2048), (2048, 1024), (2048, 6144), (6144, 2048), (2048, 151669)]


def rng_for(config_index, salt=0):
    return np.random.default_rng(SEED_BASE + config_index + 1000 * salt)


def w1_matrix(rng, k, n, scale_lo=0.005, scale_hi=0.05):
    """(bits uint8 [n][k/8], scales uint16 [n][k/128] binary16 patterns)."""
    bits = rng.integers(0, 256, size=(n, k // 8), dtype=np.uint8)
    scales = rng.uniform(scale_lo, scale_hi, size=(n, k // GROUP)).astype(np.float16)
    return bits, scales.view(np.uint16)


def activations(rng, rows, k, outlier_frac=0.01, outlier_mul=20.0):
    x = rng.standard_normal((rows, k)).astype(np.float32)
    mask = rng.random((rows, k)) < outlier_frac
    x[mask] *= np.float32(outlier_mul)
    return x


def i8_activations(rng, rows, k):
    return rng.integers(-127, 128, size=(rows, k), dtype=np.int16).astype(np.int8)
