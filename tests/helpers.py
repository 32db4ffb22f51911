"""Seeded synthetic inputs shared by the parity tests.

Q/K rows are N(0,1) per element, V is N(0,1); norm
weights are seeded around 1. The same arrays feed the oracle and the device.
"""
import numpy as np


def rng(seed):
    return np.random.default_rng(seed)


def normal(r, *shape):
    return r.standard_normal(shape).astype(np.float32)


def unit_rms_rows(x):
    """Rows rescaled to unit RMS (config 0/1 'RMS-normalised to unit RMS')."""
    x = np.asarray(x, np.float32)
    rms = np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True))
    return (x / rms).astype(np.float32)


def norm_weight(r, hd):
    return (1.0 + 0.1 * r.standard_normal(hd)).astype(np.float32)


def max_abs_diff(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))
