"""Shared test helpers: golden fixtures, weight conversion, error metrics."""
import os

import numpy as np

from oracle import bundle as B

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GGML_TYPE = {B.F32: 0, B.F16: 1, B.Q8_0: 8, B.BF16: 30}


def golden(name):
    return B.read(os.path.join(GOLDEN, name + ".b2db"))


def weight_specs(weights):
    """bundle weights -> (name, ggml type, dims, payload) for the product API."""
    return [(n, GGML_TYPE[t.dtype], t.dims, t.data) for n, t in sorted(weights.items())]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
