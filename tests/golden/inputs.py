"""Seeded inputs shared by the golden generator and the tests.

``randn`` uses numpy's legacy ``RandomState`` stream, whose output is frozen
across numpy versions, so fixtures can store seeds instead of tensors.
"""
from __future__ import annotations

import hashlib

import numpy as np


def randn(seed: int, shape) -> np.ndarray:
    return np.random.RandomState(seed).standard_normal(shape).astype(np.float32)


def digest(a: np.ndarray) -> str:
    """sha256 of the array's bytes in C order (dtype and shape are checked separately)."""
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
