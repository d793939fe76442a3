"""Seeded inputs of the numpy-tool matvec fixtures (tests/golden/numpy_tool.json).

Both the fixture generator (make_golden.py, which feeds them to the
reference's numpy tool) and the oracle test (tests/test_oracle_kats.py) build
the inputs here from the same seeds, so the fixture stores only seeds, shapes
and output bits.  numpy's default_rng (PCG64) streams are stable across numpy
versions.
"""
from __future__ import annotations

import numpy as np


def fp8_bytes(rng, n: int) -> np.ndarray:
    """E4M3 bytes with every code except the 0x7F/0xFF pair (NaN in OCP,
    +-480 in the reference's table: left out so both decoders agree)."""
    b = rng.integers(0, 254, n).astype(np.uint8)
    return np.where(b >= 0x7F, b + 1, b).astype(np.uint8)


def fp8_matvec_case(seed: int = 8101, rows: int = 256, cols: int = 512):
    """(weight [rows][cols] u8, scale [rows/128][cols/128] u8, x [cols] f32)."""
    rng = np.random.default_rng(seed)
    w = fp8_bytes(rng, rows * cols).reshape(rows, cols)
    s = rng.integers(118, 131, (rows // 128, cols // 128)).astype(np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    return w, s, x


def fp4_matvec_case(seed: int = 4101, rows: int = 256, cols: int = 512, group: int = 32):
    """(packed [rows][cols/2] u8, scale [rows][cols/group] u8, x [cols] f32)."""
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, (rows, cols // 2)).astype(np.uint8)
    s = rng.integers(121, 130, (rows, cols // group)).astype(np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    return packed, s, x


def fp4_expert_case(seed: int = 4201, hidden: int = 4096, inter: int = 2048, group: int = 32):
    """w1, w3 [inter][hidden/2], w2 [hidden][inter/2] packed with their
    [rows][cols/group] scales, and x [hidden] f32: the reference tool's fixed
    expert shape (2048 x 4096 gate/up, 4096 x 2048 down)."""
    rng = np.random.default_rng(seed)

    def mat(rows, cols):
        packed = rng.integers(0, 256, (rows, cols // 2)).astype(np.uint8)
        s = rng.integers(120, 127, (rows, cols // group)).astype(np.uint8)
        return packed, s

    w1, s1 = mat(inter, hidden)
    w3, s3 = mat(inter, hidden)
    w2, s2 = mat(hidden, inter)
    x = rng.standard_normal(hidden).astype(np.float32)
    return (w1, s1), (w3, s3), (w2, s2), x
