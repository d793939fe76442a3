"""Seeded synthetic inputs shared by the parity tests, smoke() and bench.py.

Distributions follow BASELINE.json's configs: FP8 weights are N(0, 0.05)
quantised to E4M3 with round-to-nearest-even, block scale exponents are
integers in [-8, -2] (exact as fp32 and as UE8M0); FP4 nibbles are uniform
0..15 with UE8M0 exponents uniform in [-6, 0]; the router weight is
N(0, 0.02) rounded to bf16; activations are N(0, 1).
"""
from __future__ import annotations

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def e4m3_bytes_from_f32(values: np.ndarray) -> np.ndarray:
    import torch

    t = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to(torch.float8_e4m3fn)
    return t.view(torch.uint8).numpy()


def fp8_weight(seed: int, rows: int, cols: int, block: int = 128):
    g = rng(seed)
    w = e4m3_bytes_from_f32(g.normal(0.0, 0.05, size=(rows, cols)).astype(np.float32))
    srows, scols = -(-rows // block), -(-cols // block)
    scale = (127 + g.integers(-8, -1, size=(srows, scols))).astype(np.uint8)  # 2^[-8,-2]
    return w, scale


def fp4_matrix(seed: int, rows: int, cols: int, group: int = 32):
    g = rng(seed)
    packed = g.integers(0, 256, size=(rows, (cols + 1) // 2), dtype=np.uint8)
    scales = (127 + g.integers(-6, 1, size=(rows, cols // group))).astype(np.uint8)
    return packed, scales


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bits."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = 0x7FFF + ((u >> 16) & 1)
    return ((u + rounding) >> 16).astype(np.uint16)


def router_gate(seed: int, experts: int, hidden: int) -> np.ndarray:
    return bf16_bits(rng(seed).normal(0.0, 0.02, size=(experts, hidden)).astype(np.float32))


def activations(seed: int, tokens: int, hidden: int, scale: float = 1.0) -> np.ndarray:
    return (rng(seed).normal(0.0, 1.0, size=(tokens, hidden)) * scale).astype(np.float32)


def torch_fp4_experts(seed: int, num: int, hidden: int, inter: int, device="cuda"):
    """num FP4 experts generated directly on the device (seeded torch RNG):
    returns dict of stacked uint8 tensors w1,w3 [num,inter,hidden/2],
    s1,s3 [num,inter,hidden/32], w2 [num,hidden,inter/2], s2 [num,hidden,inter/32]."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    u8 = dict(dtype=torch.uint8, device=device, generator=gen)

    def packed(*shape):
        return torch.randint(0, 256, shape, **u8)

    def scales(*shape):
        return torch.randint(121, 128, shape, **u8)

    return {
        "w1": packed(num, inter, hidden // 2), "s1": scales(num, inter, hidden // 32),
        "w3": packed(num, inter, hidden // 2), "s3": scales(num, inter, hidden // 32),
        "w2": packed(num, hidden, inter // 2), "s2": scales(num, hidden, inter // 32),
    }


def expert_views(stack: dict, e: int):
    """(w1, s1, w3, s3, w2, s2) tensors of expert e."""
    return tuple(stack[k][e] for k in ("w1", "s1", "w3", "s3", "w2", "s2"))


def max_rel_err(got: np.ndarray, ref: np.ndarray, floor: float = 1e-6) -> float:
    return float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)))


def zipf_routing(seed: int, gate_bits: np.ndarray, x: np.ndarray, s: float = 1.1,
                 strength: float = 0.7):
    """Zipf-skewed routing for raw-logit top-k: hidden column 0 of every token
    is set to 1.0 and gate column 0 to the prior -strength * s * ln(rank) over a
    seeded permutation of the experts, so logit_e = gate_e . x + prior_e and the
    per-expert token counts become uneven (popular experts, empty ones).  With
    the N(0, 0.02) gate (logit std 1.28 at hidden 4096), strength 0.7 gives
    counts close to Zipf(1.1) for 2048 tokens x top-6 over 256 experts
    (largest ~1300, 10th ~280, 100th ~15, a few experts with none).
    Returns (gate_bits, x) copies."""
    g = gate_bits.copy()
    x = x.copy()
    E = g.shape[0]
    ranks = np.empty(E, np.int64)
    ranks[rng(seed).permutation(E)] = np.arange(1, E + 1)
    prior = (-strength * s * np.log(ranks)).astype(np.float32)
    g[:, 0] = bf16_bits(prior)
    x[:, 0] = 1.0
    return g, x
