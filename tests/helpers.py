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


# ---------------------------------------------------------------------------
# DeepSeek-V4 decode layers with seeded synthetic weights, generated on the
# device (the attention projections as E4M3 of N(0, 0.05) with UE8M0 scales
# 2^[-8,-2], norms 1 + N(0, 0.1) in bf16, mHC parameters N(0, 0.02) / fixed
# scales, the MoE as torch_fp4_experts + an N(0, 0.02) bf16 router)
# ---------------------------------------------------------------------------
V4_SHAPES = {"wq_a": (1024, 4096), "wq_b": (32768, 1024), "wkv": (512, 4096),
             "wo_a": (8192, 4096), "wo_b": (4096, 8192)}


def _torch_gen(seed: int, device):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def torch_fp8_matrix(seed: int, rows: int, cols: int, device="cuda"):
    import torch

    g = _torch_gen(seed, device)
    w = (torch.randn(rows, cols, generator=g, device=device) * 0.05).to(torch.float8_e4m3fn)
    s = torch.randint(119, 126, (-(-rows // 128), -(-cols // 128)), dtype=torch.uint8,
                      generator=g, device=device)
    return w.view(torch.uint8), s


def torch_bf16_norm(seed: int, n: int, device="cuda"):
    import torch

    g = _torch_gen(seed, device)
    return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16).view(
        torch.int16)


def torch_hc_params(seed: int, hc: int, hidden: int, head: bool = False, device="cuda"):
    """(fn, scale, base): hc_pre's [(2+hc)*hc, hc*hidden] / [3] / [(2+hc)*hc], or
    with head=True hc_head's [hc, hc*hidden] / float / [hc]."""
    import torch

    g = _torch_gen(seed, device)
    mix = hc if head else (2 + hc) * hc
    fn = torch.randn(mix, hc * hidden, generator=g, device=device) * 0.02
    base = torch.randn(mix, generator=g, device=device) * 0.1
    if head:
        return fn, 0.5, base
    return fn, torch.tensor([0.5, 0.5, 0.5], device=device), base


def v4_layer(W, ctx, index: int, experts: int, seed: int, max_tokens: int = 1,
             router_mode: int = 0, device="cuda"):
    """One DeepSeek-V4-Flash-shape decode layer (hidden 4096, 64 heads of 512,
    q_lora 1024, 8 output groups, `experts` FP4 experts 4096 -> 2048 + shared,
    top-6).  Returns (V4LayerWeights, raw) with raw the device tensors."""
    import torch

    from wohper_b200.v4model import V4LayerWeights

    raw = {}
    mats = {}
    for i, (name, (r, c)) in enumerate(V4_SHAPES.items()):
        w, s = torch_fp8_matrix(seed * 100 + i, r, c, device)
        raw[name] = (w, s)
        mats[name] = W.Fp8Matrix(w, s)
    raw["q_norm"] = torch_bf16_norm(seed * 100 + 10, 1024, device)
    raw["kv_norm"] = torch_bf16_norm(seed * 100 + 11, 512, device)
    raw["sink"] = torch.randn(64, generator=_torch_gen(seed * 100 + 12, device), device=device)
    attn = W.V4Attention(**mats, q_norm=raw["q_norm"], kv_norm=raw["kv_norm"], sink=raw["sink"])
    raw["attn_norm"] = torch_bf16_norm(seed * 100 + 13, 4096, device)
    raw["ffn_norm"] = torch_bf16_norm(seed * 100 + 14, 4096, device)
    raw["hc_attn"] = torch_hc_params(seed * 100 + 15, 4, 4096, device=device)
    raw["hc_ffn"] = torch_hc_params(seed * 100 + 16, 4, 4096, device=device)
    stack = torch_fp4_experts(seed * 100 + 17, experts + 1, 4096, 2048, device=device)
    raw["stack"] = stack
    gate = torch.from_numpy(router_gate(seed * 100 + 18, experts, 4096).view(np.int16)).to(device)
    raw["gate"] = gate
    bias = None
    if router_mode == 1:
        bias = torch.randn(experts, generator=_torch_gen(seed * 100 + 19, device),
                           device=device) * 0.01
    raw["gate_bias"] = bias

    def wexp(e):
        w1, s1, w3, s3, w2, s2 = expert_views(stack, e)
        return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, 2048, 4096, 128),
                                     W.Fp4Matvec(w3, s3, 2048, 4096, 128),
                                     W.Fp4Matvec(w2, s2, 4096, 2048, 64))

    moe = W.MoeLayer(ctx, [wexp(e) for e in range(experts)], wexp(experts), gate, topk=6,
                     router_mode=router_mode, route_scale=1.5 if router_mode == 1 else 1.0,
                     gate_bias=bias, max_tokens=max_tokens)
    layer = V4LayerWeights(index, attn, raw["attn_norm"], raw["ffn_norm"], raw["hc_attn"],
                           raw["hc_ffn"], moe)
    return layer, raw


def v4_compressed_count(layer_index: int, token_pos: int) -> int:
    """Compressed rows visible at token_pos (src/compute.rs:3716-3719: at most
    (pos + 1) / ratio, capped at 512)."""
    from wohper_b200 import DEEPSEEK_V4_COMPRESS_RATIOS

    ratio = DEEPSEEK_V4_COMPRESS_RATIOS[layer_index] if layer_index < len(
        DEEPSEEK_V4_COMPRESS_RATIOS) else 0
    return 0 if ratio == 0 else min((token_pos + 1) // ratio, 512)
