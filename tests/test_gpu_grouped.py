"""Batched MoE FFN on the tensor cores (wh_moe_ffn with tokens >= 32): router
ids bit-exact with the reference router, outputs checked against the
reference's expert-major batched path (src/compute.rs:1779-1810, union in
ascending expert id, src/server/generation.rs:2487-2569), restated by the
oracle's moe_batched.

Gate (tests/grouped_check.py): the act-quantised SwiGLU hidden of every
checked row is compared with the reference's (flips counted); once the
flips' exact effect through w2 is taken out, the output is within the
normalised error |y - ref| <= 2e-6 * sum|w2 h| of every element.
"""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H
from tests.grouped_check import check_grouped

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import wohper_b200

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return wohper_b200


@pytest.fixture(scope="module")
def ctx(W):
    c = W.Context(0)
    yield c
    c.close()


def _layer(W, ctx, stack, gate_bits, E, Hd, I, max_tokens, topk=6):
    def wexp(e):
        w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
        return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, I, Hd, Hd // 32),
                                     W.Fp4Matvec(w3, s3, I, Hd, Hd // 32),
                                     W.Fp4Matvec(w2, s2, Hd, I, I // 32))

    return W.MoeLayer(ctx, [wexp(e) for e in range(E)], wexp(E),
                      torch.from_numpy(gate_bits.view(np.int16)).cuda(), topk=topk,
                      max_tokens=max_tokens)


def _check(ctx, W, layer, stack, gate, x, E, Hd, I, topk=6, sample=None):
    T = x.shape[0]
    ids = torch.zeros(T, topk, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, topk, device="cuda")
    y = layer.forward(torch.from_numpy(x).cuda(), ids=ids, weights=wts)
    ctx.sync()
    y, ids, wts = y.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    oids = np.zeros((T, topk), np.int32)
    ows = np.zeros((T, topk), np.float32)
    for t in range(T):
        _, oids[t], ows[t], _ = O.router(gate, x[t], topk, mode=0)
    np.testing.assert_array_equal(ids, oids)
    np.testing.assert_allclose(wts, ows, rtol=2e-6, atol=0)
    m = check_grouped(torch, W, layer, stack, x, y, ids, wts, E, sample=sample)
    return np.bincount(oids.reshape(-1), minlength=E), m


def test_grouped_small_layer(ctx, W):
    E, Hd, I, T = 16, 1024, 512, 64
    stack = H.torch_fp4_experts(71, E + 1, Hd, I)
    gate = H.router_gate(72, E, Hd)
    x = H.activations(73, T, Hd)
    layer = _layer(W, ctx, stack, gate, E, Hd, I, T)
    try:
        _check(ctx, W, layer, stack, gate, x, E, Hd, I)
    finally:
        layer.close()


def test_grouped_uneven_groups_multi_tile_and_empty(ctx, W):
    # Zipf-skewed routing: some experts get > 128 rows (several N tiles),
    # some get none
    E, Hd, I, T = 48, 1024, 512, 320
    stack = H.torch_fp4_experts(74, E + 1, Hd, I)
    gate, x = H.zipf_routing(75, H.router_gate(76, E, Hd), H.activations(77, T, Hd),
                            strength=1.4)
    layer = _layer(W, ctx, stack, gate, E, Hd, I, T)
    try:
        counts, _ = _check(ctx, W, layer, stack, gate, x, E, Hd, I)
    finally:
        layer.close()
    assert counts.max() > 128 and (counts == 0).sum() > 0, counts


def test_grouped_token_counts_not_multiple_of_tile(ctx, W):
    # 33 tokens (just above the grouped threshold), an odd tail in every tile
    E, Hd, I, T = 8, 512, 512, 33
    stack = H.torch_fp4_experts(78, E + 1, Hd, I)
    gate = H.router_gate(79, E, Hd)
    x = H.activations(80, T, Hd)
    layer = _layer(W, ctx, stack, gate, E, Hd, I, 64)
    try:
        _check(ctx, W, layer, stack, gate, x, E, Hd, I)
    finally:
        layer.close()


def test_grouped_v4_shape(ctx, W):
    # DeepSeek-V4-Flash expert shape (4096 -> 2048 -> 4096), 64 experts
    E, Hd, I, T = 64, 4096, 2048, 96
    stack = H.torch_fp4_experts(81, E + 1, Hd, I)
    gate, x = H.zipf_routing(82, H.router_gate(83, E, Hd), H.activations(84, T, Hd),
                            strength=1.4)
    layer = _layer(W, ctx, stack, gate, E, Hd, I, T)
    try:
        _check(ctx, W, layer, stack, gate, x, E, Hd, I)
    finally:
        layer.close()


@pytest.mark.parametrize("T", [32, 64])
def test_grouped_batched_decode_small_tiles(ctx, W, T):
    # batched decode: at most 4 routes per expert on average, so the 16-token
    # tiles run with the batched (ascending expert id) combine
    E, Hd, I = 128, 1024, 512
    stack = H.torch_fp4_experts(85 + T, E + 1, Hd, I)
    gate = H.router_gate(86, E, Hd)
    x = H.activations(87 + T, T, Hd)
    layer = _layer(W, ctx, stack, gate, E, Hd, I, T)
    try:
        _check(ctx, W, layer, stack, gate, x, E, Hd, I)
    finally:
        layer.close()


def test_grouped_v4_batch32_decode(ctx, W):
    # the decode step's batch-32 MoE: 256 V4-shape experts + shared, 32 tokens
    E, Hd, I, T = 256, 4096, 2048, 32
    stack = H.torch_fp4_experts(88, E + 1, Hd, I)
    gate = H.router_gate(89, E, Hd)
    x = H.activations(90, T, Hd)
    layer = _layer(W, ctx, stack, gate, E, Hd, I, T)
    try:
        _check(ctx, W, layer, stack, gate, x, E, Hd, I, sample=list(range(0, T, 4)))
    finally:
        layer.close()


def test_grouped_config3_shape(ctx, W):
    """BASELINE config 3 at its own shape: 256 experts + shared, 4096 -> 2048 ->
    4096, 2048 tokens with Zipf(1.1)-skewed routing (12,288 routed rows, uneven
    groups, some experts empty).  Router ids of all 2048 tokens bit-exact; the
    outputs of a seeded sample of 256 tokens through the grouped gate."""
    E, Hd, I, T = 256, 4096, 2048, 2048
    stack = H.torch_fp4_experts(85, E + 1, Hd, I)
    gate, x = H.zipf_routing(86, H.router_gate(87, E, Hd), H.activations(88, T, Hd))
    layer = _layer(W, ctx, stack, gate, E, Hd, I, T)
    sample = np.sort(np.random.default_rng(89).choice(T, 256, replace=False))
    try:
        counts, m = _check(ctx, W, layer, stack, gate, x, E, Hd, I, sample=sample)
    finally:
        layer.close()
    assert counts.sum() == T * 6 and counts.max() > 128 and (counts == 0).sum() > 0, counts
