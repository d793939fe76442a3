"""DeepSeek-V4's FP8 shared expert on the GPU: compute_deepseek_fp8_shared_expert_into_hidden
(src/compute.rs:5545-5614) alone, bit-exact against the oracle, and as the
shared expert of the MoE layer (y = shared(x) + routed, src/compute.rs:1940-1944)
on the exact kernels and on the tensor-core path."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import wohper_b200

    wohper_b200.lib()
    return wohper_b200


@pytest.fixture(scope="module")
def ctx(W):
    c = W.Context(0)
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _fp8_expert(seed, hidden, inter):
    """(numpy arrays, W.DeepSeekV4Fp8Expert, O.Fp8Expert, keep)."""
    import wohper_b200 as W

    w1, s1 = H.fp8_weight(seed, inter, hidden)
    w3, s3 = H.fp8_weight(seed + 1, inter, hidden)
    w2, s2 = H.fp8_weight(seed + 2, hidden, inter)
    we = W.DeepSeekV4Fp8Expert(W.Fp8Matrix(dev(w1), dev(s1)), W.Fp8Matrix(dev(w3), dev(s3)),
                               W.Fp8Matrix(dev(w2), dev(s2)))
    keep = []
    oe = O.Fp8Expert(O.fp8_matrix(w1, s1, inter, hidden, inter // 128, hidden // 128, keep),
                     O.fp8_matrix(w3, s3, inter, hidden, inter // 128, hidden // 128, keep),
                     O.fp8_matrix(w2, s2, hidden, inter, hidden // 128, inter // 128, keep))
    return we, oe, keep


@pytest.mark.parametrize("hidden,inter", [(4096, 2048), (1024, 512)])
def test_fp8_expert_forward_bit_exact(ctx, W, hidden, inter):
    we, oe, keep = _fp8_expert(21, hidden, inter)
    x = H.activations(22, 1, hidden).reshape(-1)
    y = torch.empty(hidden, device="cuda")
    scratch = torch.empty(W.lib().wh_fp8_expert_scratch_len(hidden, inter), device="cuda")
    W.deepseek_v4_fp8_expert_forward(ctx, we, dev(x), y, scratch)
    ctx.sync()
    st, want = O.fp8_expert_forward(oe, x)
    assert st == O.OK
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_fp8_expert_shape_errors(ctx, W):
    we, _, _ = _fp8_expert(23, 1024, 512)
    y = torch.empty(1024, device="cuda")
    scratch = torch.empty(4096, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.deepseek_v4_fp8_expert_forward(ctx, we, torch.randn(512, device="cuda"), y, scratch)
    assert e.value.kind == "InvalidShape" and "input dim" in str(e.value)
    with pytest.raises(W.WohperError) as e:
        W.deepseek_v4_fp8_expert_forward(ctx, we, torch.randn(1024, device="cuda"),
                                         torch.empty(512, device="cuda"), scratch)
    assert e.value.kind == "OutputTooSmall"
    bad = W.DeepSeekV4Fp8Expert(we.w1, we.w3, we.w1)  # w2.cols != w1.rows
    with pytest.raises(W.WohperError) as e:
        W.deepseek_v4_fp8_expert_forward(ctx, bad, torch.randn(1024, device="cuda"), y, scratch)
    assert e.value.kind == "InvalidShape" and "projection" in str(e.value)


E, HD, INTER = 16, 1024, 512


@pytest.fixture(scope="module")
def layer(ctx, W):
    stack = H.torch_fp4_experts(31, E, HD, INTER)
    gate = H.router_gate(32, E, HD)
    experts = []
    for e in range(E):
        w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
        experts.append(W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HD, HD // 32),
                                             W.Fp4Matvec(w3, s3, INTER, HD, HD // 32),
                                             W.Fp4Matvec(w2, s2, HD, INTER, INTER // 32)))
    we, oe, keep = _fp8_expert(33, HD, INTER)
    g = dev(gate.view(np.int16))
    exact = W.MoeLayer(ctx, experts, we, g, topk=6, max_tokens=64, exact=1)
    fast = W.MoeLayer(ctx, experts, we, g, topk=6, max_tokens=64, exact=0)
    yield stack, gate, oe, exact, fast
    exact.close()
    fast.close()


def _oracle_token(stack, gate, oe, x):
    n, oid, ow, _ = O.router(gate, x, 6, mode=0)
    keep = []
    arr = (O.Fp4Expert * E)()
    for e in oid:
        w1, s1, w3, s3, w2, s2 = [t.cpu().numpy() for t in H.expert_views(stack, int(e))]
        arr[e] = O.Fp4Expert(O.fp4_spec(w1, s1, INTER, HD, HD // 32, keep),
                             O.fp4_spec(w3, s3, INTER, HD, HD // 32, keep),
                             O.fp4_spec(w2, s2, HD, INTER, INTER // 32, keep))
    st, want = O.moe_combine_token(arr, oid, ow, None, x, shared_fp8=oe)
    assert st == O.OK
    return oid, want


def test_moe_with_fp8_shared_expert_exact_kernels(ctx, W, layer):
    stack, gate, oe, exact, _ = layer
    T = 3
    x = H.activations(34, T, HD)
    ids = torch.zeros(T, 6, dtype=torch.int32, device="cuda")
    y = exact.forward(dev(x), ids=ids)
    ctx.sync()
    y, ids = y.cpu().numpy(), ids.cpu().numpy()
    diff = 0
    for t in range(T):
        oid, want = _oracle_token(stack, gate, oe, x[t])
        np.testing.assert_array_equal(ids[t], oid)
        assert np.max(np.abs(y[t] - want)) <= 1e-4 * float(np.abs(want).max())
        diff += int(np.sum(y[t].view(np.uint32) != want.view(np.uint32)))
    assert diff == 0, f"{diff} outputs differ from the oracle"


def test_moe_with_fp8_shared_expert_tensor_cores(ctx, W, layer):
    stack, gate, oe, _, fast = layer
    T = 48
    x = H.activations(35, T, HD)
    y = fast.forward(dev(x))
    ctx.sync()
    y = y.cpu().numpy()
    for t in range(T):
        _, want = _oracle_token(stack, gate, oe, x[t])
        err = y[t] - want
        assert np.abs(err).max() <= 2e-3 * np.abs(want).max()
        assert np.sqrt((err ** 2).mean()) <= 1e-4 * np.sqrt((want ** 2).mean())


def test_moe_rejects_two_shared_experts(ctx, W, layer):
    import ctypes as C

    stack, gate, oe, exact, _ = layer
    we, _, _ = _fp8_expert(36, HD, INTER)
    w1, s1, w3, s3, w2, s2 = H.expert_views(stack, 0)
    fp4 = W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HD, HD // 32),
                                W.Fp4Matvec(w3, s3, INTER, HD, HD // 32),
                                W.Fp4Matvec(w2, s2, HD, INTER, INTER // 32))
    arr = (W.Fp4ExpertSpec * 1)(fp4.spec())
    sh4, sh8 = fp4.spec(), we.spec()
    d = W.MoeDesc(1, HD, INTER, arr, C.pointer(sh4), None, None, 1, 0, 1.0, 1, 1, C.pointer(sh8))
    h = C.c_void_p()
    st = W.lib().wh_moe_plan_create(ctx.handle, C.byref(d), C.byref(h))
    assert W.STATUS_NAMES[st] == "InvalidShape"
