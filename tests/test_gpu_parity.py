"""GPU parity: every kernel, called through the C ABI, against the CPU oracle
(the reference's Rust kernels restated) on the same seeded inputs.

Integer/index work (router ids) must be identical; fp32 outputs are compared
bit for bit where the kernel reproduces the reference's association order
(FP8 GEMV, FP4 matvec, act quant, router logits, the exact expert and MoE
paths).  The exp in SiLU and in the router's softmax is the host C library's
expf reproduced on the device (a table measured at context creation), so
those outputs are bit-exact as well; the spike gate max_rel < 1e-3
(src/bin/gpu_gemv_spike.rs:201) is checked besides.  The sqrt-softplus
router's log1p is the device's correctly rounded one where the reference
calls glibc's log1pf, so its route weights are compared within 2e-6.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
KATS = json.loads((GOLD / "kats.json").read_text())
NT = json.loads((GOLD / "numpy_tool.json").read_text())


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


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---------------------------------------------------------------- act quant
@pytest.mark.parametrize("block", [64, 128, 4, 1])
@pytest.mark.parametrize("scale", [1.0, 1e-3, 37.0, 3e-5])
def test_act_quant_bit_exact(ctx, W, block, scale):
    x = H.activations(100 + block, 1, 8192, scale).reshape(-1)
    x[::97] *= 1000.0  # spread amax
    want = O.act_quant(x, block)
    t = dev(x)
    W.fp8_act_quant_dequant_in_place(ctx, t, block)
    ctx.sync()
    np.testing.assert_array_equal(bits(t.cpu().numpy()), bits(want))


def test_act_quant_numpy_tool_vectors(ctx, W):
    for v in NT["act_quant"]:
        x = np.array(v["x"], np.uint32).view(np.float32)
        t = dev(x)
        W.fp8_act_quant_dequant_in_place(ctx, t, v["block"])
        ctx.sync()
        np.testing.assert_array_equal(bits(t.cpu().numpy()), np.array(v["y"], np.uint32))


# ---------------------------------------------------------------- FP8 GEMV
def _fp8_case(seed, rows, cols):
    w, s = H.fp8_weight(seed, rows, cols)
    return w, s


def test_fp8_gemv_config1_bit_exact(ctx, W):
    rows = cols = 4096
    w, s = _fp8_case(1, rows, cols)
    x = H.activations(2, 1, cols).reshape(-1)
    st, want = O.fp8_gemv(w, s, x, rows, cols, rows // 128, cols // 128)
    assert st == O.OK
    y = W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, dev(w), dev(s), dev(x))
    ctx.sync()
    got = y.cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(want))


@pytest.mark.parametrize("shape", [(1024, 4096), (4096, 8192), (8192, 4096), (32768, 1024), (512, 128)])
def test_fp8_gemv_v4_shapes_bit_exact(ctx, W, shape):
    rows, cols = shape
    w, s = _fp8_case(rows + cols, rows, cols)
    x = H.activations(3, 1, cols).reshape(-1)
    st, want = O.fp8_gemv(w, s, x, rows, cols, rows // 128, cols // 128)
    assert st == O.OK
    y = W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, dev(w), dev(s), dev(x))
    ctx.sync()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


@pytest.mark.parametrize("batch", [1, 3, 8, 32])
def test_fp8_gemv_rows_multi_act_quant_bit_exact(ctx, W, batch):
    # grouped wo_a style row range + fused act quant, batched: every column must
    # equal the single-input result (src/compute.rs:6376-6381)
    rows, cols = 8192, 4096
    w, s = _fp8_case(5, rows, cols)
    xs = H.activations(6, batch, cols)
    xq = np.stack([O.act_quant(xs[b], 64) for b in range(batch)])
    r0, r1 = 1024, 2048 + 77
    st, want = O.fp8_gemv_multi(w, s, xq, rows, cols, rows // 128, cols // 128, r0, r1)
    assert st == O.OK
    y = W.gemv_fp8_e4m3_ue8m0_rows_multi(ctx, dev(w), dev(s), dev(xs), r0, r1, act_quant_block=64)
    ctx.sync()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


@pytest.mark.parametrize("rows,cols,batch", [(32768, 1024, 32), (1024, 4096, 17), (4096, 8192, 2),
                                             (640, 512, 40), (256, 128, 5)])
def test_fp8_gemv_batched_shapes_bit_exact(ctx, W, rows, cols, batch):
    # the batched kernel (16 inputs x 32 rows per CTA, ragged input tiles) and,
    # at 128 columns, the generic kernel; rows with 0x7F/0xFF bytes take the
    # exact recompute
    w, s = _fp8_case(rows * 7 + batch, rows, cols)
    w[3, 5] = 0x7F
    w[rows - 1, cols - 1] = 0xFF
    xs = H.activations(rows + batch, batch, cols)
    st, want = O.fp8_gemv_multi(w, s, xs, rows, cols, rows // 128, cols // 128)
    assert st == O.OK
    y = W.gemv_fp8_e4m3_ue8m0_rows_multi(ctx, dev(w), dev(s), dev(xs), 0, rows)
    ctx.sync()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


def test_fp8_gemv_nan_bytes_decode_as_480(ctx, W):
    # 0x7F / 0xFF decode to +-480 in the reference (no NaN): rows holding them
    # take the exact recompute path
    rows, cols = 256, 1024
    w, s = _fp8_case(7, rows, cols)
    w[3, 5] = 0x7F
    w[100, 1000] = 0xFF
    w[200, ::64] = 0x7F
    x = H.activations(8, 1, cols).reshape(-1)
    st, want = O.fp8_gemv(w, s, x, rows, cols, rows // 128, cols // 128)
    assert st == O.OK
    y = W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, dev(w), dev(s), dev(x))
    ctx.sync()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


def test_fp8_gemv_generic_shapes_bit_exact(ctx, W):
    # KAT shape: cols 200 = 4 groups of 50 (tail path); odd rows and row groups
    k = KATS["fp8_dot_vs_f64"]
    w = np.array(k["weight"], np.uint8).reshape(1, -1)
    s = np.array(k["scales"], np.uint8).reshape(1, -1)
    x = np.array(k["input"], np.uint32).view(np.float32)
    y = W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, dev(w), dev(s), dev(x))
    ctx.sync()
    got = float(y.cpu().numpy()[0])
    assert abs(got - k["expected_f64"]) <= k["rel_tol"] * max(abs(k["expected_f64"]), 1.0)
    st, want = O.fp8_gemv(w, s, x, 1, 200, 1, 4)
    assert bits(np.float32(got)) == bits(want)[0]
    g = np.random.default_rng(9)
    for rows, cols, sr, sc in [(37, 200, 1, 4), (96, 96, 3, 2), (64, 48, 64, 1), (30, 512, 5, 8)]:
        w = g.integers(0, 256, size=(rows, cols), dtype=np.uint8)
        s = g.integers(118, 130, size=(sr, sc), dtype=np.uint8)
        x = g.standard_normal(cols).astype(np.float32)
        st, want = O.fp8_gemv(w, s, x, rows, cols, sr, sc)
        assert st == O.OK
        y = W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, dev(w), dev(s), dev(x))
        ctx.sync()
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


def test_fp8_gemv_spike_shape_gate(ctx, W):
    # the reference's own GPU acceptance: 7168x8192, max_rel < 1e-3 vs CPU
    rows, cols = 7168, 8192
    w, s = _fp8_case(11, rows, cols)
    x = H.activations(12, 1, cols).reshape(-1)
    st, want = O.fp8_gemv(w, s, x, rows, cols, rows // 128, cols // 128)
    y = W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, dev(w), dev(s), dev(x))
    ctx.sync()
    got = y.cpu().numpy()
    assert H.max_rel_err(got, want) < KATS["spike_gate"]["max_rel"]
    np.testing.assert_array_equal(bits(got), bits(want))


def test_fp8_gemv_argument_errors(ctx, W):
    w = dev(np.zeros((256, 256), np.uint8))
    s = dev(np.full((2, 2), 127, np.uint8))
    x = dev(np.zeros(256, np.float32))
    with pytest.raises(W.WohperError) as e:
        W.gemv_fp8_e4m3_ue8m0_rows(ctx, w, dev(np.full((3, 2), 127, np.uint8)), x, 0, 256)
    assert e.value.kind == "InvalidShape"
    with pytest.raises(W.WohperError) as e:
        W.gemv_fp8_e4m3_ue8m0_rows(ctx, w, s, x, 10, 10)
    assert e.value.kind == "InvalidShape"


# ---------------------------------------------------------------- FP4 matvec
def _spec(W, packed, scales, rows, cols, scale_cols):
    return W.Fp4Matvec(dev(packed), dev(scales), rows, cols, scale_cols)


@pytest.mark.parametrize("shape", [(3, 32, 4), (2, 4, 1), (100, 512, 16), (64, 4096, 128),
                                   (33, 66, 33), (9, 7, 7), (17, 96, 3)])
def test_fp4_matvec_bit_exact(ctx, W, shape):
    rows, cols, scale_cols = shape
    g = np.random.default_rng(rows * cols)
    packed = g.integers(0, 256, size=(rows, (cols + 1) // 2), dtype=np.uint8)
    scales = g.integers(120, 130, size=(rows, scale_cols), dtype=np.uint8)
    x = g.standard_normal(cols).astype(np.float32)
    st, want = O.fp4_matvec(packed, scales, rows, cols, scale_cols, x)
    assert st == O.OK
    y = torch.zeros(rows, device="cuda")
    W.fp4_e2m1_ue8m0_matvec(ctx, _spec(W, packed, scales, rows, cols, scale_cols), dev(x), y)
    ctx.sync()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


def test_fp4_kats_through_cabi(ctx, W):
    k = KATS["fp4_low_nibble_first"]
    y = torch.zeros(2, device="cuda")
    W.fp4_e2m1_ue8m0_matvec(ctx, _spec(W, np.array(k["packed"], np.uint8),
                                       np.array(k["scales"], np.uint8), 2, 4, 1),
                            dev(np.array(k["input"], np.float32)), y)
    ctx.sync()
    np.testing.assert_allclose(y.cpu().numpy(), k["expected"], atol=k["abs_tol"], rtol=0)
    k = KATS["fp4_fast_vs_per_element"]
    x = np.array(k["input"], np.uint32).view(np.float32)
    y = torch.zeros(k["rows"], device="cuda")
    W.fp4_e2m1_ue8m0_matvec(ctx, _spec(W, np.array(k["packed"], np.uint8),
                                       np.array(k["scales"], np.uint8), k["rows"], k["cols"],
                                       k["scale_cols"]), dev(x), y)
    ctx.sync()
    want = np.array(k["expected_per_element"], np.uint32).view(np.float32)
    got = y.cpu().numpy()
    assert np.all(np.abs(got - want) <= k["rel_tol"] * np.maximum(np.abs(want), 1.0))


def _kat_expert(W, w2=None):
    k = KATS["fp4_expert_forward"]

    def mv(d):
        return _spec(W, np.array(d["packed"], np.uint8), np.array(d["scales"], np.uint8),
                     d["rows"], d["cols"], d["scale_cols"])

    return W.DeepSeekV4Fp4Expert(mv(k["w1"]), mv(k["w3"]), mv(w2 or k["w2"]))


def test_fp4_expert_forward_kat(ctx, W):
    k = KATS["fp4_expert_forward"]
    e = _kat_expert(W)
    out = torch.zeros(2, device="cuda")
    scratch = torch.zeros(2, device="cuda")
    W.deepseek_v4_fp4_expert_forward(ctx, e, dev(np.array(k["input"], np.float32)), out, scratch)
    ctx.sync()
    np.testing.assert_allclose(out.cpu().numpy(), k["expected"], atol=k["abs_tol"], rtol=0)
    with pytest.raises(W.WohperError) as err:
        W.deepseek_v4_fp4_expert_forward(ctx, e, dev(np.array(k["input"], np.float32)), out,
                                         torch.zeros(1, device="cuda"))
    assert err.value.kind == "ScratchTooSmall"


def test_fp4_nonfinite_output_is_an_error(ctx, W):
    spec = _spec(W, np.full((2, 2), 0x22, np.uint8), np.full((2, 1), 255, np.uint8), 2, 4, 1)
    y = torch.zeros(2, device="cuda")
    W.fp4_e2m1_ue8m0_matvec(ctx, spec, dev(np.ones(4, np.float32)), y)
    with pytest.raises(W.WohperError) as e:
        ctx.sync()
    assert e.value.kind == "NonFiniteOutput"
    ctx.sync()  # cleared


def test_fp4_validation_order(ctx, W):
    x = dev(np.zeros(4, np.float32))
    y = torch.zeros(2, device="cuda")
    cases = [
        (dict(rows=0), "EmptyShape"),
        (dict(cols=8), "InputTooSmall"),
        (dict(scale_cols=3), "InvalidShape"),
    ]
    for change, kind in cases:
        d = dict(packed=np.zeros((2, 2), np.uint8), scales=np.full((2, 1), 127, np.uint8),
                 rows=2, cols=4, scale_cols=1)
        d.update(change)
        with pytest.raises(W.WohperError) as e:
            W.fp4_e2m1_ue8m0_matvec(ctx, _spec(W, d["packed"], d["scales"], d["rows"], d["cols"],
                                               d["scale_cols"]), x, y)
        assert e.value.kind == kind
    with pytest.raises(W.WohperError) as e:
        W.fp4_e2m1_ue8m0_matvec(ctx, _spec(W, np.zeros((2, 2), np.uint8),
                                           np.full((2, 1), 127, np.uint8), 2, 4, 1), x,
                                torch.zeros(1, device="cuda"))
    assert e.value.kind == "OutputTooSmall"


def _oracle_expert(stack, e, keep):
    w1, s1, w3, s3, w2, s2 = [t.cpu().numpy() for t in H.expert_views(stack, e)]
    inter, hb = w1.shape
    hidden = hb * 2
    return O.Fp4Expert(O.fp4_spec(w1, s1, inter, hidden, hidden // 32, keep),
                       O.fp4_spec(w3, s3, inter, hidden, hidden // 32, keep),
                       O.fp4_spec(w2, s2, hidden, inter, inter // 32, keep))


def _w_expert(W, stack, e):
    w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
    inter, hb = w1.shape
    hidden = hb * 2
    return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, inter, hidden, hidden // 32),
                                 W.Fp4Matvec(w3, s3, inter, hidden, hidden // 32),
                                 W.Fp4Matvec(w2, s2, hidden, inter, inter // 32))


@pytest.mark.parametrize("hidden,inter", [(4096, 2048), (1024, 512), (2048, 1024)])
def test_fp4_expert_forward_fast_path_bit_exact(ctx, W, hidden, inter):
    stack = H.torch_fp4_experts(21, 1, hidden, inter)
    keep = []
    oe = _oracle_expert(stack, 0, keep)
    for seed in (22, 23):
        x = H.activations(seed, 1, hidden).reshape(-1)
        st, want = O.fp4_expert_forward(oe, x)
        assert st == O.OK
        out = torch.zeros(hidden, device="cuda")
        scratch = torch.zeros(2 * inter, device="cuda")
        W.deepseek_v4_fp4_expert_forward(ctx, _w_expert(W, stack, 0), dev(x), out, scratch)
        ctx.sync()
        got = out.cpu().numpy()
        assert H.max_rel_err(got, want, floor=1e-3 * np.abs(want).max()) < 1e-3
        nd = int(np.sum(bits(got) != bits(want)))
        assert nd == 0, f"{nd} outputs differ from the oracle"


# ---------------------------------------------------------------- router
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("E,T", [(256, 16), (256, 80), (200, 45)])  # T >= 32: batched router
def test_router_ids_bit_exact(ctx, W, mode, E, T):
    Hd, K = 4096, 6
    gate = H.router_gate(31, E, Hd)
    x = H.activations(32, T, Hd)
    bias = (np.random.default_rng(33).standard_normal(E) * 0.01).astype(np.float32) if mode else None
    logits = torch.zeros(T, E, device="cuda")
    ids, w = W.route_experts(ctx, dev(gate.view(np.int16)), dev(x), K, mode=mode,
                             bias=None if bias is None else dev(bias), route_scale=1.5,
                             logits=logits)
    ctx.sync()
    ids, w, lg = ids.cpu().numpy(), w.cpu().numpy(), logits.cpu().numpy()
    for t in range(T):
        n, oid, ow, olg = O.router(gate, x[t], K, mode=mode, bias=bias, route_scale=1.5)
        np.testing.assert_array_equal(bits(lg[t]), bits(olg))
        np.testing.assert_array_equal(ids[t], oid)
        if mode == 0:
            np.testing.assert_array_equal(bits(w[t]), bits(ow))
        else:  # log1p of the softplus is the device's, not glibc's log1pf
            np.testing.assert_allclose(w[t], ow, rtol=2e-6, atol=0)


def test_router_kats(ctx, W):
    def gate_of(rows):
        return dev(H.bf16_bits(np.array(rows, np.float32)).view(np.int16))

    k = KATS["deepseek_router"]
    ids, w = W.route_experts(ctx, gate_of(k["gate"]), dev(np.array(k["x"], np.float32)), k["topk"],
                             mode=1, route_scale=k["route_scale"])
    ctx.sync()
    assert list(ids.cpu().numpy()[0]) == k["expected_ids"]
    np.testing.assert_allclose(w.cpu().numpy()[0], k["expected_weights"], atol=k["abs_tol"])
    k = KATS["deepseek_router_bias"]
    ids, w = W.route_experts(ctx, gate_of(k["gate"]), dev(np.array(k["x"], np.float32)), k["topk"],
                             mode=1, bias=dev(np.array(k["bias"], np.float32)),
                             route_scale=k["route_scale"])
    ctx.sync()
    assert list(ids.cpu().numpy()[0]) == k["expected_ids"]
    k = KATS["deepseek_router_hash"]
    row = np.array([k["tid2eid"][k["token"]]], np.int32)
    ids, w = W.route_experts(ctx, gate_of(k["gate"]), dev(np.array(k["x"], np.float32)), k["topk"],
                             mode=1, route_scale=k["route_scale"], hash_ids=dev(row))
    ctx.sync()
    assert list(ids.cpu().numpy()[0]) == k["expected_ids"]
    assert abs(float(w.sum()) - k["total"]) < k["abs_tol"]
    k = KATS["route_weight_normalisation"]
    ids, w = W.route_experts(ctx, gate_of([[2.0], [1.0]]), dev(np.ones(1, np.float32)).view(1, 1), 2)
    ctx.sync()
    np.testing.assert_allclose(w.cpu().numpy()[0], k["legacy_expected"], atol=k["abs_tol"])


# ---------------------------------------------------------------- MoE layer (config 2)
@pytest.fixture(scope="module")
def moe_layer(ctx, W):
    E, Hd, I = 256, 4096, 2048
    stack = H.torch_fp4_experts(41, E + 1, Hd, I)
    gate = H.router_gate(42, E, Hd)
    experts = [_w_expert(W, stack, e) for e in range(E)]
    shared = _w_expert(W, stack, E)
    layer = W.MoeLayer(ctx, experts, shared, dev(gate.view(np.int16)), topk=6,
                       router_mode=W.ROUTER_RAW_LOGITS, max_tokens=4, exact=1)
    fast = W.MoeLayer(ctx, experts, shared, dev(gate.view(np.int16)), topk=6,
                      router_mode=W.ROUTER_RAW_LOGITS, max_tokens=4, exact=2)
    yield stack, gate, layer, fast
    layer.close()
    fast.close()


def test_moe_ffn_config2_vs_oracle(ctx, W, moe_layer):
    stack, gate, layer, _ = moe_layer
    E, Hd = 256, 4096
    T = 3
    x = H.activations(43, T, Hd)
    ids = torch.zeros(T, 6, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, 6, device="cuda")
    y = layer.forward(dev(x), ids=ids, weights=wts)
    ctx.sync()
    y, ids, wts = y.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    total_diff = 0
    for t in range(T):
        n, oid, ow, _ = O.router(gate, x[t], 6, mode=0)
        np.testing.assert_array_equal(ids[t], oid)
        np.testing.assert_array_equal(bits(wts[t]), bits(ow))
        keep = []
        arr = (O.Fp4Expert * (E + 1))()
        for e in list(oid) + [E]:
            arr[e] = _oracle_expert(stack, e, keep)
        st, want = O.moe_combine_token(arr, oid, ow, arr[E], x[t])
        assert st == O.OK
        scale = float(np.abs(want).max())
        assert np.max(np.abs(y[t] - want)) <= 1e-4 * scale
        total_diff += int(np.sum(bits(y[t]) != bits(want)))
    assert total_diff == 0, f"{total_diff} outputs differ from the oracle"


def test_moe_ffn_batch_equals_single_token(ctx, W, moe_layer):
    _, _, layer, _ = moe_layer
    x = dev(H.activations(44, 4, 4096))
    yb = layer.forward(x)
    ys = torch.stack([layer.forward(x[t:t + 1].contiguous()).view(-1) for t in range(4)])
    ctx.sync()
    np.testing.assert_array_equal(bits(yb.cpu().numpy()), bits(ys.cpu().numpy()))


def test_moe_ffn_decode_kernel_vs_oracle_and_three_kernels(ctx, W, moe_layer):
    """One-token calls run as the persistent decode kernel (decode.cu): the
    same outputs and routes bit for bit as the three-kernel path, over several
    tokens in a row (its grid counters and act-quant counters reset between
    calls), and within the exact path's oracle tolerance."""
    stack, gate, layer, _ = moe_layer
    E, Hd = 256, 4096
    x = H.activations(47, 6, Hd)
    outs = {}
    for fused in (True, False):
        layer.set_fused_decode(fused)
        ys, idss, wss = [], [], []
        for t in range(6):
            ids = torch.zeros(1, 6, dtype=torch.int32, device="cuda")
            wts = torch.zeros(1, 6, device="cuda")
            ys.append(layer.forward(dev(x[t:t + 1]), ids=ids, weights=wts).cpu().numpy()[0])
            idss.append(ids.cpu().numpy()[0])
            wss.append(wts.cpu().numpy()[0])
        ctx.sync()
        outs[fused] = (np.array(ys), np.array(idss), np.array(wss))
    layer.set_fused_decode(False)
    np.testing.assert_array_equal(bits(outs[True][0]), bits(outs[False][0]))
    np.testing.assert_array_equal(outs[True][1], outs[False][1])
    np.testing.assert_array_equal(bits(outs[True][2]), bits(outs[False][2]))
    y, ids = outs[True][0], outs[True][1]
    for t in range(2):
        n, oid, ow, _ = O.router(gate, x[t], 6, mode=0)
        np.testing.assert_array_equal(ids[t], oid)
        keep = []
        arr = (O.Fp4Expert * (E + 1))()
        for e in list(oid) + [E]:
            arr[e] = _oracle_expert(stack, e, keep)
        st, want = O.moe_combine_token(arr, oid, ow, arr[E], x[t])
        assert st == O.OK
        assert np.max(np.abs(y[t] - want)) <= 1e-4 * float(np.abs(want).max())


@pytest.mark.parametrize("T", [1, 3])
def test_moe_ffn_host_buffers(ctx, W, moe_layer, T):
    """x and y may be pinned host memory (the device pulls x over the bus and
    writes y back): the same bits as device buffers, on the exact and the
    tensor-core paths.  Pageable host memory is refused before any kernel runs."""
    _, _, layer, fast = moe_layer
    x = H.activations(51 + T, T, 4096)
    for lay in (layer, fast):
        want = lay.forward(dev(x))
        xh = torch.from_numpy(x).pin_memory()
        yh = torch.empty(T, 4096).pin_memory()
        lay.forward(xh, yh)
        ctx.sync()
        np.testing.assert_array_equal(bits(yh.numpy()), bits(want.cpu().numpy()))
    with pytest.raises(W.WohperError) as err:
        layer.forward(torch.from_numpy(x.copy()), torch.empty(T, 4096))
    assert err.value.kind == "InvalidPointer"


@pytest.mark.parametrize("hashed", [False, True])
def test_moe_ffn_decode_kernel_deepseek_router(ctx, W, moe_layer, hashed):
    """The decode kernel with the sqrt-softplus router (selection bias, route
    scale, optional tid2eid hash rows) equals the three-kernel path bit for bit."""
    stack, gate, _, _ = moe_layer
    E, Hd = 256, 4096
    experts = [_w_expert(W, stack, e) for e in range(E)]
    bias = dev(np.random.default_rng(48).normal(0, 0.01, E).astype(np.float32))
    layer = W.MoeLayer(ctx, experts, _w_expert(W, stack, E), dev(gate.view(np.int16)), topk=6,
                       router_mode=W.ROUTER_SQRT_SOFTPLUS, gate_bias=bias, route_scale=2.5,
                       max_tokens=1, exact=1)
    x = H.activations(49, 3, Hd)
    g = np.random.default_rng(50)
    hrows = dev(np.array([g.choice(E, 6, replace=False) for _ in range(3)], np.int32))
    outs = {}
    for fused in (True, False):
        layer.set_fused_decode(fused)
        res = []
        for t in range(3):
            ids = torch.zeros(1, 6, dtype=torch.int32, device="cuda")
            hid = hrows[t:t + 1].contiguous() if hashed else None
            y = layer.forward(dev(x[t:t + 1]), ids=ids, hash_ids=hid)
            res.append((y.cpu().numpy()[0], ids.cpu().numpy()[0]))
        ctx.sync()
        outs[fused] = res
    layer.close()
    for (ya, ia), (yb, ib) in zip(outs[True], outs[False]):
        np.testing.assert_array_equal(ia, ib)
        np.testing.assert_array_equal(bits(ya), bits(yb))


@pytest.mark.parametrize("T", [1, 3])
def test_moe_ffn_config2_tensor_core_path_vs_oracle(ctx, W, moe_layer, T):
    """Decode-sized calls on the tensor-core path (desc.exact = 2): router ids
    bit-exact; outputs through the grouped-path gate (tests/grouped_check.py:
    flips of the act-quantised hidden counted and taken out, the rest within
    the normalised error 2e-6), against the single-token combine in route
    order (moe_combine_token)."""
    from tests.grouped_check import check_grouped

    stack, gate, _, fast = moe_layer
    E, Hd = 256, 4096
    x = H.activations(44 + T, T, Hd)
    ids = torch.zeros(T, 6, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, 6, device="cuda")
    y = fast.forward(dev(x), ids=ids, weights=wts)
    ctx.sync()
    y, ids, wts = y.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    for t in range(T):
        n, oid, ow, _ = O.router(gate, x[t], 6, mode=0)
        np.testing.assert_array_equal(ids[t], oid)
        np.testing.assert_array_equal(wts[t].view(np.uint32), ow.view(np.uint32))
    check_grouped(torch, W, fast, stack, x, y, ids, wts, E, route_order=True)
