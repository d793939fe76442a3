"""MLA attention core on the GPU vs the oracle's restatement of
compute_deepseek_v4_mla_attention's window/compressed softmax, weighted sum and
inverse RoPE (src/compute.rs:4080-4185): bit-exact at DeepSeek-V4-Flash's shape
(64 heads x 512 = 448 nope + 64 rope) across window edges, compressed-row counts,
sink on and off, YaRN and plain rope, underflowing weights and NaN keys."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HEADS, HD, NOPE = 64, 512, 448


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


def _same(got, want):
    """Bit-equal, except that a NaN only has to be a NaN."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    np.testing.assert_array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))


def _case(seed, token_pos, comp_n, stride=HD, q_scale=0.05):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((HEADS, HD)) * q_scale).astype(np.float32)
    keys = rng.standard_normal((token_pos + 1, stride)).astype(np.float32)
    comp = rng.standard_normal((comp_n, HD)).astype(np.float32) if comp_n else None
    sink = rng.standard_normal(HEADS).astype(np.float32)
    return q, keys, comp, sink


def _check(W, ctx, q, keys, token_pos, comp, sink, layer=2, window=128):
    theta, yarn = W.deepseek_rope_for_layer(layer)
    fr = W.rope_inv_freqs(HD - NOPE, theta, yarn)
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(keys).cuda()
    dc = None if comp is None else torch.from_numpy(comp).cuda()
    ds = None if sink is None else torch.from_numpy(sink).cuda()
    got = W.mla_attention(ctx, dq, dk, token_pos, fr, NOPE, window=window, compressed=dc,
                          sink=ds)
    ctx.sync()
    want = O.mla_attention(q, keys, token_pos, window, comp, sink, fr, NOPE)
    _same(got.cpu().numpy(), want)
    return want


def _device_expf(W, ctx, x):
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    yd = torch.empty_like(xd)
    W._check(W.lib().wh_debug_ref_expf(ctx.handle, xd.data_ptr(), yd.data_ptr(), xd.numel(),
                                       None))
    ctx.sync()
    return yd.cpu().numpy()


def test_device_expf_equals_the_host_libm(ctx, W):
    import ctypes as C

    k, v = C.c_void_p(), C.c_void_p()
    n = W.lib().wh_debug_expf_table(C.byref(k), C.byref(v))
    assert n > 0
    keys = np.ctypeslib.as_array(C.cast(k, C.POINTER(C.c_uint32)), (n,)).copy()
    rng = np.random.default_rng(5)
    lo_p, hi_p = 0, np.float32(89.0).view(np.uint32)
    lo_n, hi_n = 0x80000000, np.float32(-104.0).view(np.uint32)
    rand = np.concatenate([rng.integers(lo_p, hi_p, 4 << 20, dtype=np.uint32),
                           rng.integers(lo_n, hi_n, 4 << 20, dtype=np.uint32)]).view(np.float32)
    special = np.array([0.0, -0.0, 1.0, -1.0, 88.72, 88.73, 89.0, 100.0, -87.3, -103.9, -104.0,
                        -200.0, 1e-30, -1e-45, np.inf, -np.inf, np.nan], np.float32)
    for x in (keys.view(np.float32), rand, special):
        _same(_device_expf(W, ctx, x), O.expf(x))


# positions at and around the 128-row window edge; compressed rows as a ratio-4
# layer would hold them ((pos + 1) // 4), and a ratio-128 layer
@pytest.mark.parametrize("token_pos,comp_n", [(0, 0), (5, 1), (126, 31), (127, 32),
                                              (128, 32), (300, 75), (4095, 1024),
                                              (4095, 32)])
@pytest.mark.parametrize("use_sink", [True, False])
def test_mla_attention_bit_exact(ctx, W, token_pos, comp_n, use_sink):
    q, keys, comp, sink = _case(token_pos * 3 + comp_n, token_pos, comp_n)
    _check(W, ctx, q, keys, token_pos, comp, sink if use_sink else None)


def test_mla_attention_plain_rope_layer_and_wider_cache_rows(ctx, W):
    # layer 0: theta 10000, no YaRN, no compressed rows; cache rows wider than head_dim
    q, keys, comp, sink = _case(41, 200, 0, stride=HD + 64)
    _check(W, ctx, q, keys, 200, None, sink, layer=0)


def test_mla_attention_peaked_scores_underflow(ctx, W):
    # large queries: most weights underflow to zero, the max row dominates
    q, keys, comp, sink = _case(42, 400, 100, q_scale=4.0)
    want = _check(W, ctx, q, keys, 400, comp, sink)
    assert np.isfinite(want).all()


def test_mla_attention_nan_key_row(ctx, W):
    # a NaN key never becomes the max; its weight makes the sum NaN and the
    # reference then skips the division (denom > 0 is false)
    q, keys, comp, sink = _case(43, 150, 10)
    keys[140, 17] = np.nan
    want = _check(W, ctx, q, keys, 150, comp, sink)
    assert np.isnan(want).all()


def test_mla_attention_small_window(ctx, W):
    q, keys, comp, sink = _case(44, 50, 4)
    _check(W, ctx, q, keys, 50, comp, sink, window=7)


@pytest.mark.parametrize("heads,hd,nope,misalign", [(6, 96, 64, False), (3, 90, 58, False),
                                                    (64, 512, 448, True), (5, 520, 456, False)])
def test_mla_attention_other_shapes(ctx, W, heads, hd, nope, misalign):
    # head groups of 2 and 1, a partial 64-feature slice, head_dim not a multiple
    # of 4, and a query that is not 16-byte aligned (the scalar staging path)
    rng = np.random.default_rng(heads * 1000 + hd)
    q = (rng.standard_normal((heads, hd)) * 0.1).astype(np.float32)
    keys = rng.standard_normal((140, hd + 6)).astype(np.float32)
    comp = rng.standard_normal((9, hd)).astype(np.float32)
    sink = rng.standard_normal(heads).astype(np.float32)
    fr = W.rope_inv_freqs(hd - nope, 10000.0)
    if misalign:
        buf = torch.empty(q.size + 1, device="cuda")
        dq = buf[1:].view(heads, hd)
        dq.copy_(torch.from_numpy(q))
    else:
        dq = torch.from_numpy(q).cuda()
    got = W.mla_attention(ctx, dq, torch.from_numpy(keys).cuda(), 139, fr, nope,
                          compressed=torch.from_numpy(comp).cuda(),
                          sink=torch.from_numpy(sink).cuda())
    ctx.sync()
    _same(got.cpu().numpy(), O.mla_attention(q, keys, 139, 128, comp, sink, fr, nope))


def test_mla_attention_long_compressed_history(ctx, W):
    # 12,100 visible rows: the output kernel takes head groups of 2
    q, keys, comp, sink = _case(45, 99, 12000)
    _check(W, ctx, q, keys, 99, comp, sink)


def test_mla_attention_argument_errors(ctx, W):
    q = torch.zeros(HEADS, HD, device="cuda")
    k = torch.zeros(10, HD, device="cuda")
    fr = W.rope_inv_freqs(64, 10000.0)
    with pytest.raises(W.WohperError) as e:
        W.mla_attention(ctx, q, k, 5, fr, NOPE + 1)  # odd rope part
    assert e.value.kind == "InvalidShape"
    q2 = torch.zeros(2, 320, device="cuda")
    k2 = torch.zeros(10, 320, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.mla_attention(ctx, q2, k2, 5, W.rope_inv_freqs(130, 10000.0), 190)  # rope > 128
    assert e.value.kind == "Unsupported"
    q3 = torch.zeros(2, 9, device="cuda")
    k3 = torch.zeros(10, 9, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.mla_attention(ctx, q3, k3, 5, W.rope_inv_freqs(6, 10000.0), 3)  # odd nope_dim
    assert e.value.kind == "Unsupported"
    big = torch.zeros(60000, HD, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.mla_attention(ctx, q, k, 5, fr, NOPE, compressed=big)  # rows beyond shared memory
    assert e.value.kind == "Unsupported"
