"""CPU checks of the MLA attention restatement (oracle) and of the C-ABI's host
rope_inv_freqs: the reference's own known-answer tests for the rope frequencies
(src/compute.rs:8556-8600), its layer rope selection, and the attention core
against a float64 softmax formula."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import wohper_b200 as W


def test_oracle_rope_yarn_known_answers():
    # yarn_scales_low_frequencies_and_keeps_high_ones (src/compute.rs:8556-8572)
    plain = O.rope_inv_freqs(64, W.DEEPSEEK_V4_COMPRESS_ROPE_THETA)
    yarn = O.rope_inv_freqs(64, W.DEEPSEEK_V4_COMPRESS_ROPE_THETA, W.DEEPSEEK_V4_YARN)
    assert len(plain) == 32 and len(yarn) == 32
    assert abs(yarn[0] - plain[0]) < 1e-6
    assert abs(yarn[31] - plain[31] / 16.0) < 1e-6 * max(1.0, plain[31])
    assert plain[20] / 16.0 < yarn[20] < plain[20]


def test_host_rope_inv_freqs_matches_the_oracle_bitwise():
    for theta, yarn in [(10000.0, None), (160000.0, W.DEEPSEEK_V4_YARN),
                        (10000.0, W.DEEPSEEK_V4_YARN), (50000.0, (4.0, 32.0, 1.0, 4096))]:
        for dim in (2, 4, 64, 128):
            a = O.rope_inv_freqs(dim, theta, yarn)
            b = W.rope_inv_freqs(dim, theta, yarn)
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_layer_rope_selection_follows_compress_ratios():
    # deepseek_layer_rope_selection_follows_compress_ratios (src/compute.rs:8574-8583)
    assert W.deepseek_rope_for_layer(0) == (10000.0, None)
    assert W.deepseek_rope_for_layer(1) == (10000.0, None)
    assert W.deepseek_rope_for_layer(2)[0] == W.DEEPSEEK_V4_COMPRESS_ROPE_THETA
    assert W.deepseek_rope_for_layer(2)[1] is not None
    assert W.deepseek_rope_for_layer(42)[0] == W.DEEPSEEK_V4_COMPRESS_ROPE_THETA
    assert W.deepseek_rope_for_layer(43) == (10000.0, None)
    assert W.deepseek_rope_for_layer(1000) == (10000.0, None)
    assert len(W.DEEPSEEK_V4_COMPRESS_RATIOS) == 44


def _f64_attention(q, keys, token_pos, window, comp, sink, inv_freqs, nope):
    heads, hd = q.shape
    start = max(0, token_pos + 1 - window)
    rows = keys[start:token_pos + 1, :hd].astype(np.float64)
    if comp is not None:
        rows = np.concatenate([rows, comp.astype(np.float64)])
    s = q.astype(np.float64) @ rows.T * hd ** -0.5
    m = s.max(1, keepdims=True)
    w = np.exp(s - m)
    den = w.sum(1, keepdims=True)
    if sink is not None:
        den = den + np.exp(sink.astype(np.float64)[:, None] - m)
    o = w @ rows / den
    ang = token_pos * inv_freqs.astype(np.float64)
    c, sn = np.cos(ang), -np.sin(ang)
    e, od = o[:, nope::2].copy(), o[:, nope + 1::2].copy()
    o[:, nope::2] = e * c - od * sn
    o[:, nope + 1::2] = e * sn + od * c
    return o


@pytest.mark.parametrize("token_pos,comp_n,use_sink", [(0, 0, False), (5, 0, True),
                                                      (200, 0, True), (300, 75, True),
                                                      (129, 3, False)])
def test_oracle_attention_matches_the_f64_formula(token_pos, comp_n, use_sink):
    rng = np.random.default_rng(token_pos * 7 + comp_n)
    heads, hd, nope, stride = 4, 512, 448, 520
    q = rng.standard_normal((heads, hd)).astype(np.float32) * 0.1
    keys = rng.standard_normal((token_pos + 1, stride)).astype(np.float32)
    comp = rng.standard_normal((comp_n, hd)).astype(np.float32) if comp_n else None
    sink = rng.standard_normal(heads).astype(np.float32) if use_sink else None
    fr = O.rope_inv_freqs(64, 160000.0, W.DEEPSEEK_V4_YARN)
    got = O.mla_attention(q, keys, token_pos, 128, comp, sink, fr, nope)
    want = _f64_attention(q, keys, token_pos, 128, comp, sink, fr, nope)
    np.testing.assert_allclose(got, want, rtol=2e-4, atol=2e-5)


def test_oracle_attention_single_position_returns_the_rotated_key():
    # one visible position and no sink: the weight is exp(0) = 1 and the output
    # is the key with the inverse RoPE applied
    rng = np.random.default_rng(3)
    q = rng.standard_normal((2, 8)).astype(np.float32)
    keys = rng.standard_normal((1, 8)).astype(np.float32)
    fr = O.rope_inv_freqs(4, 10000.0)
    got = O.mla_attention(q, keys, 0, 128, None, None, fr, 4)
    np.testing.assert_array_equal(got[0], keys[0])
    np.testing.assert_array_equal(got[1], keys[0])


def _expf_table():
    import ctypes as C

    k, v = C.c_void_p(), C.c_void_p()
    n = W.lib().wh_debug_expf_table(C.byref(k), C.byref(v))
    keys = np.ctypeslib.as_array(C.cast(k, C.POINTER(C.c_uint32)), (abs(n),)).copy()
    vals = np.ctypeslib.as_array(C.cast(v, C.POINTER(C.c_float)), (abs(n),)).copy()
    return n, keys, vals


def test_expf_lookup_band_covers_every_host_difference():
    # the device looks x up only when exp(x) lies within the band of a float
    # rounding midpoint; every input where the host expf differs from the
    # once-rounded double exp must lie well inside it
    n, keys, vals = _expf_table()
    near = W.lib().wh_debug_expf_near()
    assert 2.0 ** -44 <= near <= 2.0 ** -30
    assert np.log2(near) == np.round(np.log2(near))  # a power of two
    x = keys.view(np.float32)
    yd = np.exp(x.astype(np.float64))
    c = yd.astype(np.float32)
    differs = c.view(np.uint32) != vals.view(np.uint32)
    other = np.where(yd > c.astype(np.float64), np.nextafter(c, np.float32(np.inf)),
                     np.nextafter(c, np.float32(-np.inf))).astype(np.float64)
    dist = np.abs(yd - 0.5 * (c.astype(np.float64) + other)) / yd
    assert differs.any()
    assert dist[differs].max() <= near / 2


def test_expf_table_is_sorted_and_holds_the_host_expf():
    # the device's exp is the once-rounded double exp except at these inputs,
    # where it returns the host libm's expf (the value Rust's f32::exp gives)
    n, keys, vals = _expf_table()
    assert n > 0, "a host expf difference fell outside the device's midpoint gate"
    assert (np.diff(keys.astype(np.int64)) > 0).all()
    x = keys.view(np.float32)
    assert ((x > -104.0) & (x < 89.0)).all()
    np.testing.assert_array_equal(O.expf(x).view(np.uint32), vals.view(np.uint32))
    # every entry is a difference or a near-midpoint case: the once-rounded
    # double exp differs from the host expf on most of them
    differs = (np.exp(x.astype(np.float64)).astype(np.float32).view(np.uint32)
               != vals.view(np.uint32))
    assert differs.sum() > 0.9 * len(x)
