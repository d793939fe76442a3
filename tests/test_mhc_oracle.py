"""CPU checks of the mHC restatement (oracle/wohper_oracle.cpp, hc_*): the
reference's own tests of the hyper-connection functions (src/compute.rs:8457-8522)
and a float64 restatement of the same formulas."""
from __future__ import annotations

import numpy as np

import oracle as O


def test_sinkhorn_split_produces_doubly_normalized_comb():
    # hc_sinkhorn_split_produces_doubly_normalized_comb (src/compute.rs:8457-8486)
    hc = 4
    mix_hc = (2 + hc) * hc
    mixes = np.arange(mix_hc, dtype=np.float32) * np.float32(0.1) - np.float32(1.0)
    scale = np.array([0.5, 0.7, 0.9], np.float32)
    base = np.arange(mix_hc, dtype=np.float32) * np.float32(0.01)
    st, pre, post, comb = O.hc_split_sinkhorn(mixes, scale, base, hc, 20, 1e-6)
    assert st == O.OK
    assert ((pre > 0) & (pre < 1 + 1e-5)).all()
    assert ((post > 0) & (post < 2)).all()
    c = comb.reshape(hc, hc)
    assert (np.abs(c.sum(1) - 1) < 1e-3).all()
    assert (np.abs(c.sum(0) - 1) < 1e-3).all()


def test_hc_pre_and_post_roundtrip_shapes():
    # hc_pre_and_post_roundtrip_shapes (src/compute.rs:8488-8522)
    hc, hidden = 2, 3
    hc_dim, mix_hc = hc * hidden, (2 + hc) * hc
    fn = np.array([[(j + d) * 0.05 for d in range(hc_dim)] for j in range(mix_hc)], np.float32)
    scale = np.array([0.4, 0.6, 0.8], np.float32)
    base = np.arange(mix_hc, dtype=np.float32) * np.float32(0.02)
    x = np.arange(hc_dim, dtype=np.float32) * np.float32(0.3) - np.float32(0.5)
    st, y, post, comb = O.hc_pre(fn, scale, base, x, hc, hidden, 20, 1e-6)
    assert st == O.OK and np.isfinite(y).all()
    out = O.hc_post(y, x, post, comb, hc, hidden)
    assert np.isfinite(out).all()
    expected = post[1] * y[0] + comb[1] * x[0] + comb[hc + 1] * x[hidden]
    assert abs(out[hidden] - expected) < 1e-5 * max(1.0, abs(expected))


def test_hc_pre_size_errors():
    hc, hidden = 2, 3
    fn = np.zeros((8, 5), np.float32)  # hc_dim 5 != 6: "hc_pre sizes"
    st, *_ = O.hc_pre(fn, np.ones(3, np.float32), np.zeros(8, np.float32),
                      np.zeros(6, np.float32), hc, hidden)
    assert st == O.ERR_INVALID_SHAPE
    st, *_ = O.hc_split_sinkhorn(np.zeros(8, np.float32), np.ones(2, np.float32),
                                 np.zeros(8, np.float32), 2)  # scale shorter than 3
    assert st == O.ERR_INVALID_SHAPE


def _f64_pre(fn, scale, base, x, hc, hidden, iters, eps):
    x64 = x.astype(np.float64)
    inv = 1.0 / np.sqrt((x64 * x64).mean() + eps)
    mix = fn.astype(np.float64) @ x64 * inv
    sig = lambda v: 1.0 / (1.0 + np.exp(-v))
    pre = sig(mix[:hc] * scale[0] + base[:hc]) + eps
    post = 2.0 * sig(mix[hc:2 * hc] * scale[1] + base[hc:2 * hc])
    c = (mix[2 * hc:] * scale[2] + base[2 * hc:]).reshape(hc, hc)
    c = np.exp(c - c.max(1, keepdims=True))
    c = c / c.sum(1, keepdims=True) + eps
    c = c / (c.sum(0, keepdims=True) + eps)
    for _ in range(1, iters):
        c = c / (c.sum(1, keepdims=True) + eps)
        c = c / (c.sum(0, keepdims=True) + eps)
    y = (pre[:, None] * x64.reshape(hc, hidden)).sum(0)
    return y, post, c.reshape(-1)


def test_hc_pre_matches_the_f64_formula_at_the_v4_shape():
    rng = np.random.default_rng(4)
    hc, hidden = 4, 4096
    mix_hc = (2 + hc) * hc
    fn = (rng.standard_normal((mix_hc, hc * hidden)) * 0.01).astype(np.float32)
    scale = np.array([0.3, 0.2, 0.5], np.float32)
    base = (rng.standard_normal(mix_hc) * 0.1).astype(np.float32)
    x = rng.standard_normal(hc * hidden).astype(np.float32)
    st, y, post, comb = O.hc_pre(fn, scale, base, x, hc, hidden)
    assert st == O.OK
    wy, wp, wc = _f64_pre(fn, scale, base, x, hc, hidden, 20, 1e-6)
    np.testing.assert_allclose(y, wy, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(post, wp, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(comb, wc, rtol=1e-3, atol=1e-5)
