"""mHC hyper-connections on the GPU vs the oracle's restatement of hc_pre_into,
hc_split_sinkhorn_scalar, hc_post_into and hc_head_pool (src/compute.rs:4945-5132):
bit-exact at DeepSeek-V4's shape (hc 4 x hidden 4096) for one and several tokens,
at small and ragged shapes (scalar path), with a NaN input, and the errors."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

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


def _same(got, want):
    """Bit-equal, except that a NaN only has to be a NaN."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    np.testing.assert_array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))


def _params(seed, hc, hidden, rows=None):
    rng = np.random.default_rng(seed)
    rows = (2 + hc) * hc if rows is None else rows
    fn = (rng.standard_normal((rows, hc * hidden)) * 0.01).astype(np.float32)
    scale = np.array([0.3, 0.2, 0.5], np.float32)
    base = (rng.standard_normal(rows) * 0.1).astype(np.float32)
    return fn, scale, base


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _check_pre_post(W, ctx, hc, hidden, T, seed, x=None, iters=20):
    fn, scale, base = _params(seed, hc, hidden)
    rng = np.random.default_rng(seed + 1)
    if x is None:
        x = rng.standard_normal((T, hc * hidden)).astype(np.float32)
    res = rng.standard_normal((T, hc * hidden)).astype(np.float32)
    y, post, comb = W.hc_pre(ctx, _dev(fn), _dev(scale), _dev(base), _dev(x), hc, hidden,
                             sinkhorn_iters=iters)
    out = W.hc_post(ctx, y, _dev(res), post, comb, hc, hidden)
    ctx.sync()
    y, post, comb, out = (v.cpu().numpy() for v in (y, post, comb, out))
    for t in range(T):
        st, oy, op, oc = O.hc_pre(fn, scale, base, x[t], hc, hidden, iters, 1e-6)
        assert st == O.OK
        _same(y[t], oy)
        _same(post[t], op)
        _same(comb[t].reshape(-1), oc)
        # hc_post checked on the device's own y/post/comb (equal to the oracle's)
        _same(out[t], O.hc_post(y[t], res[t], post[t], comb[t].reshape(-1), hc, hidden))
    return y


@pytest.mark.parametrize("T", [1, 3, 16, 40])
def test_hc_pre_post_v4_shape_bit_exact(ctx, W, T):
    _check_pre_post(W, ctx, 4, 4096, T, 10 + T)


@pytest.mark.parametrize("hc,hidden,iters", [(2, 3, 20), (3, 7, 5), (4, 130, 1), (8, 64, 20),
                                             (1, 33, 0)])
def test_hc_pre_post_small_and_ragged(ctx, W, hc, hidden, iters):
    # hc * hidden not a multiple of 4 takes the scalar chain; 8 copies use 81 chains
    _check_pre_post(W, ctx, hc, hidden, 2, 100 + hc * hidden, iters=iters)


def test_hc_pre_nan_input(ctx, W):
    hc, hidden = 4, 256
    x = np.random.default_rng(3).standard_normal((1, hc * hidden)).astype(np.float32)
    x[0, 17] = np.nan
    _check_pre_post(W, ctx, hc, hidden, 1, 7, x=x)


@pytest.mark.parametrize("hc,hidden,T", [(4, 4096, 2), (3, 11, 1), (4, 256, 33)])
def test_hc_head_bit_exact(ctx, W, hc, hidden, T):
    fn, _, base = _params(21, hc, hidden, rows=hc)
    x = np.random.default_rng(22).standard_normal((T, hc * hidden)).astype(np.float32)
    got = W.hc_head(ctx, _dev(fn), 0.7, _dev(base), _dev(x), hc, hidden)
    ctx.sync()
    got = got.cpu().numpy()
    for t in range(T):
        _same(got[t], O.hc_head(fn, 0.7, base, x[t], hc, hidden, 1e-6))


def test_hc_argument_errors(ctx, W):
    fn, scale, base = _params(1, 4, 16)
    x = torch.zeros(1, 64, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.hc_pre(ctx, _dev(fn), _dev(scale), _dev(base), x, 9, 16)
    assert e.value.kind == "Unsupported"
    with pytest.raises(W.WohperError) as e:
        W.hc_pre(ctx, _dev(fn), _dev(scale), _dev(base), x, 4, 16, sinkhorn_iters=-1)
    assert e.value.kind == "InvalidShape"
    with pytest.raises(W.WohperError) as e:
        W.hc_pre(ctx, None, _dev(scale), _dev(base), x, 4, 16)
    assert e.value.kind == "InvalidPointer"
