"""BF16 lm_head top-k on the GPU vs the oracle's restatement of
score_bf16_lm_head_topk + push_topk_candidate + the final total_cmp sort
(src/compute.rs:2838-2962): every row's logit bit-exact, and the same tokens
in the same order with the same logits, ties and NaNs included (those take the
kernel's exact replay of the reference's replacement order)."""
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


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _same(got, want):
    """Bit-equal, except that a NaN only has to be a NaN (payloads differ
    between the AVX2 oracle and the GPU)."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    np.testing.assert_array_equal(_bits(got[ok]), _bits(want[ok]))


def _weight(seed, rows, cols, std=0.02):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    w = (torch.randn(rows, cols, device="cuda", generator=g) * std).to(torch.bfloat16)
    return w.view(torch.int16)


def _run(W, ctx, w, x, k, row_base=0):
    rows = w.shape[0]
    logits = torch.empty(rows, device="cuda")
    t, v = W.lm_head_topk_score(ctx, w, x, k, row_base=row_base, logits=logits)
    ctx.sync()
    return t.cpu().numpy().astype(np.uint32), v.cpu().numpy(), logits.cpu().numpy()


def _check(W, ctx, w, x, k, row_base=0):
    tg, vg, lg = _run(W, ctx, w, x, k, row_base)
    n, to, vo, lo = O.lm_head_topk(w.cpu().numpy().view(np.uint16), x.cpu().numpy(), k, row_base)
    _same(lg, lo)
    assert n == len(tg)
    np.testing.assert_array_equal(tg, to)
    _same(vg, vo)
    return tg, vg


@pytest.mark.parametrize("k", [1, 50, 128])
def test_lm_head_deepseek_vocab_bit_exact(ctx, W, k):
    # DeepSeek-V3/V4 vocabulary x hidden: 129280 x 4096 bf16 (1.06 GB)
    w = _weight(7, 129280, 4096)
    x = torch.randn(4096, device="cuda", generator=torch.Generator(device="cuda").manual_seed(8))
    _check(W, ctx, w, x, k, row_base=0)


def test_lm_head_row_base_tail_and_small_shapes(ctx, W):
    w = _weight(9, 5000, 4104)  # 4104 = 256 chunks of 16 + an 8-column tail
    x = torch.randn(4104, device="cuda")
    _check(W, ctx, w, x, 10, row_base=100000)
    # rows < k: every row, sorted
    w2 = _weight(10, 20, 256)
    x2 = torch.randn(256, device="cuda")
    _check(W, ctx, w2, x2, 50)
    _check(W, ctx, w2, x2, 0)  # top_k.max(1)


@pytest.mark.parametrize("k", [1, 2, 3, 5, 8])
def test_lm_head_ties_follow_the_reference_replacement_order(ctx, W, k):
    # duplicate rows give equal logits inside the top k and at its boundary; the
    # reference keeps and orders them by its vector positions
    w = _weight(11, 8192, 512)
    x = torch.randn(512, device="cuda")
    _, _, lg = _run(W, ctx, w, x, 1)
    order = np.argsort(-lg, kind="stable")
    top, mid = int(order[0]), int(order[3])
    for r in (10, 500, 4097, 8000):
        w[r] = w[top]
    for r in (3, 77, 6000):
        w[r] = w[mid]
    _check(W, ctx, w, x, k)


def test_lm_head_nan_rows_and_nan_input(ctx, W):
    w = _weight(12, 4096, 256)
    x = torch.randn(256, device="cuda")
    w[123, 7] = 0x7FC0  # bf16 quiet NaN in one row
    tg, vg = _check(W, ctx, w, x, 8)
    assert 123 not in tg.tolist()  # a NaN logit never beats the minimum
    xn = x.clone()
    xn[5] = float("nan")
    tg, vg, lg = _run(W, ctx, w, xn, 4)
    n, to, vo, lo = O.lm_head_topk(w.cpu().numpy().view(np.uint16), xn.cpu().numpy(), 4)
    np.testing.assert_array_equal(tg, to)
    assert np.isnan(vg).all() and np.isnan(vo).all()


def test_lm_head_argument_errors(ctx, W):
    w = _weight(13, 64, 256)
    x = torch.randn(255, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.lm_head_topk_score(ctx, w, x, 4)
    assert e.value.kind == "InvalidShape"
    w0 = torch.empty(0, 256, dtype=torch.int16, device="cuda")
    with pytest.raises(W.WohperError) as e:
        W.lm_head_topk_score(ctx, w0, torch.randn(256, device="cuda"), 4)
    assert e.value.kind == "InvalidShape"
    wodd = _weight(14, 64, 250)
    with pytest.raises(W.WohperError) as e:
        W.lm_head_topk_score(ctx, wodd, torch.randn(250, device="cuda"), 4)
    assert e.value.kind == "Unsupported"


def test_lm_head_candidate_overflow_takes_the_replay(ctx, W):
    # all-zero rows share one histogram bin: more candidates than the selection
    # holds, so the exact replay runs.  Row 7000 replaces the first minimum of
    # the reference's vector (row 0), not the latest of the equal rows
    w = torch.zeros(20000, 256, dtype=torch.int16, device="cuda")
    w[7000, 3] = 0x3F80  # one row with logit x[3]
    x = torch.randn(256, device="cuda")
    x[3] = abs(float(x[3])) + 1.0
    tg, vg = _check(W, ctx, w, x, 5)
    assert tg.tolist() == [7000, 1, 2, 3, 4]


def _check_batch(W, ctx, w, xs, k, row_base=0):
    """The several-token call against the single-token call, token by token:
    the same tokens, logits and per-row logits, bit for bit."""
    rows = w.shape[0]
    T = xs.shape[0]
    logits = torch.empty(T, rows, device="cuda")
    tb, vb = W.lm_head_topk_score_batch(ctx, w, xs, k, row_base=row_base, logits=logits)
    ctx.sync()
    tb, vb, lb = tb.cpu().numpy().astype(np.uint32), vb.cpu().numpy(), logits.cpu().numpy()
    for t in range(T):
        ts, vs, ls = _run(W, ctx, w, xs[t], k, row_base)
        _same(lb[t], ls)
        np.testing.assert_array_equal(tb[t], ts)
        _same(vb[t], vs)
    return tb, vb


@pytest.mark.parametrize("T", [3, 9, 32])
def test_lm_head_batch_deepseek_vocab_matches_per_token(ctx, W, T):
    w = _weight(21, 129280, 4096)
    g = torch.Generator(device="cuda").manual_seed(22 + T)
    xs = torch.randn(T, 4096, device="cuda", generator=g)
    _check_batch(W, ctx, w, xs, 50)
    # one token against the oracle as well
    tb, vb = _check_batch(W, ctx, w, xs[:1], 8)
    n, to, vo, lo = O.lm_head_topk(w.cpu().numpy().view(np.uint16), xs[0].cpu().numpy(), 8)
    np.testing.assert_array_equal(tb[0], to)
    _same(vb[0], vo)


def test_lm_head_batch_tiles_strides_ties_and_nans(ctx, W):
    # 8192 and 16384 columns take 4- and 2-token tiles; a strided input; an
    # 8-column tail; duplicate rows (ties) and a NaN row and a NaN input
    for cols, T in ((8192, 7), (16384, 5), (4104, 11)):
        w = _weight(30 + T, 3000, cols)
        buf = torch.randn(T, cols + 12, device="cuda")
        xs = buf[:, :cols]
        w[17] = w[2900]
        w[400] = w[2900]
        w[1234, 5] = 0x7FC0
        xs[T - 1, 3] = float("nan")
        tb, _ = _check_batch(W, ctx, w, xs, 6, row_base=777)
        assert all(1234 + 777 not in tb[t].tolist() for t in range(T - 1))


def test_lm_head_batch_argument_errors(ctx, W):
    w = _weight(40, 64, 256)
    with pytest.raises(W.WohperError) as e:
        W.lm_head_topk_score_batch(ctx, w, torch.randn(0, 256, device="cuda"), 4)
    assert e.value.kind == "EmptyShape"
    with pytest.raises(W.WohperError) as e:
        W.lm_head_topk_score_batch(ctx, w, torch.randn(2, 256, device="cuda"), 4,
                                   scratch=torch.empty(64, dtype=torch.uint8, device="cuda"))
    assert e.value.kind == "ScratchTooSmall"
