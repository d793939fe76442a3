"""Parity gate of the tensor-core (grouped) MoE path against the oracle.

The grouped GEMMs multiply exactly (FP4 weights as E4M3, act-quantised E4M3
tokens, UE8M0 scales) and round the SwiGLU hidden with the reference's act
quant (ties to the lower grid entry, the host libm's expf in SiLU).  What may
still differ is the tensor core's accumulation order in the w1/w3 and w2
contractions.  Through w1/w3 it can only move a hidden value onto the
neighbouring E4M3 grid point when its act quant lands on the other side of a
midpoint (a "grid flip"); through w2 it is rounding noise.

The gate reads the act-quantised hidden of every sampled (token, expert) row
out of the call's scratch (wh_moe_scratch_field) and the reference's from the
oracle, counts the flips, and requires

    |y - ref - sum_k c_k W2_k (h_k - h_ref_k)| <= tol * D,
    D = sum_k |c_k| |W2_k| |h_k|            (per output element),

i.e. once the flips' exact effect is taken out, the rest is within the
grouped path's normalised-error bound tol = 2e-6 (|y - y_hat| / sum|w x|), the
bound for a tensor-core accumulation order over K up to 4096.  It also
reports the normalised error of the raw outputs and the flip count.
"""
from __future__ import annotations

import numpy as np

import oracle as O
from tests import helpers as H

FP4_LUT = np.array([0, 0.125, 1, 1.5, 2, 3, 4, 6, 0, -0.125, -1, -1.5, -2, -3, -4, -6],
                   np.float64)
NORM_TOL = 2e-6


def _w2_dense(torch, stack, e):
    """W2 of expert e decoded to float64 [hidden][inter] on the device."""
    w2, s2 = stack["w2"][e], stack["s2"][e]
    lut = torch.tensor(FP4_LUT, device=w2.device)
    vals = torch.stack([lut[(w2 & 15).long()], lut[(w2 >> 4).long()]], dim=-1)
    vals = vals.reshape(w2.shape[0], -1)
    sc = torch.where(s2 == 0, torch.zeros_like(s2, dtype=torch.float64),
                     torch.pow(2.0, s2.double() - 127))
    return vals * sc.repeat_interleave(32, dim=1)


def _oracle_expert(stack, e, keep):
    w1, s1, w3, s3, w2, s2 = [t.cpu().numpy() for t in H.expert_views(stack, e)]
    inter, hb = w1.shape
    hidden = hb * 2
    return O.Fp4Expert(O.fp4_spec(w1, s1, inter, hidden, hidden // 32, keep),
                       O.fp4_spec(w3, s3, inter, hidden, hidden // 32, keep),
                       O.fp4_spec(w2, s2, hidden, inter, inter // 32, keep))


def check_grouped(torch, W, layer, stack, x, y, ids, weights, E, sample=None, route_order=False,
                  tol=NORM_TOL):
    """x [T][hidden] f32 numpy (the call's input), y its output (numpy), ids /
    weights the routes it returned (numpy).  sample: token indices to check
    (default all).  route_order: the reference is the single-token combine
    (moe_combine_token) instead of the batched one.  Returns a dict of
    metrics; raises AssertionError when the gate fails."""
    T, hidden = x.shape
    topk = ids.shape[1]
    inter = layer.inter
    sample = np.arange(T) if sample is None else np.asarray(sample)
    S = len(sample)
    R = T * topk + T
    slot = layer.scratch_field(T, W.MOE_FIELD_SLOT, torch.int32, (T, topk)).cpu().numpy()
    offs = layer.scratch_field(T, W.MOE_FIELD_OFFSETS, torch.int32, (E + 2,)).cpu().numpy()
    cw = layer.scratch_field(T, W.MOE_FIELD_COMBINE_W, torch.float32, (T, topk)).cpu().numpy()
    hq = layer.scratch_field(T, W.MOE_FIELD_HQ, torch.uint8, (R, inter))
    hsf = layer.scratch_field(T, W.MOE_FIELD_HSF, torch.uint8, (R, inter // 32))

    # the rows of the sampled (token, slot) pairs; slot topk = the shared expert
    rows = np.zeros((S, topk + 1), np.int64)
    for i, t in enumerate(sample):
        for k in range(topk):
            rows[i, k] = offs[ids[t, k]] + slot[t, k]
        rows[i, topk] = offs[E] + t
    ridx = torch.from_numpy(rows.reshape(-1)).to(hq.device)
    hg = hq[ridx].view(torch.float8_e4m3fn).float().double()
    hg = hg * torch.pow(2.0, hsf[ridx].double() - 127).repeat_interleave(32, dim=1)
    hg = hg.view(S, topk + 1, inter)

    # the reference: router ids/weights were checked by the caller; outputs and
    # the act-quantised hidden of every sampled row from the oracle
    keep: list = []
    used = sorted(set(ids[sample].reshape(-1).tolist()) | {E})
    arr = (O.Fp4Expert * (E + 1))()
    for e in used:
        arr[e] = _oracle_expert(stack, e, keep)
    xs = np.ascontiguousarray(x[sample])
    if route_order:
        want = np.zeros((S, hidden), np.float32)
        for i, t in enumerate(sample):
            st, want[i] = O.moe_combine_token(arr, ids[t], weights[t], arr[E], x[t])
            assert st == O.OK
    else:
        st, want = O.moe_batched(arr, E, np.ascontiguousarray(ids[sample]),
                                 np.ascontiguousarray(weights[sample]), arr[E], xs)
        assert st == O.OK
    href = np.zeros((S, topk + 1, inter), np.float32)
    for i, t in enumerate(sample):
        for k in range(topk + 1):
            e = ids[t, k] if k < topk else E
            st, href[i, k] = O.fp4_expert_hidden(arr[e], x[t])
            assert st in (O.OK, O.ERR_NON_FINITE_OUTPUT)
    hr = torch.from_numpy(href).to(hg.device).double()
    dh = hg - hr
    flips = int((dh != 0).sum().item())

    # the flips' effect and the normalisation, expert by expert
    coef = np.ones((S, topk + 1), np.float64)
    coef[:, :topk] = cw[sample]
    if route_order:
        # one routed expert: unweighted (src/compute.rs:1960-1966)
        single = (ids[sample] >= 0).sum(1) == 1
        coef[single, 0] = 1.0
    pred = torch.zeros(S, hidden, dtype=torch.float64, device=hg.device)
    D = torch.zeros(S, hidden, dtype=torch.float64, device=hg.device)
    by_e: dict = {}
    for i, t in enumerate(sample):
        for k in range(topk + 1):
            e = int(ids[t, k]) if k < topk else E
            by_e.setdefault(e, []).append((i, k))
    ct = torch.from_numpy(coef).to(hg.device)
    for e, pairs in by_e.items():
        w2 = _w2_dense(torch, stack, e)
        ii = torch.tensor([p[0] for p in pairs], device=hg.device)
        kk = torch.tensor([p[1] for p in pairs], device=hg.device)
        c = ct[ii, kk].unsqueeze(1)
        if flips:
            pred.index_add_(0, ii, c * (dh[ii, kk] @ w2.T))
        D.index_add_(0, ii, c.abs() * (hg[ii, kk].abs() @ w2.abs().T))
    yg = torch.from_numpy(np.ascontiguousarray(y[sample])).to(hg.device).double()
    wt = torch.from_numpy(want).to(hg.device).double()
    raw = ((yg - wt).abs() / D.clamp_min(1e-300)).max().item()
    resid = ((yg - wt - pred).abs() / D.clamp_min(1e-300)).max().item()
    flip_tokens = int(((dh != 0).flatten(1).any(1)).sum().item())
    m = {"tokens_checked": S, "hidden_values": S * (topk + 1) * inter, "flips": flips,
         "tokens_with_flips": flip_tokens, "norm_err_raw": raw, "norm_err_after_flips": resid,
         "max_abs_over_max_ref": float(np.abs(y[sample] - want).max() / np.abs(want).max())}
    print("grouped parity:", m)
    assert np.isfinite(y[sample]).all()
    assert resid <= tol, m
    return m
