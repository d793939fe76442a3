"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU oracle (liboracle.so).

The oracle restates the reference engine's Rust CPU kernels (see
wohper_oracle.h).  Only tests/, ``__graft_entry__.smoke()`` and bench.py's
cpu_baseline / ``--impl reference`` arm import this module, as the checker or
the timed CPU baseline.  The product package ``wohper_b200`` never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

OK = 0
ERR_EMPTY_SHAPE = 1
ERR_INVALID_SHAPE = 2
ERR_PACKED_WEIGHT_TOO_SMALL = 3
ERR_SCALE_TOO_SMALL = 4
ERR_INPUT_TOO_SMALL = 5
ERR_OUTPUT_TOO_SMALL = 6
ERR_SCRATCH_TOO_SMALL = 7
ERR_NON_FINITE_OUTPUT = 8


class Fp4Spec(C.Structure):
    _fields_ = [
        ("packed_weight", C.c_void_p),
        ("packed_len", C.c_size_t),
        ("ue8m0_scales", C.c_void_p),
        ("scales_len", C.c_size_t),
        ("rows", C.c_size_t),
        ("cols", C.c_size_t),
        ("scale_cols", C.c_size_t),
    ]


class Fp4Expert(C.Structure):
    _fields_ = [("w1", Fp4Spec), ("w3", Fp4Spec), ("w2", Fp4Spec)]


class Fp8Matrix(C.Structure):
    _fields_ = [
        ("weight", C.c_void_p),
        ("scale", C.c_void_p),
        ("rows", C.c_size_t),
        ("cols", C.c_size_t),
        ("scale_rows", C.c_size_t),
        ("scale_cols", C.c_size_t),
    ]


class Fp8Expert(C.Structure):
    _fields_ = [("w1", Fp8Matrix), ("w3", Fp8Matrix), ("w2", Fp8Matrix)]


def build() -> Path:
    """Compile liboracle.so with oracle/Makefile (g++, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sz, vp, f, i = C.c_size_t, C.c_void_p, C.c_float, C.c_int
        L.orc_set_threads.argtypes = [i]
        L.orc_get_threads.restype = i
        L.orc_decode_fp8_e4m3.argtypes = [C.c_uint8, f]
        L.orc_decode_fp8_e4m3.restype = f
        L.orc_decode_ue8m0_scale.argtypes = [C.c_uint8]
        L.orc_decode_ue8m0_scale.restype = f
        L.orc_decode_fp4_e2m1.argtypes = [C.c_uint8, f]
        L.orc_decode_fp4_e2m1.restype = f
        for n in ("orc_fp8_e4m3_base_lut", "orc_ue8m0_scale_lut", "orc_fp4_e2m1_base_lut",
                  "orc_fp8_e4m3_sorted_lut"):
            getattr(L, n).argtypes = [vp]
        L.orc_fp8_dot_row.argtypes = [vp, vp, sz, sz, vp, i]
        L.orc_fp8_dot_row.restype = f
        L.orc_fp8_gemv_rows.argtypes = [vp, sz, sz, sz, vp, sz, sz, sz, sz, sz, vp, sz, vp, sz]
        L.orc_fp8_gemv_rows.restype = i
        L.orc_fp8_gemv_rows_multi.argtypes = [vp, sz, sz, sz, vp, sz, sz, sz, sz, sz, vp, sz, sz,
                                              vp, sz]
        L.orc_fp8_gemv_rows_multi.restype = i
        L.orc_fp8_act_quant_dequant_in_place.argtypes = [vp, sz, sz]
        L.orc_bf16_dot_row.argtypes = [vp, vp, sz, i]
        L.orc_bf16_dot_row.restype = f
        L.orc_bf16_gemv.argtypes = [vp, sz, sz, vp, vp]
        L.orc_bf16_gemv.restype = i
        L.orc_lm_head_topk.argtypes = [vp, sz, sz, vp, sz, C.c_uint32, vp, vp, vp]
        L.orc_lm_head_topk.restype = i
        L.orc_expf_n.argtypes = [vp, vp, sz]
        L.orc_expf_n.restype = None
        L.orc_rope_inv_freqs.argtypes = [sz, f, f, f, f, sz, vp]
        L.orc_rope_inv_freqs.restype = None
        L.orc_mla_attention.argtypes = [vp, sz, sz, sz, vp, sz, sz, sz, vp, sz, vp, vp, vp]
        L.orc_mla_attention.restype = None
        L.orc_rms_norm.argtypes = [vp, sz, vp, vp]
        L.orc_rms_norm.restype = None
        L.orc_v4_attention.argtypes = [C.c_void_p, sz, vp, vp, sz, vp, sz, vp]
        L.orc_v4_attention.restype = i
        L.orc_hc_split_sinkhorn.argtypes = [vp, sz, vp, sz, vp, sz, sz, sz, f, vp, vp, vp]
        L.orc_hc_split_sinkhorn.restype = i
        L.orc_hc_pre.argtypes = [vp, sz, sz, vp, sz, vp, vp, sz, sz, sz, f, vp, vp, vp]
        L.orc_hc_pre.restype = i
        L.orc_hc_post.argtypes = [vp, vp, vp, vp, vp, sz, sz]
        L.orc_hc_post.restype = None
        L.orc_hc_head.argtypes = [vp, f, vp, vp, sz, sz, f, vp]
        L.orc_hc_head.restype = None
        L.orc_fp4_matvec.argtypes = [C.POINTER(Fp4Spec), vp, sz, vp, sz, i]
        L.orc_fp4_matvec.restype = i
        L.orc_fp4_expert_forward.argtypes = [C.POINTER(Fp4Expert), vp, sz, vp, sz, vp, sz]
        L.orc_fp4_expert_forward.restype = i
        L.orc_fp4_expert_scratch_len.argtypes = [sz]
        L.orc_fp4_expert_scratch_len.restype = sz
        L.orc_fp8_expert_forward.argtypes = [C.POINTER(Fp8Expert), vp, sz, vp]
        L.orc_fp8_expert_forward.restype = i
        L.orc_router.argtypes = [vp, sz, sz, vp, sz, i, vp, f, vp, vp, vp, vp]
        L.orc_router.restype = i
        L.orc_deepseek_sqrtsoftplus_route.argtypes = [vp, sz, vp, sz, f, vp, vp]
        L.orc_deepseek_sqrtsoftplus_route.restype = sz
        L.orc_moe_combine_token.argtypes = [C.POINTER(Fp4Expert), vp, vp, sz,
                                            C.POINTER(Fp4Expert), C.POINTER(Fp8Expert), vp, sz,
                                            vp]
        L.orc_moe_combine_token.restype = i
        L.orc_moe_batched.argtypes = [C.POINTER(Fp4Expert), sz, vp, vp, sz, sz,
                                      C.POINTER(Fp4Expert), vp, sz, vp]
        L.orc_moe_batched.restype = i
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return lib().orc_get_threads()


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


def fp4_spec(packed, scales, rows, cols, scale_cols, keep: list) -> Fp4Spec:
    packed = _c(packed, np.uint8)
    scales = _c(scales, np.uint8)
    keep += [packed, scales]
    return Fp4Spec(packed.ctypes.data, packed.size, scales.ctypes.data, scales.size, rows, cols,
                   scale_cols)


def fp4_expert(w1: dict, w3: dict, w2: dict, keep: list) -> Fp4Expert:
    mk = lambda d: fp4_spec(d["packed"], d["scales"], d["rows"], d["cols"], d["scale_cols"], keep)
    return Fp4Expert(mk(w1), mk(w3), mk(w2))


def fp8_matrix(weight, scale, rows, cols, scale_rows, scale_cols, keep: list) -> Fp8Matrix:
    weight = _c(weight, np.uint8)
    scale = _c(scale, np.uint8)
    keep += [weight, scale]
    return Fp8Matrix(weight.ctypes.data, scale.ctypes.data, rows, cols, scale_rows, scale_cols)


def fp8_expert_forward(expert: Fp8Expert, x):
    """compute_deepseek_fp8_shared_expert_into_hidden: (status, output[w2.rows])."""
    x = _c(x, np.float32)
    y = np.zeros(expert.w2.rows, np.float32)
    st = lib().orc_fp8_expert_forward(C.byref(expert), _p(x), x.size, _p(y))
    return st, y


def luts() -> dict:
    L = lib()
    out = {}
    for key, n, fn in (("fp8", 256, L.orc_fp8_e4m3_base_lut), ("ue8m0", 256, L.orc_ue8m0_scale_lut),
                       ("fp4", 16, L.orc_fp4_e2m1_base_lut),
                       ("sorted", 256, L.orc_fp8_e4m3_sorted_lut)):
        a = np.zeros(n, np.float32)
        fn(_p(a))
        out[key] = a
    return out


def act_quant(x, block: int = 64) -> np.ndarray:
    v = _c(x, np.float32).copy()
    lib().orc_fp8_act_quant_dequant_in_place(_p(v), v.size, block)
    return v


def fp8_dot_row(w, s, col_group, x, avx2=True) -> float:
    w, s, x = _c(w, np.uint8), _c(s, np.uint8), _c(x, np.float32)
    return lib().orc_fp8_dot_row(_p(w), _p(s), s.size, col_group, _p(x), int(avx2))


def fp8_gemv(weight, scale, x, rows, cols, scale_rows, scale_cols, row_start=0, row_end=None):
    row_end = rows if row_end is None else row_end
    w, s, x = _c(weight, np.uint8), _c(scale, np.uint8), _c(x, np.float32)
    y = np.zeros(row_end - row_start, np.float32)
    st = lib().orc_fp8_gemv_rows(_p(w), w.size, rows, cols, _p(s), s.size, scale_rows,
                                 scale_cols, row_start, row_end, _p(x), x.size, _p(y), y.size)
    return st, y


def fp8_gemv_multi(weight, scale, xs, rows, cols, scale_rows, scale_cols, row_start=0,
                   row_end=None):
    row_end = rows if row_end is None else row_end
    w, s, xs = _c(weight, np.uint8), _c(scale, np.uint8), _c(xs, np.float32)
    count = xs.shape[0]
    n = row_end - row_start
    y = np.zeros((count, n), np.float32)
    st = lib().orc_fp8_gemv_rows_multi(_p(w), w.size, rows, cols, _p(s), s.size, scale_rows,
                                       scale_cols, row_start, row_end, _p(xs), count,
                                       xs.shape[1], _p(y), n)
    return st, y


def bf16_dot_row(row_u16, x, avx2=True) -> float:
    r, x = _c(row_u16, np.uint16), _c(x, np.float32)
    return lib().orc_bf16_dot_row(_p(r), _p(x), x.size, int(avx2))


def bf16_gemv(w_u16, x):
    w, x = _c(w_u16, np.uint16), _c(x, np.float32)
    y = np.zeros(w.shape[0], np.float32)
    st = lib().orc_bf16_gemv(_p(w), w.shape[0], w.shape[1], _p(x), _p(y))
    return st, y


def expf(x):
    """The host C library's expf, elementwise (Rust's f32::exp)."""
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_expf_n(_p(x), _p(y), x.size)
    return y


def rope_inv_freqs(rope_dim, theta, yarn=None):
    """rope_inv_freqs (src/compute.rs:2591-2621); yarn = (factor, beta_fast,
    beta_slow, original_seq_len) or None."""
    out = np.zeros(rope_dim // 2, np.float32)
    fa, bf, bs, osl = yarn if yarn else (0.0, 0.0, 0.0, 0)
    lib().orc_rope_inv_freqs(rope_dim, theta, fa, bf, bs, osl, _p(out))
    return out


def hc_split_sinkhorn(mixes, scale, base, hc, iters=20, eps=1e-6):
    """hc_split_sinkhorn_scalar (src/compute.rs:4945-4991) -> (status, pre, post, comb)."""
    m, sc, b = _c(mixes, np.float32), _c(scale, np.float32), _c(base, np.float32)
    pre, post = np.zeros(hc, np.float32), np.zeros(hc, np.float32)
    comb = np.zeros(hc * hc, np.float32)
    st = lib().orc_hc_split_sinkhorn(_p(m), m.size, _p(sc), sc.size, _p(b), b.size, hc, iters,
                                     eps, _p(pre), _p(post), _p(comb))
    return st, pre, post, comb


def hc_pre(fn, scale, base, x, hc, hidden, iters=20, eps=1e-6):
    """hc_pre_into (src/compute.rs:5016-5053) for one token: fn [mix_hc, hc*hidden],
    x [hc*hidden] -> (status, y [hidden], post [hc], comb [hc*hc])."""
    fn, sc, b, x = (_c(fn, np.float32), _c(scale, np.float32), _c(base, np.float32),
                    _c(x, np.float32))
    y = np.zeros(hidden, np.float32)
    post, comb = np.zeros(hc, np.float32), np.zeros(hc * hc, np.float32)
    st = lib().orc_hc_pre(_p(fn), fn.shape[0], fn.shape[1], _p(sc), sc.size, _p(b), _p(x), hc,
                          hidden, iters, eps, _p(y), _p(post), _p(comb))
    return st, y, post, comb


def hc_post(y, residual, post, comb, hc, hidden):
    """hc_post_into (src/compute.rs:5055-5089) for one token -> out [hc*hidden]."""
    y, r, p, c = (_c(y, np.float32), _c(residual, np.float32), _c(post, np.float32),
                  _c(comb, np.float32))
    out = np.zeros(hc * hidden, np.float32)
    lib().orc_hc_post(_p(y), _p(r), _p(p), _p(c), _p(out), hc, hidden)
    return out


def hc_head(fn, scale, base, x, hc, hidden, eps=1e-6):
    """hc_head_pool (src/compute.rs:5091-5132) for one token -> pooled [hidden]."""
    fn, b, x = _c(fn, np.float32), _c(base, np.float32), _c(x, np.float32)
    pooled = np.zeros(hidden, np.float32)
    lib().orc_hc_head(_p(fn), float(scale), _p(b), _p(x), hc, hidden, eps, _p(pooled))
    return pooled


def mla_attention(q, keys, token_pos, window, compressed, sink, inv_freqs, nope_dim):
    """The attention core of compute_deepseek_v4_mla_attention: q [heads, head_dim],
    keys [positions, stride], compressed [count, head_dim] or None, sink [heads] or
    None -> out [heads, head_dim]."""
    q = _c(q, np.float32)
    keys = _c(keys, np.float32)
    heads, hd = q.shape
    comp = None if compressed is None else _c(compressed, np.float32)
    sk = None if sink is None else _c(sink, np.float32)
    fr = _c(inv_freqs, np.float32)
    out = np.zeros((heads, hd), np.float32)
    lib().orc_mla_attention(_p(q), heads, hd, nope_dim, _p(keys), keys.shape[1], token_pos,
                            window, _p(comp), 0 if comp is None else comp.shape[0], _p(sk),
                            _p(fr), _p(out))
    return out


def lm_head_topk(w_u16, x, top_k, row_base=0):
    """score_bf16_lm_head_topk + push_topk_candidate + the final sort: returns
    (count, tokens, logits of the top-k, all logits)."""
    w, x = _c(w_u16, np.uint16), _c(x, np.float32)
    rows, cols = w.shape
    k = max(int(top_k), 1)
    tok = np.zeros(k, np.uint32)
    val = np.zeros(k, np.float32)
    logits = np.zeros(rows, np.float32)
    n = lib().orc_lm_head_topk(_p(w), rows, cols, _p(x), k, row_base, _p(tok), _p(val),
                               _p(logits))
    return n, tok[:max(n, 0)], val[:max(n, 0)], logits


def fp4_matvec(packed, scales, rows, cols, scale_cols, x, path=0, out_len=None):
    keep: list = []
    spec = fp4_spec(packed, scales, rows, cols, scale_cols, keep)
    x = _c(x, np.float32)
    y = np.zeros(rows if out_len is None else out_len, np.float32)
    st = lib().orc_fp4_matvec(C.byref(spec), _p(x), x.size, _p(y), y.size, path)
    return st, y


def fp4_expert_forward(expert: Fp4Expert, x, out_len=None, scratch_len=None):
    x = _c(x, np.float32)
    y = np.zeros(expert.w2.rows if out_len is None else out_len, np.float32)
    sl = 2 * expert.w1.rows if scratch_len is None else scratch_len
    scratch = np.zeros(max(sl, 1), np.float32)
    st = lib().orc_fp4_expert_forward(C.byref(expert), _p(x), x.size, _p(y), y.size, _p(scratch),
                                      sl)
    return st, y


def router(gate_u16, x, topk, mode=0, bias=None, route_scale=1.0, hash_ids=None):
    g, x = _c(gate_u16, np.uint16), _c(x, np.float32)
    E, H = g.shape
    b = None if bias is None else _c(bias, np.float32)
    h = None if hash_ids is None else _c(hash_ids, np.int32)
    ids = np.full(topk, -1, np.int32)
    w = np.zeros(topk, np.float32)
    logits = np.zeros(E, np.float32)
    n = lib().orc_router(_p(g), E, H, _p(x), topk, mode, _p(b), route_scale, _p(h), _p(ids),
                         _p(w), _p(logits))
    return n, ids, w, logits


def deepseek_sqrtsoftplus_route(logits, topk, route_scale, bias=None):
    l = _c(logits, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    ids = np.zeros(topk, np.int32)
    w = np.zeros(topk, np.float32)
    n = lib().orc_deepseek_sqrtsoftplus_route(_p(l), l.size, _p(b), topk, route_scale, _p(ids),
                                              _p(w))
    return ids[:n], w[:n]


def moe_combine_token(experts_arr, ids, weights, shared_fp4, x, shared_fp8=None):
    ids, weights, x = _c(ids, np.int32), _c(weights, np.float32), _c(x, np.float32)
    y = np.zeros(x.size, np.float32)
    sh4 = C.byref(shared_fp4) if shared_fp4 is not None else None
    sh8 = C.byref(shared_fp8) if shared_fp8 is not None else None
    st = lib().orc_moe_combine_token(experts_arr, _p(ids), _p(weights), ids.size, sh4, sh8,
                                     _p(x), x.size, _p(y))
    return st, y


def moe_batched(experts_arr, num_experts, ids, weights, shared_fp4, x):
    ids, weights, x = _c(ids, np.int32), _c(weights, np.float32), _c(x, np.float32)
    T, K = ids.shape
    y = np.zeros_like(x)
    sh4 = C.byref(shared_fp4) if shared_fp4 is not None else None
    st = lib().orc_moe_batched(experts_arr, num_experts, _p(ids), _p(weights), T, K, sh4, _p(x),
                               x.shape[1], _p(y))
    return st, y


def fp4_expert_hidden(expert: Fp4Expert, x):
    """(status, h): the act-quantised SwiGLU hidden the reference's expert
    forward feeds to w2 (src/deepseek_v4.rs:586-596) -- the first `inter`
    floats of its scratch once deepseek_v4_fp4_expert_forward_scalar returns."""
    x = _c(x, np.float32)
    inter = expert.w1.rows
    y = np.zeros(expert.w2.rows, np.float32)
    scratch = np.zeros(2 * inter, np.float32)
    st = lib().orc_fp4_expert_forward(C.byref(expert), _p(x), x.size, _p(y), y.size, _p(scratch),
                                      2 * inter)
    return st, scratch[:inter].copy()


def rms_norm(x, weight_bf16=None):
    """apply_weighted_rms_norm / rms_norm_in_place of each row of x."""
    x = _c(x, np.float32)
    w = None if weight_bf16 is None else _c(weight_bf16, np.uint16)
    rows = x.reshape(-1, x.shape[-1])
    out = np.zeros_like(rows)
    for i in range(rows.shape[0]):
        lib().orc_rms_norm(_p(rows[i]), rows.shape[1], _p(w), _p(out[i]))
    return out.reshape(x.shape)


class V4Attn(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in ("hidden", "heads", "head_dim", "nope_dim",
                                          "q_lora_rank", "o_groups", "o_lora_rank", "window")] + [
        ("wq_a", Fp8Matrix), ("wq_b", Fp8Matrix), ("wkv", Fp8Matrix), ("wo_a", Fp8Matrix),
        ("wo_b", Fp8Matrix), ("q_norm", C.c_void_p), ("kv_norm", C.c_void_p),
        ("sink", C.c_void_p)]


def v4_attention(layer: V4Attn, token_pos, hidden, kv_cache, compressed, inv_freqs):
    """compute_deepseek_v4_mla_attention for one token: (status, out [hidden]);
    kv_cache [positions, stride] (numpy, row token_pos is written)."""
    h = np.array(hidden, np.float32, copy=True)
    comp = None if compressed is None else _c(compressed, np.float32)
    fr = _c(inv_freqs, np.float32)
    st = lib().orc_v4_attention(C.byref(layer), token_pos, _p(h), _p(kv_cache),
                                kv_cache.shape[1], _p(comp), 0 if comp is None else comp.shape[0],
                                _p(fr))
    return st, h
