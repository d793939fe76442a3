"""The composed DeepSeek-V4 decode step (wohper_b200/v4model.py) against the
oracle's composition of the same reference functions: two layers of the
V4-Flash shape (a window-only layer with plain RoPE and a compressed layer
with YaRN, 16 routed FP4 experts + shared), the pooled head and the lm_head
top-k, for two sequences at different positions.  Every kernel is bit-exact,
so the residual stream after the layers, the KV rows written and the top-k
tokens and logits must be equal bit for bit."""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

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


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def np_(t):
    return t.detach().cpu().numpy()


def _oracle_layer(raw, E):
    keep = []
    m = {n: O.fp8_matrix(np_(w), np_(s), w.shape[0], w.shape[1], s.shape[0], s.shape[1], keep)
         for n, (w, s) in ((n, raw[n]) for n in H.V4_SHAPES)}
    qn, kn, sink = np_(raw["q_norm"]).view(np.uint16), np_(raw["kv_norm"]).view(np.uint16), \
        np_(raw["sink"]).astype(np.float32)
    keep += [qn, kn, sink]
    spec = O.V4Attn(4096, 64, 512, 448, 1024, 8, 1024, 128, m["wq_a"], m["wq_b"], m["wkv"],
                    m["wo_a"], m["wo_b"], qn.ctypes.data, kn.ctypes.data, sink.ctypes.data)
    arr = (O.Fp4Expert * (E + 1))()
    for e in range(E + 1):
        w1, s1, w3, s3, w2, s2 = [np_(t) for t in H.expert_views(raw["stack"], e)]
        arr[e] = O.Fp4Expert(O.fp4_spec(w1, s1, 2048, 4096, 128, keep),
                             O.fp4_spec(w3, s3, 2048, 4096, 128, keep),
                             O.fp4_spec(w2, s2, 4096, 2048, 64, keep))
    return spec, arr, keep


def test_v4_decode_step_two_layers_bit_exact(ctx, W):
    from wohper_b200.v4model import V4Decoder

    E, B, hc, Hd = 16, 2, 4, 4096
    positions = [700, 300]
    layers, raws = [], []
    for li in (0, 2):
        L, raw = H.v4_layer(W, ctx, li, E, seed=500 + li, max_tokens=B)
        layers.append(L)
        raws.append(raw)
    kv = [[torch.from_numpy(H.activations(510 + 10 * b + i, positions[b] + 4, 512)).cuda()
           for i in range(2)] for b in range(B)]
    comp = [[(torch.from_numpy(H.activations(530 + 10 * b + i, n, 512)).cuda() if n else None)
             for i, n in enumerate(H.v4_compressed_count(L.index, positions[b]) for L in layers)]
            for b in range(B)]
    head = H.torch_hc_params(540, hc, Hd, head=True)
    final_norm = H.torch_bf16_norm(541, Hd)
    vocab = 4096
    lm = torch.from_numpy(H.router_gate(542, vocab, Hd).view(np.int16)).cuda()
    x0 = H.activations(543, B, hc * Hd)
    kv_host = [[np_(t).copy() for t in row] for row in kv]
    dec = V4Decoder(ctx, layers, head, final_norm, lm, kv, comp, batch=B, top_k=8)
    x = torch.from_numpy(x0).cuda()
    toks, vals = dec.step(x, positions)
    ctx.sync()
    toks, vals, x_got = np_(toks), np_(vals), np_(x)

    # the oracle's composition of the same reference functions
    specs = [_oracle_layer(r, E) for r in raws]
    for b in range(B):
        xs = x0[b].copy()
        for i, (L, raw) in enumerate(zip(layers, raws)):
            spec, arr, _ = specs[i]
            fr = W.rope_inv_freqs(64, *W.deepseek_rope_for_layer(L.index))
            fn, sc, base = [np_(t) for t in raw["hc_attn"]]
            st, y, post, cm = O.hc_pre(fn, sc, base, xs, hc, Hd)
            assert st == O.OK
            y = O.rms_norm(y, np_(raw["attn_norm"]).view(np.uint16))
            cmp = comp[b][i]
            st, y = O.v4_attention(spec, positions[b], y, kv_host[b][i],
                                   None if cmp is None else np_(cmp), fr)
            assert st == O.OK
            xs = O.hc_post(y, xs, post, cm, hc, Hd)
            fn, sc, base = [np_(t) for t in raw["hc_ffn"]]
            st, y, post, cm = O.hc_pre(fn, sc, base, xs, hc, Hd)
            y = O.rms_norm(y, np_(raw["ffn_norm"]).view(np.uint16))
            _, ids, w, _ = O.router(np_(raw["gate"]).view(np.uint16), y, 6, mode=0)
            st, y = O.moe_combine_token(arr, ids, w, arr[E], y)
            assert st == O.OK
            xs = O.hc_post(y, xs, post, cm, hc, Hd)
            np.testing.assert_array_equal(bits(np_(kv[b][i])[positions[b]]),
                                          bits(kv_host[b][i][positions[b]]))
        assert np.array_equal(bits(x_got[b]), bits(xs)), f"residual stream of sequence {b}"
        fn, sc, base = head
        pooled = O.hc_head(np_(fn), sc, np_(base), xs, hc, Hd)
        pooled = O.rms_norm(pooled, np_(final_norm).view(np.uint16))
        n, t_ref, v_ref, _ = O.lm_head_topk(np_(lm).view(np.uint16), pooled, 8)
        assert np.array_equal(toks[b, :n], t_ref[:n].astype(np.int32))
        assert np.array_equal(bits(vals[b, :n]), bits(v_ref[:n]))
    for L in layers:
        L.moe.close()
