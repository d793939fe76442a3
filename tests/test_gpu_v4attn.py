"""DeepSeek-V4 attention block on the GPU, bit-exact against the oracle's
restatement of the reference: the weighted RMS norm (apply_weighted_rms_norm /
rms_norm_in_place, src/compute.rs:3077-3115,7110-7122), the grouped wo_a
GEMV (src/compute.rs:4244-4258) and the whole MLA projection path
(compute_deepseek_v4_mla_attention, src/compute.rs:3924-4293) at the
DeepSeek-V4-Flash shape on both rope kinds (plain on a window-only layer,
YaRN on a compressed layer)."""
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


def norm_weight(seed, n):
    return H.bf16_bits(1.0 + 0.1 * H.rng(seed).normal(size=n).astype(np.float32))


@pytest.mark.parametrize("segments,n,weighted", [(1, 4096, True), (1, 1024, True),
                                                  (64, 512, False), (3, 77, True)])
def test_rms_norm_bit_exact(ctx, W, segments, n, weighted):
    x = H.activations(300 + n, segments, n, scale=3.0)
    w = norm_weight(301, n) if weighted else None
    got = W.rms_norm(ctx, torch.from_numpy(x).cuda(),
                     torch.from_numpy(w.view(np.int16)).cuda() if weighted else None)
    ctx.sync()
    want = O.rms_norm(x, w)
    assert np.array_equal(bits(got.cpu().numpy()), bits(want))


def test_fp8_gemv_grouped_wo_a_bit_exact(ctx, W):
    # V4-Flash wo_a: 8 groups of 1024 rows, each over its 4096-wide slice of the
    # 32768 attention outputs, act quant per group
    rows, cols, groups = 8192, 4096, 8
    w, s = H.fp8_weight(310, rows, cols)
    x = H.activations(311, 1, cols * groups).reshape(-1)
    got = W.gemv_fp8_e4m3_ue8m0_grouped(ctx, torch.from_numpy(w).cuda(),
                                        torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda(),
                                        rows // groups, cols, act_quant_block=64)
    ctx.sync()
    xq = O.act_quant(x, 64)
    want = np.concatenate([
        O.fp8_gemv(w, s, xq[g * cols:(g + 1) * cols], rows, cols, rows // 128, cols // 128,
                   g * (rows // groups), (g + 1) * (rows // groups))[1] for g in range(groups)])
    assert np.array_equal(bits(got.cpu().numpy()), bits(want))


def _v4_layer(W, seed, dev="cuda"):
    hd, heads, nope, ql, og, ol, hid = 512, 64, 448, 1024, 8, 1024, 4096
    shapes = {"wq_a": (ql, hid), "wq_b": (heads * hd, ql), "wkv": (hd, hid),
              "wo_a": (og * ol, heads * hd // og), "wo_b": (hid, og * ol)}
    host, dev_m, keep = {}, {}, []
    for i, (name, (r, c)) in enumerate(shapes.items()):
        w, s = H.fp8_weight(seed + i, r, c)
        host[name] = O.fp8_matrix(w, s, r, c, s.shape[0], s.shape[1], keep)
        dev_m[name] = W.Fp8Matrix(torch.from_numpy(w).to(dev), torch.from_numpy(s).to(dev))
    qn, kn = norm_weight(seed + 10, ql), norm_weight(seed + 11, hd)
    sink = H.rng(seed + 12).normal(0.0, 1.0, heads).astype(np.float32)
    keep += [qn, kn, sink]
    layer = W.V4Attention(**dev_m, q_norm=torch.from_numpy(qn.view(np.int16)).to(dev),
                          kv_norm=torch.from_numpy(kn.view(np.int16)).to(dev),
                          sink=torch.from_numpy(sink).to(dev))
    spec = O.V4Attn(hid, heads, hd, nope, ql, og, ol, W.DEEPSEEK_V4_SLIDING_WINDOW,
                    host["wq_a"], host["wq_b"], host["wkv"], host["wo_a"], host["wo_b"],
                    qn.ctypes.data, kn.ctypes.data, sink.ctypes.data)
    return layer, spec, keep


@pytest.mark.parametrize("layer_index,token_pos,n_comp", [(0, 300, 0), (2, 700, 175)])
def test_v4_attention_projection_path_bit_exact(ctx, W, layer_index, token_pos, n_comp):
    layer, spec, keep = _v4_layer(W, 320 + layer_index)
    theta, yarn = W.deepseek_rope_for_layer(layer_index)
    fr = W.rope_inv_freqs(64, theta, yarn)
    positions, stride = token_pos + 8, 512
    kv = H.activations(330 + layer_index, positions, stride)
    comp = H.activations(331, n_comp, 512) if n_comp else None
    x = H.activations(332 + layer_index, 1, 4096).reshape(-1)
    x = O.rms_norm(x, norm_weight(333, 4096))  # the normed attention input
    kv_d = torch.from_numpy(kv).cuda()
    hid = torch.from_numpy(x).cuda()
    W.v4_attention(ctx, layer, token_pos, hid, kv_d, fr,
                   None if comp is None else torch.from_numpy(comp).cuda())
    ctx.sync()
    kv_h = kv.copy()
    st, want = O.v4_attention(spec, token_pos, x, kv_h, comp, fr)
    assert st == O.OK
    assert np.array_equal(bits(kv_d.cpu().numpy()[token_pos]), bits(kv_h[token_pos])), "kv row"
    got = hid.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert np.array_equal(bits(got), bits(want))


def test_v4_attention_batch_of_tokens_bit_exact(ctx, W):
    # three sequences, two at the same position (one norm launch covers both)
    layer, spec, keep = _v4_layer(W, 340)
    theta, yarn = W.deepseek_rope_for_layer(2)
    fr = W.rope_inv_freqs(64, theta, yarn)
    pos = [500, 500, 260]
    kvs = [H.activations(341 + t, p + 4, 512) for t, p in enumerate(pos)]
    comps = [H.activations(345 + t, H.v4_compressed_count(2, p), 512) for t, p in enumerate(pos)]
    x = O.rms_norm(H.activations(349, 3, 4096), norm_weight(350, 4096))
    kv_d = [torch.from_numpy(k).cuda() for k in kvs]
    hid = torch.from_numpy(x).cuda()
    W.v4_attention(ctx, layer, pos, hid, kv_d, fr, [torch.from_numpy(c).cuda() for c in comps])
    ctx.sync()
    got = hid.cpu().numpy()
    for t, p in enumerate(pos):
        kv_h = kvs[t].copy()
        st, want = O.v4_attention(spec, p, x[t], kv_h, comps[t], fr)
        assert st == O.OK
        assert np.array_equal(bits(kv_d[t].cpu().numpy()[p]), bits(kv_h[p])), t
        assert np.array_equal(bits(got[t]), bits(want)), t
