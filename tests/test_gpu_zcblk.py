"""Expert loader parity on the GPU: FP4 expert blocks written in the
reference's ZCBLK01 / experts-pack format (by the package's writer, which
tests/test_zcblk_golden.py pins byte for byte to the reference converter)
are read from disk into HBM and must (a) land byte-identical to the source
arrays, (b) drive the MoE layer to outputs bit-identical to the same weights
uploaded directly, and (c) match the CPU oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HID, INT, E = 512, 256, 8


@pytest.fixture(scope="module")
def W():
    import wohper_b200

    wohper_b200.lib()
    return wohper_b200


@pytest.fixture(scope="module")
def ZB(W):
    from wohper_b200 import zcblk

    return zcblk


@pytest.fixture(scope="module")
def ctx(W):
    c = W.Context(0)
    yield c
    c.close()


def _arrays(seed):
    w1, s1 = H.fp4_matrix(seed, INT, HID)
    w3, s3 = H.fp4_matrix(seed + 1, INT, HID)
    w2, s2 = H.fp4_matrix(seed + 2, HID, INT)
    return w1, s1, w3, s3, w2, s2


def _model(ZB, tmp_path, pack=True, layers=(0, 1)):
    """Two layers of E experts; returns (model path, {(layer, expert): arrays})."""
    src, specs = {}, []
    for L in layers:
        ex = {}
        for e in range(E):
            a = _arrays(1000 * (L + 1) + 10 * e)
            src[(L, e)] = a
            ex[e] = ZB.deepseek_fp4_expert_tensors(f"layers.{L}.ffn.experts.{e}", *a)
        gate = ZB.BlockTensor(f"layers.{L}.ffn.gate.weight", 11, 2404, 9, (E, HID),
                              H.router_gate(7 + L, E, HID).tobytes())
        specs.append(ZB.LayerSpec(L, [gate], ex))
    out = tmp_path / "dense_core.bin"
    ZB.write_model(out, specs, hidden_size=HID, pack=pack)
    return out, src


def _check_bytes(expert, arrays):
    got = [t.cpu().numpy() for m in (expert.w1, expert.w3, expert.w2)
           for t in (m.packed_weight, m.ue8m0_scales)]
    w1, s1, w3, s3, w2, s2 = arrays
    for g, want in zip(got, (w1, s1, w3, s3, w2, s2)):
        np.testing.assert_array_equal(g, want.reshape(-1))
    assert (expert.w1.rows, expert.w1.cols, expert.w2.rows, expert.w2.cols) == (INT, HID, HID, INT)


def _torch_expert(W, arrays):
    w1, s1, w3, s3, w2, s2 = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]
    return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INT, HID, HID // 32),
                                 W.Fp4Matvec(w3, s3, INT, HID, HID // 32),
                                 W.Fp4Matvec(w2, s2, HID, INT, INT // 32))


def _oracle_expert(arrays, keep):
    w1, s1, w3, s3, w2, s2 = arrays
    return O.Fp4Expert(O.fp4_spec(w1, s1, INT, HID, HID // 32, keep),
                       O.fp4_spec(w3, s3, INT, HID, HID // 32, keep),
                       O.fp4_spec(w2, s2, HID, INT, INT // 32, keep))


def test_loader_pack_bytes_and_moe_parity(ctx, W, ZB, tmp_path):
    model, src = _model(ZB, tmp_path, pack=True)
    man = ZB.ModelManifest(model)
    assert man.layer_count() == 2 and man.expert_source(1, 3)[4] == ZB.SOURCE_PACK
    loader = ZB.ExpertLoader(ctx, man, threads=3)
    order = [5, 0, 7, 2, 1, 6, 3, 4]
    arena, experts = loader.load(1, order)
    torch.cuda.synchronize()
    by_id = dict(zip(order, experts))
    for e in range(E):
        _check_bytes(by_id[e], src[(1, e)])
    # the MoE layer over loaded weights == over directly uploaded weights == oracle
    shared_arrays = _arrays(77)
    blk = ZB.pack_block(ZB.deepseek_fp4_expert_tensors("layers.1.ffn.shared", *shared_arrays))
    shared = ZB.upload_fp4_expert(ctx, blk)
    _check_bytes(shared, shared_arrays)
    gate = H.router_gate(8, E, HID)
    g = torch.from_numpy(gate.view(np.int16)).cuda()
    loaded = W.MoeLayer(ctx, [by_id[e] for e in range(E)], shared, g, topk=6, max_tokens=4,
                        exact=1)
    direct = W.MoeLayer(ctx, [_torch_expert(W, src[(1, e)]) for e in range(E)],
                        _torch_expert(W, shared_arrays), g, topk=6, max_tokens=4, exact=1)
    x = H.activations(9, 3, HID)
    xd = torch.from_numpy(x).cuda()
    ids = torch.zeros(3, 6, dtype=torch.int32, device="cuda")
    wts = torch.zeros(3, 6, device="cuda")
    y1 = loaded.forward(xd, ids=ids, weights=wts)
    y2 = direct.forward(xd)
    ctx.sync()
    assert torch.equal(y1, y2)
    y1, ids, wts = y1.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    keep = []
    arr = (O.Fp4Expert * (E + 1))()
    for e in range(E):
        arr[e] = _oracle_expert(src[(1, e)], keep)
    arr[E] = _oracle_expert(shared_arrays, keep)
    diff = 0
    for t in range(3):
        n, oid, ow, _ = O.router(gate, x[t], 6, mode=0)
        np.testing.assert_array_equal(ids[t], oid)
        st, want = O.moe_combine_token(arr, oid, ow, arr[E], x[t])
        assert st == O.OK
        assert np.max(np.abs(y1[t] - want)) <= 1e-4 * float(np.abs(want).max())
        diff += int(np.sum(y1[t].view(np.uint32) != want.view(np.uint32)))
    assert diff == 0
    loaded.close()
    direct.close()
    loader.close()


@pytest.mark.parametrize("direct_io", [False, True])
def test_loader_shard_files_and_slot_reuse(ctx, W, ZB, tmp_path, direct_io):
    model, src = _model(ZB, tmp_path, pack=False)
    man = ZB.ModelManifest(model)
    assert man.expert_source(0, 0)[4] == ZB.SOURCE_SHARD
    loader = ZB.ExpertLoader(ctx, man, threads=2, direct_io=direct_io)
    for rep in range(2):  # the second pass reuses every staging slot
        for li in (0, 1):
            ids = list(range(E)) if rep == 0 else list(reversed(range(E)))
            _, experts = loader.load(li, ids)
            torch.cuda.synchronize()
            for e, ex in zip(ids, experts):
                _check_bytes(ex, src[(li, e)])
    loader.close()


def test_loader_errors(ctx, W, ZB, tmp_path):
    model, src = _model(ZB, tmp_path, pack=True)
    man = ZB.ModelManifest(model)
    loader = ZB.ExpertLoader(ctx, man, threads=4)
    need = loader.arena_bytes(0, [0, 1])
    small = torch.empty(need - 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(W.WohperError) as e:
        loader.load(0, [0, 1], arena=small)
    assert e.value.kind == "OutputTooSmall"
    with pytest.raises(W.WohperError) as e:
        loader.load(0, [0, 1], arena=torch.empty(need, dtype=torch.uint8))
    assert e.value.kind == "InvalidPointer"
    with pytest.raises(W.WohperError) as e:
        loader.load(0, [0, 42])
    assert e.value.kind == "InvalidExpert"
    # a corrupt block: the reader thread's parse error reaches the caller
    path, off, _db, _pb, _k = man.expert_source(0, 3)
    with open(path, "r+b") as f:
        f.seek(off)
        f.write(b"ZCBLK99\0")
    with pytest.raises(W.WohperError) as e:
        loader.load(0, list(range(E)))
    assert e.value.kind == "InvalidQuantBlockMagic"
    # the loader stays usable
    _, ex = loader.load(0, [0, 1, 2, 4])
    torch.cuda.synchronize()
    for e_, x in zip([0, 1, 2, 4], ex):
        _check_bytes(x, src[(0, e_)])
    loader.close()


def test_upload_expert_forward_matches_direct(ctx, W, ZB):
    arrays = _arrays(55)
    blk = ZB.pack_block(ZB.deepseek_fp4_expert_tensors("layers.0.ffn.experts.0", *arrays))
    ex = ZB.upload_fp4_expert(ctx, blk)
    _check_bytes(ex, arrays)
    x = torch.from_numpy(H.activations(56, 1, HID).reshape(-1)).cuda()
    n = W.deepseek_v4_fp4_expert_scratch_len(INT)
    y1 = torch.empty(HID, device="cuda")
    y2 = torch.empty(HID, device="cuda")
    W.deepseek_v4_fp4_expert_forward(ctx, ex, x, y1, torch.empty(n, device="cuda"))
    W.deepseek_v4_fp4_expert_forward(ctx, _torch_expert(W, arrays), x, y2,
                                     torch.empty(n, device="cuda"))
    ctx.sync()
    assert torch.equal(y1, y2)
    keep = []
    st, want = O.fp4_expert_forward(_oracle_expert(arrays, keep), x.cpu().numpy())
    assert st == O.OK
    np.testing.assert_array_equal(y1.cpu().numpy().view(np.uint32), want.view(np.uint32))
