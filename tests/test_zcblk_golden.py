"""ZCBLK01 / ZCINF01 format parity on CPU (no GPU needed: the parser, the
manifest loader and the writer are host code).

Golden data: tests/golden/zcblk/deepseek_tiny.tar.gz is the output of the
reference's own DeepSeek converter and experts-pack builder on a tiny
synthetic checkpoint, and expected.json records what the converter assigned
to every tensor (tests/golden/zcblk/make_zcblk_golden.py made both).

1. the oracle (oracle/zcblk.py) reads every block of the fixture back to the
   converter's names, codes, shapes and source bytes;
2. the C library agrees with the oracle field by field (header, layers,
   experts, sources, every tensor record, the FP4 suffix bridge);
3. the package's writer reproduces the reference's files byte for byte;
4. the same error kind and reason as the oracle on malformed blocks, manifests,
   shard maps and pack indexes, including the reference's own model_format.rs
   unit tests restated.
"""
from __future__ import annotations

import json
import shutil
import struct
import tarfile
from pathlib import Path

import numpy as np
import pytest

from oracle import zcblk as Z

HERE = Path(__file__).resolve().parent
GOLD = HERE / "golden" / "zcblk"
EXPECTED = json.loads((GOLD / "expected.json").read_text())

# oracle error kind -> wh_status
KIND_STATUS = {
    "InvalidQuantBlockMagic": 30, "UnsupportedQuantBlockVersion": 31,
    "TruncatedQuantBlock": 32, "InvalidQuantBlock": 33, "TensorIndexOutOfRange": 34,
    "InvalidShape": 2, "Io": 40, "InvalidMagic": 41, "UnsupportedVersion": 42,
    "Unaligned": 43, "TruncatedManifest": 44, "LayerCountMismatch": 45,
    "InvalidExpertTable": 46, "ShardMap": 47, "InvalidExpert": 48,
}
# kinds whose reason is a fixed string shared by the reference, the oracle and the library
EXACT_DETAIL = {"TruncatedQuantBlock", "InvalidQuantBlock", "InvalidShape", "Unaligned"}


@pytest.fixture(scope="module")
def W():
    import wohper_b200 as W

    W.lib()
    return W


@pytest.fixture(scope="module")
def ZB(W):
    from wohper_b200 import zcblk

    return zcblk


@pytest.fixture()
def tree(tmp_path):
    with tarfile.open(GOLD / "deepseek_tiny.tar.gz") as t:
        t.extractall(tmp_path, filter="data")
    return tmp_path


def _expert_blocks(m, model):
    out = {}
    for li, L in enumerate(m.layers):
        for e in L.experts:
            out[(li, e["expert_id"])] = Z.read_expert_block(m, model, li, e["expert_id"])
    return out


def _dense_block(m, model, li):
    L = m.layers[li]
    with open(model, "rb") as f:
        f.seek(L.dense_offset)
        return f.read(L.dense_payload_bytes)


def _block_name(L, eid=None):
    if eid is not None:
        return f"layer{L.layer_id}_expert{eid}"
    return "global_aux" if L.flags & 0xFF == Z.LAYER_BLOCK_GLOBAL_AUX else f"dense_layer_{L.layer_id}"


# --------------------------------------------------------------------------
# 1. oracle vs the reference converter's output
def test_oracle_reads_reference_converter_output(tree):
    import hashlib

    model = tree / "dense_core.bin"
    m = Z.load_manifest(model)
    assert m.header["num_layers"] == 3 and m.header["hidden_size"] == EXPECTED["hidden"]
    assert [(L.layer_id, L.flags, len(L.experts)) for L in m.layers] == [(0, 1, 0), (0, 0, 4),
                                                                         (1, 0, 4)]
    assert m.pack_file is not None and len(m.pack) == 8 and len(m.shards) == 8
    blocks = {_block_name(L): _dense_block(m, model, li) for li, L in enumerate(m.layers)}
    for (li, eid), b in _expert_blocks(m, model).items():
        blocks[_block_name(m.layers[li], eid)] = b
    assert set(blocks) == set(EXPECTED["blocks"])
    for name, b in blocks.items():
        h = Z.parse_quant_block(b)
        got = [Z.tensor(b, h, i) for i in range(h.tensor_count)]
        assert [t.name.decode() for t in got] == EXPECTED["blocks"][name]
        for t in got:
            x = EXPECTED["tensors"][t.name.decode()]
            assert (t.dtype_original, t.quant_format, t.role, t.dims) == \
                (x["dtype_original"], x["quant_format"], x["role"], x["shape"])
            assert hashlib.sha256(b[t.data_pos:t.data_pos + t.data_len]).hexdigest() == x["sha256"]
    w1, w3, w2 = Z.fp4_expert_from_block(blocks["layer1_expert2"])
    assert (w1.rows, w1.cols, w1.scale_cols) == (EXPECTED["inter"], EXPECTED["hidden"], 2)
    assert (w2.rows, w2.cols, w2.scale_cols) == (EXPECTED["hidden"], EXPECTED["inter"], 1)


# --------------------------------------------------------------------------
# 2. the C library vs the oracle
def _c_status(W, fn):
    try:
        return 0, fn()
    except W.WohperError as e:
        return e.status, str(e).split(": ", 1)[1] if ": " in str(e) else ""


def test_library_block_parse_matches_oracle(tree, W, ZB):
    model = tree / "dense_core.bin"
    m = Z.load_manifest(model)
    blocks = [_dense_block(m, model, li) for li in range(len(m.layers))]
    blocks += list(_expert_blocks(m, model).values())
    for b in blocks:
        h = Z.parse_quant_block(b)
        ch = ZB.parse_quant_block(b)
        assert (ch.tensor_count, ch.quant_format, ch.flags, ch.record_table_offset,
                ch.names_offset) == (h.tensor_count, h.quant_format, h.flags,
                                     h.record_table_offset, h.names_offset)
        for i in range(h.tensor_count):
            t, ct = Z.tensor(b, h, i), ZB.block_tensor(b, i)
            assert (ct.dtype_original, ct.quant_format, ct.rank, ct.flags, ct.data_pos,
                    ct.data_len, ct.shape_pos) == (t.dtype_original, t.quant_format, t.rank,
                                                   t.flags, t.data_pos, t.data_len, t.shape_pos)
            assert b[ct.name_pos:ct.name_pos + ct.name_len] == t.name
            assert (ct.scale, ct.zero_point) == (t.scale, t.zero_point)
            assert ZB.tensor_dims(b, ct) == t.dims
        st, _ = _c_status(W, lambda: ZB.block_tensor(b, h.tensor_count))
        assert st == KIND_STATUS["TensorIndexOutOfRange"]
    for b in _expert_blocks(m, model).values():
        want = Z.fp4_expert_from_block(b)
        v = ZB.deepseek_v4_fp4_expert_from_quant_block(b)
        for o, c in zip(want, (v.w1, v.w3, v.w2)):
            assert (c.weight_pos, c.weight_len, c.scale_pos, c.scale_len, c.rows, c.cols,
                    c.scale_cols) == (o.weight_pos, o.weight_len, o.scale_pos, o.scale_len,
                                      o.rows, o.cols, o.scale_cols)
        t = ZB.find_tensor_by_suffix(b, ".w3.weight")
        assert b[t.name_pos:t.name_pos + t.name_len].endswith(b".w3.weight")


def _manifest_view_oracle(m, model):
    layers = [(L.layer_id, L.flags, L.dense_offset, L.dense_disk_bytes, L.dense_payload_bytes,
               L.dense_dequant_bytes, [tuple(e[k] for k in Z.EXPERT_FIELDS) for e in L.experts])
              for L in m.layers]
    srcs = {}
    for li, L in enumerate(m.layers):
        for e in L.experts:
            p, off, db, pb = Z.expert_source(m, model, li, e["expert_id"])
            srcs[(li, e["expert_id"])] = (str(p), off, db, pb)
    return layers, srcs


def _manifest_view_lib(cm):
    layers, srcs = [], {}
    for li in range(cm.layer_count()):
        d = cm.layer(li)
        ex = cm.experts(li)
        layers.append((d.layer_id, d.flags, d.dense_offset, d.dense_disk_bytes,
                       d.dense_payload_bytes, d.dense_dequant_bytes,
                       [tuple(getattr(e, k) for k in Z.EXPERT_FIELDS) for e in ex]))
        for e in ex:
            p, off, db, pb, _kind = cm.expert_source(li, e.expert_id)
            srcs[(li, e.expert_id)] = (p, off, db, pb)
    return layers, srcs


def test_library_manifest_matches_oracle(tree, W, ZB):
    model = tree / "dense_core.bin"
    m = Z.load_manifest(model)
    cm = ZB.ModelManifest(model)
    h = cm.header
    for k in Z.ENGINE_FIELDS:
        v = getattr(h, k)
        assert (bytes(v) if k == "magic" else v) == m.header[k], k
    assert _manifest_view_lib(cm) == _manifest_view_oracle(m, model)
    assert cm.expert_source(1, 2)[4] == ZB.SOURCE_PACK
    st, _ = _c_status(W, lambda: cm.expert_source(1, 99))
    assert st == KIND_STATUS["InvalidExpert"]
    assert cm.read_expert_block(2, 3) == Z.read_expert_block(m, model, 2, 3)


def test_shard_file_path(tree, W, ZB):
    """Without the pack index, experts resolve to their shard files; cut the
    shards back out of the pack (build_experts_pack copies them verbatim)."""
    model = tree / "dense_core.bin"
    m = Z.load_manifest(model)
    pack = (tree / "dense_core.experts_pack.bin").read_bytes()
    shards = json.loads((tree / "dense_core.shards.json").read_text())
    index = json.loads((tree / "dense_core.experts_pack.index.json").read_text())
    pos = {(e["layer_id"], e["expert_id"]): e for e in index["entries"]}
    for s in shards["experts"]:
        e = pos[(s["layer_id"], s["expert_id"])]
        p = tree / s["path"]
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_bytes(pack[e["offset"]:e["offset"] + e["disk_bytes"]])
    before = _expert_blocks(m, model)
    (tree / "dense_core.experts_pack.index.json").unlink()
    m2 = Z.load_manifest(model)
    cm = ZB.ModelManifest(model)
    assert m2.pack_file is None
    assert _manifest_view_lib(cm) == _manifest_view_oracle(m2, model)
    for (li, eid), b in before.items():
        path, off, _db, _pb, kind = cm.expert_source(li, eid)
        assert kind == ZB.SOURCE_SHARD and off == 0 and path.endswith(f"expert{eid}.zcblk")
        assert cm.read_expert_block(li, eid) == b == Z.read_expert_block(m2, model, li, eid)


# --------------------------------------------------------------------------
# 3. the writer reproduces the reference's bytes
def _tensors_of(b):
    from wohper_b200.zcblk import BlockTensor

    h = Z.parse_quant_block(b)
    out = []
    for i in range(h.tensor_count):
        t = Z.tensor(b, h, i)
        out.append(BlockTensor(t.name.decode(), t.dtype_original, t.quant_format, t.flags,
                               tuple(t.dims), b[t.data_pos:t.data_pos + t.data_len], t.scale,
                               t.zero_point))
    return out


def test_writer_reproduces_reference_files(tree, tmp_path, ZB):
    model = tree / "dense_core.bin"
    m = Z.load_manifest(model)
    eb = _expert_blocks(m, model)
    for b in eb.values():
        assert ZB.pack_block(_tensors_of(b)) == b
    glob = _tensors_of(_dense_block(m, model, 0))
    layers = []
    for li in (1, 2):
        L = m.layers[li]
        layers.append(ZB.LayerSpec(L.layer_id, _tensors_of(_dense_block(m, model, li)),
                                   {e["expert_id"]: _tensors_of(eb[(li, e["expert_id"])])
                                    for e in L.experts}))
    out = tmp_path / "w" / "dense_core.bin"
    ZB.write_model(out, layers, hidden_size=EXPECTED["hidden"], global_tensors=glob,
                   num_attention_heads=2, num_kv_heads=1, active_experts_per_token=2)
    assert out.read_bytes() == model.read_bytes()
    ref_map = json.loads((tree / "dense_core.shards.json").read_text())
    our_map = json.loads((out.parent / "dense_core.shards.json").read_text())
    assert our_map["format"] == ref_map["format"] and our_map["experts"] == ref_map["experts"]
    ZB.build_experts_pack(out)
    assert (out.parent / "dense_core.experts_pack.bin").read_bytes() == \
        (tree / "dense_core.experts_pack.bin").read_bytes()
    ours = json.loads((out.parent / "dense_core.experts_pack.index.json").read_text())
    ref = json.loads((tree / "dense_core.experts_pack.index.json").read_text())
    assert ours == ref
    assert not (out.parent / "experts" / "layer0_expert0.zcblk").exists()
    # pack=True writes the same pack directly
    out2 = tmp_path / "w2" / "dense_core.bin"
    ZB.write_model(out2, layers, hidden_size=EXPECTED["hidden"], global_tensors=glob,
                   num_attention_heads=2, num_kv_heads=1, active_experts_per_token=2, pack=True)
    assert out2.read_bytes() == model.read_bytes()
    assert (out2.parent / "dense_core.experts_pack.bin").read_bytes() == \
        (tree / "dense_core.experts_pack.bin").read_bytes()
    assert json.loads((out2.parent / "dense_core.experts_pack.index.json").read_text()) == ref


# --------------------------------------------------------------------------
# 4. errors: same kind and reason as the oracle
def _oracle_err(fn):
    try:
        fn()
        return None
    except Z.FormatError as e:
        return e.kind, e.detail


def _same_error(W, oracle_fn, lib_fn, what):
    want = _oracle_err(oracle_fn)
    st, detail = _c_status(W, lib_fn)
    if want is None:
        assert st == 0, (what, st, detail)
        return
    assert st == KIND_STATUS[want[0]], (what, want, st, detail)
    if want[0] in EXACT_DETAIL:
        assert detail == want[1], (what, want, detail)


def _mutations(b):
    """(label, mutated block) pairs covering every check of the parser and
    the FP4 suffix bridge."""
    h = Z.parse_quant_block(b)
    ts = [Z.tensor(b, h, i) for i in range(h.tensor_count)]
    rec = lambda i: h.record_table_offset + 52 * i  # noqa: E731
    by = {t.name.decode().rsplit(".", 2)[-2] + "." + t.name.decode().rsplit(".", 1)[-1]: i
          for i, t in enumerate(ts)}

    def put(buf, off, fmt, v):
        buf = bytearray(buf)
        struct.pack_into(fmt, buf, off, v)
        return bytes(buf)

    w1w, w1s, w2w = by["w1.weight"], by["w1.scale"], by["w2.weight"]
    out = [
        ("ok", b),
        ("empty", b""),
        ("short header", b[:39]),
        ("magic", b"ZCBLK02\0" + b[8:]),
        ("version", put(b, 8, "<I", 2)),
        ("record table beyond", put(b, 12, "<I", 10_000)),
        ("record table before header", put(b, 24, "<Q", 8)),
        ("record table overflow", put(b, 24, "<Q", 2 ** 64 - 8)),
        ("names beyond", put(b, 32, "<Q", len(b) + 1)),
        ("truncated in data", b[:ts[-1].data_pos + 3]),
        ("name offset beyond", put(b, rec(w1w) + 12, "<Q", len(b))),
        ("name offset overflow", put(b, rec(w1w) + 12, "<Q", 2 ** 64 - 1)),
        ("name length beyond", put(b, ts[w1w].name_pos - 2, "<H", 65535)),
        ("shape offset beyond", put(b, rec(w1s) + 20, "<Q", len(b) - 2)),
        ("shape rank mismatch", put(b, rec(w1s) + 4, "<I", 3)),
        ("data beyond", put(b, rec(w2w) + 36, "<Q", len(b))),
        ("data overflow", put(b, rec(w2w) + 28, "<Q", 2 ** 64 - 4)),
        ("weight not fp4", put(b, rec(w1w) + 2, "<H", 2401)),
        ("scale not ue8m0", put(b, rec(w1s) + 2, "<H", 2404)),
        ("weight rank 1", put(put(b, rec(w1w) + 4, "<I", 1), ts[w1w].shape_pos, "<I", 1)),
        ("zero rows", put(b, ts[w1w].shape_pos + 4, "<Q", 0)),
        ("scale rows differ", put(b, ts[w1s].shape_pos + 4, "<Q", 31)),
        ("weight too small", put(b, rec(w1w) + 36, "<Q", ts[w1w].data_len - 1)),
        ("scale too small", put(b, rec(w1s) + 36, "<Q", ts[w1s].data_len - 1)),
        ("weight size overflow", put(put(b, ts[w1w].shape_pos + 4, "<Q", 2 ** 62),
                                     ts[w1s].shape_pos + 4, "<Q", 2 ** 62)),
        ("projection mismatch", put(b, ts[w2w].shape_pos + 12, "<Q", 8)),
        ("missing suffix", bytes(b).replace(b".w3.weight", b".w9.weight")),
        ("duplicate suffix", bytes(b).replace(b".w3.weight", b".w1.weight")),
    ]
    return out


def test_block_errors_match_oracle(tree, W, ZB):
    model = tree / "dense_core.bin"
    m = Z.load_manifest(model)
    b = Z.read_expert_block(m, model, 1, 0)
    for label, mb in _mutations(b):
        _same_error(W, lambda: Z.fp4_expert_from_block(mb),
                    lambda: ZB.deepseek_v4_fp4_expert_from_quant_block(mb), label)
        _same_error(W, lambda: [Z.tensor(mb, Z.parse_quant_block(mb), i)
                                for i in range(Z.parse_quant_block(mb).tensor_count)],
                    lambda: [ZB.block_tensor(mb, i)
                             for i in range(ZB.parse_quant_block(mb).tensor_count)],
                    label + " (records)")


def _write_json(p, obj):
    p.write_text(obj if isinstance(obj, str) else json.dumps(obj))


def _manifest_mutations(tree):
    model = tree / "dense_core.bin"
    raw = model.read_bytes()
    hdr = dict(zip(Z.ENGINE_FIELDS, Z.ENGINE_HEADER.unpack_from(raw, 0)))
    mo = hdr["manifest_offset"]
    mh = Z.MANIFEST_HEADER.unpack_from(raw, mo)
    lo, eo = mo + mh[4], mo + mh[5]

    def put(off, fmt, v):
        b = bytearray(raw)
        struct.pack_into(fmt, b, off, v)
        return bytes(b)

    shards = json.loads((tree / "dense_core.shards.json").read_text())
    index = json.loads((tree / "dense_core.experts_pack.index.json").read_text())
    U = Z.ENGINE_HEADER.size
    return [
        ("ok", raw, None, None),
        ("magic", b"ZCINF02\0" + raw[8:], None, None),
        ("version", put(8, "<I", 2), None, None),
        ("block alignment", put(104, "<I", 4096), None, None),
        ("manifest offset unaligned", put(24, "<Q", mo + 8), None, None),
        ("tokenizer offset unaligned", put(40, "<Q", 7), None, None),
        ("router metadata unaligned", put(56, "<Q", 7), None, None),
        ("truncated header", raw[:U - 1], None, None),
        ("layer count", put(80, "<I", 4), None, None),
        ("layer table beyond EOF", put(mo + 16, "<Q", len(raw)), None, None),
        ("dense offset unaligned", put(lo + 8, "<Q", 4096), None, None),
        ("dense disk unaligned", put(lo + 72 + 16, "<Q", 4096), None, None),
        ("expert table range", put(lo + 72 + 48, "<I", 99), None, None),
        ("expert layer id", put(eo + 56 * 5, "<I", 0), None, None),
        ("expert disk unaligned", put(eo + 56 * 2 + 16, "<Q", 4096), None, None),
        ("expert offset unaligned", put(eo + 56 * 2 + 8, "<Q", 4096), None, None),
        ("shard map format", raw, dict(shards, format="other"), None),
        ("shard map legacy format", raw, dict(shards, format="zeroclaw-sharded-experts"), None),
        ("shard map not json", raw, "{", None),
        ("shard map missing field", raw,
         dict(shards, experts=[{k: v for k, v in shards["experts"][0].items() if k != "path"}]),
         None),
        ("shard map negative", raw,
         dict(shards, experts=[dict(shards["experts"][0], layer_id=-1)]), None),
        ("shard map u32 overflow", raw,
         dict(shards, experts=[dict(shards["experts"][0], expert_id=2 ** 32)]), None),
        ("shard map float", raw,
         dict(shards, experts=[dict(shards["experts"][0], disk_bytes=2097152.0)]), None),
        ("shard map unaligned", raw,
         dict(shards, experts=[dict(shards["experts"][0], disk_bytes=4096)]), None),
        ("shard map defaults", raw,
         dict(shards, experts=[{k: v for k, v in shards["experts"][0].items()
                                if k not in ("dequant_bytes", "quant_format", "checksum")}]),
         None),
        ("shard map duplicate field", raw,
         '{"format": "wohper-sharded-experts", "experts": [{"layer_id": 0, "layer_id": 1, '
         '"expert_id": 0, "path": "a", "disk_bytes": 0, "payload_bytes": 0}]}', None),
        ("shard map unicode path", raw,
         '{"format": "wohper-sharded-experts", "experts": [{"layer_id": 0, "expert_id": 1, '
         '"path": "experts/\\u00e9\\ud83d\\ude00.zcblk", "disk_bytes": 2097152, '
         '"payload_bytes": 1}]}', "DELETE"),
        ("pack format", raw, None, dict(index, format="x")),
        ("pack legacy format", raw, None, dict(index, format="zeroclaw-experts-pack")),
        ("pack file missing", raw, None, dict(index, pack_file="nope.bin")),
        ("pack offset unaligned", raw, None,
         dict(index, entries=[dict(index["entries"][0], offset=4096)])),
        ("pack disk unaligned", raw, None,
         dict(index, entries=[dict(index["entries"][0], disk_bytes=4096)])),
        ("pack missing field", raw, None,
         dict(index, entries=[{k: v for k, v in index["entries"][0].items() if k != "offset"}])),
        ("pack entries not a list", raw, None, dict(index, entries={})),
    ]


def test_manifest_errors_match_oracle(tree, W, ZB):
    model = tree / "dense_core.bin"
    orig = {p: p.read_bytes() for p in (model, tree / "dense_core.shards.json",
                                        tree / "dense_core.experts_pack.index.json")}
    for label, raw, shard_map, pack_index in _manifest_mutations(tree):
        for p, b in orig.items():
            p.write_bytes(b)
        model.write_bytes(raw)
        for p, v in ((tree / "dense_core.shards.json", shard_map),
                     (tree / "dense_core.experts_pack.index.json", pack_index)):
            if v == "DELETE":
                p.unlink()
            elif v is not None:
                _write_json(p, v)
        _same_error(W, lambda: Z.load_manifest(model), lambda: ZB.ModelManifest(model), label)
        if _oracle_err(lambda: Z.load_manifest(model)) is None:
            m = Z.load_manifest(model)
            cm = ZB.ModelManifest(model)
            assert _manifest_view_lib(cm) == _manifest_view_oracle(m, model), label
    st, _ = _c_status(W, lambda: ZB.ModelManifest(tree / "missing.bin"))
    assert st == KIND_STATUS["Io"]


def _rust_unit_model(tmp_path, shard_experts, layers):
    """A model file holding `layers` (flags, layer_id, [expert ids]) with
    2 MB-aligned placeholder blocks and a shard map, as the reference's
    model_format.rs tests set up their manifests in memory
    (src/model_format.rs:567-709)."""
    A = Z.ALIGN_2MB
    experts = [(lid, eid) for flags, lid, ids in layers for eid in ids]
    man = bytearray(Z.MANIFEST_HEADER.pack(len(layers), len(experts), 0, 0, 40,
                                           40 + 72 * len(layers),
                                           40 + 72 * len(layers) + 56 * len(experts)))
    first = 0
    for flags, lid, ids in layers:
        man += Z.LAYER_DESC.pack(lid, flags, A, A, 16, 16, 0, 0, first, len(ids), 2400, 1, 0)
        first += len(ids)
    for lid, eid in experts:
        man += Z.EXPERT_DESC.pack(lid, eid, 0, A, 16, 16, 2400, eid, 11)
    hdr = Z.ENGINE_HEADER.pack(Z.MODEL_MAGIC, 1, 0, 2 * A, A, len(man), 0, 0, 0, 0, 2, 2,
                               len(layers), 64, 0, 0, 4, 2, A, 2400, 0, 0)
    model = tmp_path / "dense_core.bin"
    model.write_bytes(hdr + b"\0" * (A - len(hdr)) + bytes(man))
    entries = [dict(layer_id=l, expert_id=e, path=f"experts/layer{l}_expert{e}.zcblk",
                    disk_bytes=A, payload_bytes=16, dequant_bytes=16, quant_format=2400,
                    checksum=11 * (e + 1)) for l, e in shard_experts]
    (tmp_path / "dense_core.shards.json").write_text(
        json.dumps({"format": "wohper-sharded-experts", "experts": entries}))
    return model


def test_reference_shard_map_unit_tests(tmp_path, W, ZB):
    """shard_map_ignores_catalog_entries_outside_compact_manifest and
    shard_map_merge_extends_compute_layer_expert_table
    (src/model_format.rs:567-709), through the oracle and the library."""
    d1 = tmp_path / "a"
    d1.mkdir()
    model = _rust_unit_model(d1, [(0, 0), (0, 8)], [(0, 0, [0])])
    m = Z.load_manifest(model)
    cm = ZB.ModelManifest(model)
    assert sorted(m.shards) == [(0, 0)] and len(m.layers[0].experts) == 1
    assert cm.layer(0).num_experts == 1
    assert cm.expert_source(0, 0)[4] == ZB.SOURCE_SHARD
    st, _ = _c_status(W, lambda: cm.expert_source(0, 8))
    assert st == KIND_STATUS["InvalidExpert"]

    d2 = tmp_path / "b"
    d2.mkdir()
    model = _rust_unit_model(d2, [(0, 0), (0, 8), (1, 3)], [(1, 0, []), (0, 0, [0])])
    m = Z.load_manifest(model, merge_sidecar_experts=True)
    cm = ZB.ModelManifest(model, merge_sidecar_experts=True)
    assert sorted(m.shards) == [(0, 0), (0, 8)]
    assert m.layers[0].experts == [] and [e["expert_id"] for e in m.layers[1].experts] == [0, 8]
    e8 = m.layers[1].experts[1]
    assert (e8["disk_offset"], e8["quant_format"], e8["dequant_bytes"]) == (0, 2400, 16)
    assert _manifest_view_lib(cm) == _manifest_view_oracle(m, model)
    assert cm.layer(0).num_experts == 0 and cm.layer(1).num_experts == 2
    assert cm.expert_source(1, 8)[4] == ZB.SOURCE_SHARD
