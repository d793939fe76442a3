"""TEST INFRASTRUCTURE ONLY: a CPU restatement of the reference's ZCBLK01 block
parser, its DeepSeek FP4 expert suffix bridge and the ZCINF01 manifest loader
(Wohper, engine/zc_infer_core).  Only tests/ and bench.py's cpu_baseline /
``--impl reference`` arm use it, as the checker or the timed CPU baseline; the
product package ``wohper_b200`` never imports it.

Every function names the Rust function it restates (path:line inside the
reference project).  Errors are raised as ``FormatError(kind, detail)`` where
``kind`` is the variant name of ComputeError (src/compute.rs:329-343) or
ModelFormatError (src/model_format.rs:31-55) and ``detail`` is the variant's
&'static str payload (or, for Unaligned, the field name), so a test can compare
the kind and the reason with the C library's status and detail string.

Parity pin: tests/test_zcblk_golden.py checks this module against blocks,
manifests, shard maps and experts packs written by the reference's own
converter (tools/stream_convert_deepseek_v4.py) and pack builder
(tools/build_experts_pack.py), committed as tests/golden/zcblk/.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

# src/model_format.rs:10-20
MODEL_MAGIC = b"ZCINF01\0"
QUANT_BLOCK_MAGIC = b"ZCBLK01\0"
FORMAT_VERSION = 1
QUANT_BLOCK_VERSION = 1
QUANT_BLOCK_HEADER_SIZE = 40
QUANT_TENSOR_RECORD_SIZE = 52
LAYER_BLOCK_COMPUTE = 0
LAYER_BLOCK_GLOBAL_AUX = 1
ALIGN_2MB = 2 * 1024 * 1024  # src/lib.rs:10

# src/deepseek_v4.rs:41-47
QUANT_DEEPSEEK_RAW_MIXED = 2400
QUANT_DEEPSEEK_FP8_E4M3 = 2401
QUANT_DEEPSEEK_FP4_E2M1_PACKED = 2402
QUANT_DEEPSEEK_UE8M0_SCALE = 2403

U64_MAX = (1 << 64) - 1

# EngineHeader (src/model_format.rs:57-81), ManifestHeader (:83-93),
# LayerBlockDescDisk (:95-111), ExpertBlockDescDisk (:113-125): #[repr(C)]
# structs read raw from the file, little-endian.
ENGINE_HEADER = struct.Struct("<8sIIQQQQQQQIIIIIIIIIIQQ")
MANIFEST_HEADER = struct.Struct("<IIIIQQQ")
LAYER_DESC = struct.Struct("<IIQQQQIIIIIIQ")
EXPERT_DESC = struct.Struct("<IIQQQQIIQ")
ENGINE_FIELDS = ("magic", "version", "endian", "file_size", "manifest_offset", "manifest_size",
                 "tokenizer_offset", "tokenizer_size", "router_metadata_offset",
                 "router_metadata_size", "model_family", "architecture", "num_layers",
                 "hidden_size", "num_attention_heads", "num_kv_heads", "experts_per_layer",
                 "active_experts_per_token", "block_alignment", "disk_quant_format",
                 "manifest_checksum", "file_checksum")
LAYER_FIELDS = ("layer_id", "flags", "dense_offset", "dense_disk_bytes", "dense_payload_bytes",
                "dense_dequant_bytes", "tensor_count", "first_tensor_index",
                "first_expert_index", "num_experts", "quant_format", "checksum_kind", "checksum")
EXPERT_FIELDS = ("layer_id", "expert_id", "disk_offset", "disk_bytes", "payload_bytes",
                 "dequant_bytes", "quant_format", "route_rank_hint", "checksum")


class FormatError(Exception):
    def __init__(self, kind: str, detail: str = ""):
        super().__init__(f"{kind}: {detail}")
        self.kind = kind
        self.detail = detail


# --------------------------------------------------------------------------
# little-endian field reads: read_le_bytes and friends (src/compute.rs:7175-7214)
def _le(buf: bytes, off: int, n: int, fmt: str, fld: str):
    if off + n > U64_MAX:
        raise FormatError("InvalidQuantBlock", "read range overflow")
    if off + n > len(buf):
        raise FormatError("TruncatedQuantBlock", fld)
    return struct.unpack_from(fmt, buf, off)[0]


def _u16(b, o, f):
    return _le(b, o, 2, "<H", f)


def _u32(b, o, f):
    return _le(b, o, 4, "<I", f)


def _u64(b, o, f):
    return _le(b, o, 8, "<Q", f)


def _f32(b, o, f):
    return _le(b, o, 4, "<f", f)


@dataclass
class BlockHeader:
    tensor_count: int
    quant_format: int
    flags: int
    record_table_offset: int
    names_offset: int


@dataclass
class Tensor:
    dtype_original: int
    quant_format: int
    rank: int
    flags: int
    name: bytes
    name_pos: int
    shape_pos: int
    dims: list
    data_pos: int
    data_len: int
    scale: float
    zero_point: float

    @property
    def role(self) -> int:  # QuantTensorLayout::role (src/compute.rs:501-505)
        return self.flags & 0xFFFF


def parse_quant_block(buf: bytes) -> BlockHeader:
    """parse_quant_block (src/compute.rs:1099-1147)."""
    if len(buf) < QUANT_BLOCK_HEADER_SIZE:
        raise FormatError("TruncatedQuantBlock", "block header")
    if bytes(buf[0:8]) != QUANT_BLOCK_MAGIC:
        raise FormatError("InvalidQuantBlockMagic", "")
    version = _u32(buf, 8, "block.version")
    if version != QUANT_BLOCK_VERSION:
        raise FormatError("UnsupportedQuantBlockVersion", str(version))
    count = _u32(buf, 12, "block.tensor_count")
    qf = _u32(buf, 16, "block.quant_format")
    flags = _u32(buf, 20, "block.flags")
    rto = _u64(buf, 24, "block.record_table_offset")
    nmo = _u64(buf, 32, "block.names_offset")
    record_bytes = count * QUANT_TENSOR_RECORD_SIZE
    record_end = rto + record_bytes
    if record_end > U64_MAX:
        raise FormatError("InvalidQuantBlock", "record table range overflow")
    if rto < QUANT_BLOCK_HEADER_SIZE or record_end > len(buf):
        raise FormatError("TruncatedQuantBlock", "record table")
    if nmo > len(buf):
        raise FormatError("TruncatedQuantBlock", "names blob")
    return BlockHeader(count, qf, flags, rto, nmo)


def read_name_blob(buf: bytes, names_offset: int, name_offset: int):
    """read_name_blob (src/compute.rs:7136-7154): [len:u16][bytes]."""
    absolute = names_offset + name_offset
    if absolute > U64_MAX:
        raise FormatError("InvalidQuantBlock", "name offset overflow")
    n = _u16(buf, absolute, "name.len")
    start = absolute + 2
    end = start + n
    if end > len(buf):
        raise FormatError("TruncatedQuantBlock", "name blob")
    return bytes(buf[start:end]), start


def read_shape_layout(buf: bytes, shape_offset: int, expected_rank: int):
    """read_shape_layout (src/compute.rs:7156-7178): [rank:u32][dims:u64 x rank]."""
    rank = _u32(buf, shape_offset, "shape.rank")
    if rank != expected_rank:
        raise FormatError("InvalidQuantBlock", "shape rank mismatch")
    end = shape_offset + 4 + rank * 8
    if end > U64_MAX:
        raise FormatError("InvalidQuantBlock", "shape end overflow")
    if end > len(buf):
        raise FormatError("TruncatedQuantBlock", "shape blob")
    return [struct.unpack_from("<Q", buf, shape_offset + 4 + 8 * i)[0] for i in range(rank)]


def tensor(buf: bytes, h: BlockHeader, index: int) -> Tensor:
    """QuantBlockLayout::tensor (src/compute.rs:545-595)."""
    if index >= h.tensor_count:
        raise FormatError("TensorIndexOutOfRange", f"index={index}, count={h.tensor_count}")
    ro = h.record_table_offset + index * QUANT_TENSOR_RECORD_SIZE
    if ro + QUANT_TENSOR_RECORD_SIZE > len(buf):
        raise FormatError("TruncatedQuantBlock", "tensor record")
    rec = bytes(buf[ro:ro + QUANT_TENSOR_RECORD_SIZE])
    dt, qf, rank, flags, name_off, shape_off, data_off, data_len, sc, zp = struct.unpack(
        "<HHIIQQQQff", rec)
    name, name_pos = read_name_blob(buf, h.names_offset, name_off)
    dims = read_shape_layout(buf, shape_off, rank)
    end = data_off + data_len
    if end > U64_MAX:
        raise FormatError("InvalidQuantBlock", "tensor data range overflow")
    if end > len(buf):
        raise FormatError("TruncatedQuantBlock", "tensor data")
    return Tensor(dt, qf, rank, flags, name, name_pos, shape_off, dims, data_off, data_len, sc, zp)


def element_count(t: Tensor) -> int:
    """ShapeLayout::element_count (src/compute.rs:522-531)."""
    n = 1
    for d in t.dims:
        n *= d
        if n > U64_MAX:
            raise FormatError("InvalidQuantBlock", "shape element count overflow")
    return n


def tensor_by_role(buf: bytes, h: BlockHeader, role: int) -> Optional[Tensor]:
    """QuantBlockLayout::tensor_by_role (src/compute.rs:601-612)."""
    for i in range(h.tensor_count):
        t = tensor(buf, h, i)
        if t.role == role:
            return t
    return None


def find_tensor_by_suffix(buf: bytes, h: BlockHeader, suffix: bytes) -> Tensor:
    """find_tensor_by_suffix (src/compute.rs:1149-1169)."""
    found = None
    for i in range(h.tensor_count):
        t = tensor(buf, h, i)
        if t.name.endswith(suffix):
            if found is not None:
                raise FormatError("InvalidQuantBlock", "duplicate DeepSeek expert tensor suffix")
            found = t
    if found is None:
        raise FormatError("InvalidQuantBlock", "missing DeepSeek expert tensor suffix")
    return found


@dataclass
class Fp4View:
    weight_pos: int
    weight_len: int
    scale_pos: int
    scale_len: int
    rows: int
    cols: int
    scale_cols: int


def fp4_matvec_from_tensors(w: Tensor, s: Tensor) -> Fp4View:
    """deepseek_fp4_matvec_from_tensors (src/compute.rs:1199-1247)."""
    if w.quant_format != QUANT_DEEPSEEK_FP4_E2M1_PACKED:
        raise FormatError("InvalidQuantBlock", "DeepSeek expert weight is not FP4 E2M1 packed")
    if s.quant_format != QUANT_DEEPSEEK_UE8M0_SCALE:
        raise FormatError("InvalidQuantBlock", "DeepSeek expert scale is not UE8M0")
    if w.rank != 2 or s.rank != 2:
        raise FormatError("InvalidShape", "DeepSeek FP4 expert rank")
    rows, packed_cols = w.dims
    scale_rows, scale_cols = s.dims
    if rows == 0 or packed_cols == 0 or scale_cols == 0 or scale_rows != rows:
        raise FormatError("InvalidShape", "DeepSeek FP4 expert shape")
    cols = packed_cols * 2
    if cols > U64_MAX:
        raise FormatError("InvalidShape", "DeepSeek FP4 expert cols overflow")
    req_w = rows * packed_cols
    if req_w > U64_MAX:
        raise FormatError("InvalidShape", "DeepSeek FP4 expert weight overflow")
    if w.data_len < req_w:
        raise FormatError("TruncatedQuantBlock", "DeepSeek FP4 expert weight")
    req_s = rows * scale_cols
    if req_s > U64_MAX:
        raise FormatError("InvalidShape", "DeepSeek FP4 expert scale overflow")
    if s.data_len < req_s:
        raise FormatError("TruncatedQuantBlock", "DeepSeek FP4 expert scale")
    return Fp4View(w.data_pos, req_w, s.data_pos, req_s, rows, cols, scale_cols)


def fp4_expert_from_block(buf: bytes):
    """parse_quant_block + deepseek_v4_fp4_expert_from_quant_block
    (src/compute.rs:1249-1267): w1, w3, w2 by name suffix."""
    h = parse_quant_block(buf)
    views = []
    for p in (b".w1", b".w3", b".w2"):
        w = find_tensor_by_suffix(buf, h, p + b".weight")
        s = find_tensor_by_suffix(buf, h, p + b".scale")
        views.append(fp4_matvec_from_tensors(w, s))
    w1, w3, w2 = views
    if w1.cols != w3.cols or w1.rows != w3.rows or w2.cols != w1.rows:
        raise FormatError("InvalidShape", "DeepSeek FP4 expert projection")
    return w1, w3, w2


# --------------------------------------------------------------------------
# ZCINF01 manifest (src/model_format.rs)
def _aligned(field_name: str, value: int):
    """validate_aligned (src/model_format.rs:543-548)."""
    if value & (ALIGN_2MB - 1):
        raise FormatError("Unaligned", field_name)


@dataclass
class Layer:
    layer_id: int
    flags: int
    dense_offset: int
    dense_disk_bytes: int
    dense_payload_bytes: int
    dense_dequant_bytes: int
    experts: list = field(default_factory=list)


@dataclass
class Manifest:
    header: dict
    layers: list
    base_dir: Path
    shards: dict  # (layer, expert) -> dict(path, disk_bytes, payload_bytes, checksum)
    pack_file: Optional[Path]
    pack: dict  # (layer, expert) -> (offset, disk_bytes, payload_bytes)


def _read_exact(f, offset: int, n: int) -> bytes:
    f.seek(offset)
    b = f.read(n)
    if len(b) != n:
        raise FormatError("Io", "failed to fill whole buffer")
    return b


def _with_extension(path: Path, ext: str) -> Path:
    """Rust Path::with_extension: replace the last extension (or add one)."""
    name = path.name
    stem = name[:name.rfind(".")] if "." in name[1:] else name
    return path.with_name(stem + "." + ext)


class _JsonObject(dict):
    """A JSON object that remembers which keys it saw more than once: serde
    rejects a struct field given twice, Python's json keeps the last."""
    dups: frozenset = frozenset()


def _pairs(pairs):
    d, seen, dups = _JsonObject(), set(), set()
    for k, v in pairs:
        if k in seen:
            dups.add(k)
        seen.add(k)
        d[k] = v
    d.dups = frozenset(dups)
    return d


def _no_dup(obj, key: str):
    if key in getattr(obj, "dups", ()):
        raise FormatError("ShardMap", f"duplicate field `{key}`")


def _json_u(obj: dict, key: str, bits: int, default=None):
    _no_dup(obj, key)
    if key not in obj:
        if default is None:
            raise FormatError("ShardMap", f"missing field `{key}`")
        return default
    v = obj[key]
    if isinstance(v, bool) or not isinstance(v, int) or v < 0 or v >= (1 << bits):
        raise FormatError("ShardMap", f"invalid value for `{key}`")
    return v


def _json_s(obj: dict, key: str, default=None):
    _no_dup(obj, key)
    if key not in obj:
        if default is None:
            raise FormatError("ShardMap", f"missing field `{key}`")
        return default
    v = obj[key]
    if not isinstance(v, str):
        raise FormatError("ShardMap", f"invalid type for `{key}`")
    return v


def _load_json(path: Path):
    try:
        return json.loads(path.read_text(encoding="utf-8"), object_pairs_hook=_pairs)
    except (ValueError, UnicodeDecodeError) as e:
        raise FormatError("ShardMap", str(e)) from None


def _load_shard_map(model_path: Path, base_dir: Path, layers: list, merge: bool) -> dict:
    """load_optional_shard_map (src/model_format.rs:339-436)."""
    shard_path = _with_extension(model_path, "shards.json")
    if not shard_path.exists():
        return {}
    disk = _load_json(shard_path)
    if not isinstance(disk, dict):
        raise FormatError("ShardMap", "shard map is not an object")
    fmt = _json_s(disk, "format", "")
    _no_dup(disk, "experts")
    experts = disk.get("experts", [])
    if not isinstance(experts, list):
        raise FormatError("ShardMap", "invalid type for `experts`")
    parsed = []
    for e in experts:
        if not isinstance(e, dict):
            raise FormatError("ShardMap", "invalid type for expert entry")
        parsed.append(dict(layer_id=_json_u(e, "layer_id", 32),
                           expert_id=_json_u(e, "expert_id", 32),
                           path=_json_s(e, "path"),
                           disk_bytes=_json_u(e, "disk_bytes", 64),
                           payload_bytes=_json_u(e, "payload_bytes", 64),
                           dequant_bytes=_json_u(e, "dequant_bytes", 64, 0),
                           quant_format=_json_u(e, "quant_format", 32, 0),
                           checksum=_json_u(e, "checksum", 64, 0)))
    if fmt not in ("wohper-sharded-experts", "zeroclaw-sharded-experts"):
        raise FormatError("ShardMap", "unsupported shard map format")
    known = {(x["layer_id"], x["expert_id"]) for L in layers for x in L.experts}
    out = {}
    merged = 0
    for e in parsed:
        key = (e["layer_id"], e["expert_id"])
        in_manifest = key in known
        if not in_manifest and not merge:
            continue
        _aligned("expert_shard.disk_bytes", e["disk_bytes"])
        if not in_manifest:
            target = next((L for L in layers
                           if L.flags & 0xFF == LAYER_BLOCK_COMPUTE and L.layer_id == key[0]), None)
            if target is None:
                continue
            tmpl = target.experts[0]["quant_format"] if target.experts else 0
            target.experts.append(dict(layer_id=key[0], expert_id=key[1], disk_offset=0,
                                       disk_bytes=e["disk_bytes"],
                                       payload_bytes=e["payload_bytes"],
                                       dequant_bytes=e["dequant_bytes"],
                                       quant_format=e["quant_format"] or tmpl,
                                       route_rank_hint=key[1], checksum=e["checksum"]))
            merged += 1
        out[key] = dict(path=base_dir / e["path"], disk_bytes=e["disk_bytes"],
                        payload_bytes=e["payload_bytes"], checksum=e["checksum"])
    if merged:
        for L in layers:
            L.experts.sort(key=lambda x: x["expert_id"])  # stable, like sort_by_key
    return out


def _load_pack(model_path: Path):
    """load_optional_expert_pack (src/model_format.rs:463-505)."""
    index_path = _with_extension(model_path, "experts_pack.index.json")
    if not index_path.exists():
        return None, {}
    disk = _load_json(index_path)
    if not isinstance(disk, dict):
        raise FormatError("ShardMap", "pack index is not an object")
    fmt = _json_s(disk, "format", "")
    pack_name = _json_s(disk, "pack_file", "")
    _no_dup(disk, "entries")
    entries = disk.get("entries", [])
    if not isinstance(entries, list):
        raise FormatError("ShardMap", "invalid type for `entries`")
    parsed = []
    for e in entries:
        if not isinstance(e, dict):
            raise FormatError("ShardMap", "invalid type for pack entry")
        parsed.append((_json_u(e, "layer_id", 32), _json_u(e, "expert_id", 32),
                       _json_u(e, "offset", 64), _json_u(e, "disk_bytes", 64),
                       _json_u(e, "payload_bytes", 64)))
    if fmt not in ("wohper-experts-pack", "zeroclaw-experts-pack"):
        raise FormatError("ShardMap", "unsupported experts pack format")
    pack_file = index_path.parent / pack_name
    if not pack_file.exists():
        raise FormatError("ShardMap", "experts pack file missing")
    out = {}
    for lid, eid, off, db, pb in parsed:
        _aligned("expert_pack.offset", off)
        _aligned("expert_pack.disk_bytes", db)
        out[(lid, eid)] = (off, db, pb)
    return pack_file, out


def load_manifest(path, merge_sidecar_experts: bool = False) -> Manifest:
    """ModelManifest::load (src/model_format.rs:193-263) with
    validate_header / validate_layer / validate_expert (:507-541)."""
    path = Path(path)
    try:
        f = open(path, "rb")
    except OSError as e:
        raise FormatError("Io", os.strerror(e.errno or 0)) from None
    with f:
        hv = ENGINE_HEADER.unpack(_read_exact(f, 0, ENGINE_HEADER.size))
        hdr = dict(zip(ENGINE_FIELDS, hv))
        if hdr["magic"] != MODEL_MAGIC:
            raise FormatError("InvalidMagic", "")
        if hdr["version"] != FORMAT_VERSION:
            raise FormatError("UnsupportedVersion", str(hdr["version"]))
        if hdr["block_alignment"] != ALIGN_2MB:
            raise FormatError("Unaligned", "block_alignment")
        for fld in ("manifest_offset", "tokenizer_offset", "router_metadata_offset"):
            _aligned(fld, hdr[fld])
        mh = MANIFEST_HEADER.unpack(_read_exact(f, hdr["manifest_offset"], MANIFEST_HEADER.size))
        layer_count, expert_count, _, _, ldo, edo, _ = mh
        if layer_count != hdr["num_layers"]:
            raise FormatError("LayerCountMismatch",
                              f"header={hdr['num_layers']}, manifest={layer_count}")
        lraw = _read_exact(f, hdr["manifest_offset"] + ldo, layer_count * LAYER_DESC.size)
        eraw = _read_exact(f, hdr["manifest_offset"] + edo, expert_count * EXPERT_DESC.size)
    experts = [dict(zip(EXPERT_FIELDS, EXPERT_DESC.unpack_from(eraw, i * EXPERT_DESC.size)))
               for i in range(expert_count)]
    layers = []
    for i in range(layer_count):
        d = dict(zip(LAYER_FIELDS, LAYER_DESC.unpack_from(lraw, i * LAYER_DESC.size)))
        _aligned("dense_offset", d["dense_offset"])
        _aligned("dense_disk_bytes", d["dense_disk_bytes"])
        start, end = d["first_expert_index"], d["first_expert_index"] + d["num_experts"]
        if end > len(experts):
            raise FormatError("InvalidExpertTable", str(d["layer_id"]))
        lst = []
        for e in experts[start:end]:
            if e["disk_offset"] == 0:
                _aligned("expert.disk_bytes", e["disk_bytes"])
            else:
                _aligned("expert.disk_offset", e["disk_offset"])
                _aligned("expert.disk_bytes", e["disk_bytes"])
            if e["layer_id"] != d["layer_id"]:
                raise FormatError("InvalidExpertTable", str(d["layer_id"]))
            lst.append(dict(e))
        layers.append(Layer(d["layer_id"], d["flags"], d["dense_offset"], d["dense_disk_bytes"],
                            d["dense_payload_bytes"], d["dense_dequant_bytes"], lst))
    base_dir = path.parent
    shards = _load_shard_map(path, base_dir, layers, merge_sidecar_experts)
    pack_file, pack = _load_pack(path)
    return Manifest(hdr, layers, base_dir, shards, pack_file, pack)


def expert_source(m: Manifest, model_path, layer_index: int, expert_id: int):
    """MoEIoScheduler::enqueue_expert_read (src/scheduler.rs:148-193): the pack
    entry if the pack has the expert, else the manifest's block, read from the
    expert's shard file when the shard map names one and from the model file
    otherwise.  Returns (path, offset, disk_bytes, payload_bytes)."""
    L = m.layers[layer_index]
    e = next((x for x in L.experts if x["expert_id"] == expert_id), None)
    if e is None:
        raise FormatError("InvalidExpert", f"layer={L.layer_id}, expert={expert_id}")
    key = (L.layer_id, expert_id)
    if key in m.pack:
        off, db, pb = m.pack[key]
        return m.pack_file, off, db, pb
    sh = m.shards.get(key)
    return (sh["path"] if sh else Path(model_path)), e["disk_offset"], e["disk_bytes"], \
        e["payload_bytes"]


def read_expert_block(m: Manifest, model_path, layer_index: int, expert_id: int) -> bytes:
    """The block bytes the reference hands parse_quant_block: payload_bytes at
    the resolved offset (src/scheduler.rs; src/direct_io.rs reads disk_bytes and
    the caller slices the payload)."""
    p, off, _db, pb = expert_source(m, model_path, layer_index, expert_id)
    with open(p, "rb") as f:
        return _read_exact(f, off, pb)
