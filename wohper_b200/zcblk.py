"""ZCBLK01 tensor blocks, ZCINF01 model files and the FP4 expert loader.

Reading goes through the C library (include/wohper_b200.h):

* :func:`parse_quant_block`, :func:`block_tensor`, :func:`find_tensor_by_suffix`
  and :func:`deepseek_v4_fp4_expert_from_quant_block` replace the reference's
  block parser and its DeepSeek FP4 suffix bridge (src/compute.rs:545-595,
  1099-1267), working on block bytes in host memory;
* :class:`ModelManifest` replaces ``ModelManifest::load`` with the shard map
  and experts pack index (src/model_format.rs:193-505);
* :class:`ExpertLoader` streams FP4 expert blocks from the model's files into
  one device arena (reader threads + pinned staging + copy engines) and hands
  back :class:`~wohper_b200.DeepSeekV4Fp4Expert` objects for ``MoeLayer``.

Writing is plain Python and produces the bytes the reference's converter
(tools/stream_convert_deepseek_v4.py) and pack builder
(tools/build_experts_pack.py) write for the same tensors: :func:`pack_block`,
:func:`deepseek_fp4_expert_tensors` and :func:`write_model`.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

from . import (Context, DeepSeekV4Fp4Expert, Fp4ExpertSpec, Fp4Matvec, _check, _stream, lib)

ALIGN_2MB = 2 * 1024 * 1024
MODEL_MAGIC = b"ZCINF01\0"
QUANT_BLOCK_MAGIC = b"ZCBLK01\0"
QUANT_DEEPSEEK_RAW_MIXED = 2400
QUANT_DEEPSEEK_FP8_E4M3 = 2401
QUANT_DEEPSEEK_FP4_E2M1_PACKED = 2402
QUANT_DEEPSEEK_UE8M0_SCALE = 2403
DTYPE_INT8 = 3          # the converter's code for I8 (packed E2M1 pairs)
DTYPE_F8_E8M0 = 102     # ... and for F8_E8M0 scales
ROLE_GATE_PROJ, ROLE_UP_PROJ, ROLE_DOWN_PROJ = 6, 7, 8
CHECKSUM_BLAKE2B64 = 1
SOURCE_MODEL, SOURCE_SHARD, SOURCE_PACK = 0, 1, 2

_ENGINE_HEADER = struct.Struct("<8sIIQQQQQQQIIIIIIIIIIQQ")
_MANIFEST_HEADER = struct.Struct("<IIIIQQQ")
_LAYER_DESC = struct.Struct("<IIQQQQIIIIIIQ")
_EXPERT_DESC = struct.Struct("<IIQQQQIIQ")
_BLOCK_HEADER = struct.Struct("<8sIIIIQQ")
_RECORD = struct.Struct("<HHIIQQQQff")


# --------------------------------------------------------------------------
# C structs
class BlockHeader(C.Structure):
    """wh_zcblk_header == QuantBlockHeader (src/compute.rs:431-438)."""
    _fields_ = [("tensor_count", C.c_uint32), ("quant_format", C.c_uint32),
                ("flags", C.c_uint32), ("reserved", C.c_uint32),
                ("record_table_offset", C.c_uint64), ("names_offset", C.c_uint64)]


class TensorRecord(C.Structure):
    """wh_zcblk_tensor: QuantTensorLayout (src/compute.rs:440-451) as positions."""
    _fields_ = [("dtype_original", C.c_uint16), ("quant_format", C.c_uint16),
                ("rank", C.c_uint32), ("flags", C.c_uint32), ("name_pos", C.c_uint64),
                ("name_len", C.c_uint64), ("shape_pos", C.c_uint64), ("data_pos", C.c_uint64),
                ("data_len", C.c_uint64), ("scale", C.c_float), ("zero_point", C.c_float),
                ("reserved", C.c_uint32)]

    @property
    def role(self) -> int:
        return self.flags & 0xFFFF


class Fp4View(C.Structure):
    _fields_ = [("weight_pos", C.c_uint64), ("weight_len", C.c_uint64),
                ("scale_pos", C.c_uint64), ("scale_len", C.c_uint64), ("rows", C.c_uint64),
                ("cols", C.c_uint64), ("scale_cols", C.c_uint64)]


class Fp4ExpertView(C.Structure):
    _fields_ = [("w1", Fp4View), ("w3", Fp4View), ("w2", Fp4View)]


class EngineHeader(C.Structure):
    """wh_engine_header == EngineHeader (src/model_format.rs:57-81)."""
    _fields_ = [("magic", C.c_uint8 * 8), ("version", C.c_uint32), ("endian", C.c_uint32),
                ("file_size", C.c_uint64), ("manifest_offset", C.c_uint64),
                ("manifest_size", C.c_uint64), ("tokenizer_offset", C.c_uint64),
                ("tokenizer_size", C.c_uint64), ("router_metadata_offset", C.c_uint64),
                ("router_metadata_size", C.c_uint64), ("model_family", C.c_uint32),
                ("architecture", C.c_uint32), ("num_layers", C.c_uint32),
                ("hidden_size", C.c_uint32), ("num_attention_heads", C.c_uint32),
                ("num_kv_heads", C.c_uint32), ("experts_per_layer", C.c_uint32),
                ("active_experts_per_token", C.c_uint32), ("block_alignment", C.c_uint32),
                ("disk_quant_format", C.c_uint32), ("manifest_checksum", C.c_uint64),
                ("file_checksum", C.c_uint64)]


class LayerDesc(C.Structure):
    """wh_model_layer == MoELayerBlockDesc without its expert list."""
    _fields_ = [("layer_id", C.c_uint32), ("flags", C.c_uint32), ("dense_offset", C.c_uint64),
                ("dense_disk_bytes", C.c_uint64), ("dense_payload_bytes", C.c_uint64),
                ("dense_dequant_bytes", C.c_uint64), ("num_experts", C.c_uint32),
                ("reserved", C.c_uint32)]


class ExpertDesc(C.Structure):
    """wh_model_expert == ExpertBlockDescDisk (src/model_format.rs:113-125)."""
    _fields_ = [("layer_id", C.c_uint32), ("expert_id", C.c_uint32), ("disk_offset", C.c_uint64),
                ("disk_bytes", C.c_uint64), ("payload_bytes", C.c_uint64),
                ("dequant_bytes", C.c_uint64), ("quant_format", C.c_uint32),
                ("route_rank_hint", C.c_uint32), ("checksum", C.c_uint64)]


class ExpertSource(C.Structure):
    _fields_ = [("path", C.c_char_p), ("offset", C.c_uint64), ("disk_bytes", C.c_uint64),
                ("payload_bytes", C.c_uint64), ("kind", C.c_int), ("reserved", C.c_int)]


def _buf(block):
    """(pointer, length, keep-alive) for bytes / bytearray / numpy uint8 arrays."""
    if isinstance(block, (bytes, bytearray)):
        b = (C.c_uint8 * len(block)).from_buffer_copy(block) if isinstance(block, bytes) \
            else (C.c_uint8 * len(block)).from_buffer(block)
        return C.cast(b, C.c_void_p), len(block), b
    import numpy as np

    a = np.ascontiguousarray(block, dtype=np.uint8)
    return C.c_void_p(a.ctypes.data), a.nbytes, a


# --------------------------------------------------------------------------
# Blocks
def parse_quant_block(block) -> BlockHeader:
    """parse_quant_block (src/compute.rs:1099-1147)."""
    p, n, _k = _buf(block)
    h = BlockHeader()
    _check(lib().wh_zcblk_parse(p, n, C.byref(h)))
    return h


def block_tensor(block, index: int) -> TensorRecord:
    """QuantBlockLayout::tensor (src/compute.rs:545-595)."""
    p, n, _k = _buf(block)
    t = TensorRecord()
    _check(lib().wh_zcblk_tensor_at(p, n, index, C.byref(t)))
    return t


def tensor_dims(block, t: TensorRecord) -> list:
    """ShapeLayout::dim for every axis (src/compute.rs:514-520)."""
    p, n, _k = _buf(block)
    out, v = [], C.c_uint64()
    for i in range(t.rank):
        _check(lib().wh_zcblk_tensor_dim(p, n, C.byref(t), i, C.byref(v)))
        out.append(int(v.value))
    return out


def find_tensor_by_suffix(block, suffix: str) -> TensorRecord:
    """find_tensor_by_suffix (src/compute.rs:1149-1169)."""
    p, n, _k = _buf(block)
    t = TensorRecord()
    _check(lib().wh_zcblk_find_suffix(p, n, suffix.encode(), C.byref(t)))
    return t


def deepseek_v4_fp4_expert_from_quant_block(block) -> Fp4ExpertView:
    """parse_quant_block + deepseek_v4_fp4_expert_from_quant_block
    (src/compute.rs:1199-1267): positions and shapes of w1, w3, w2."""
    p, n, _k = _buf(block)
    v = Fp4ExpertView()
    _check(lib().wh_zcblk_fp4_expert(p, n, C.byref(v)))
    return v


def fp4_expert_device_bytes(payload_bytes: int) -> int:
    return int(lib().wh_fp4_expert_device_bytes(payload_bytes))


def upload_fp4_expert(ctx: Context, block, dst=None, stream=None) -> DeepSeekV4Fp4Expert:
    """One FP4 expert block in host memory -> device tensors (wh_fp4_expert_upload).
    The returned expert's tensors are views of `dst` (allocated if None)."""
    import torch

    p, n, keep = _buf(block)
    if dst is None:
        dst = torch.empty(fp4_expert_device_bytes(n), dtype=torch.uint8,
                          device=f"cuda:{ctx.device}")
    s = stream if stream is not None else torch.cuda.current_stream(ctx.device)
    spec = Fp4ExpertSpec()
    _check(lib().wh_fp4_expert_upload(ctx.handle, p, n, dst.data_ptr(), dst.numel(),
                                      C.byref(spec), _stream(s)))
    s.synchronize()  # the copies read `block`
    del keep
    return _expert_from_spec(spec, dst)


def _expert_from_spec(spec: Fp4ExpertSpec, arena) -> DeepSeekV4Fp4Expert:
    base = arena.data_ptr()

    def mv(s):
        w0 = s.packed_weight - base
        s0 = s.ue8m0_scales - base
        return Fp4Matvec(arena[w0:w0 + s.packed_len], arena[s0:s0 + s.scales_len], int(s.rows),
                         int(s.cols), int(s.scale_cols))

    return DeepSeekV4Fp4Expert(mv(spec.w1), mv(spec.w3), mv(spec.w2))


# --------------------------------------------------------------------------
# Model manifest
class ModelManifest:
    """ModelManifest::load (src/model_format.rs:193-263): the ZCINF01 header,
    the layer and expert tables, MODEL.shards.json and
    MODEL.experts_pack.index.json."""

    def __init__(self, path, merge_sidecar_experts: bool = False):
        self.path = str(path)
        h = C.c_void_p()
        _check(lib().wh_model_open(self.path.encode(), int(bool(merge_sidecar_experts)),
                                   C.byref(h)))
        self.handle = h

    @property
    def header(self) -> EngineHeader:
        out = EngineHeader()
        _check(lib().wh_model_get_header(self.handle, C.byref(out)))
        return out

    def layer_count(self) -> int:
        return int(lib().wh_model_layer_count(self.handle))

    def layer(self, layer_index: int) -> LayerDesc:
        out = LayerDesc()
        _check(lib().wh_model_get_layer(self.handle, layer_index, C.byref(out)))
        return out

    def experts(self, layer_index: int) -> list:
        out = []
        for j in range(self.layer(layer_index).num_experts):
            e = ExpertDesc()
            _check(lib().wh_model_get_expert(self.handle, layer_index, j, C.byref(e)))
            out.append(e)
        return out

    def expert_source(self, layer_index: int, expert_id: int):
        """(path, offset, disk_bytes, payload_bytes, kind) as
        MoEIoScheduler::enqueue_expert_read resolves it (src/scheduler.rs:148-193)."""
        s = ExpertSource()
        _check(lib().wh_model_expert_source(self.handle, layer_index, expert_id, C.byref(s)))
        return (s.path.decode(), int(s.offset), int(s.disk_bytes), int(s.payload_bytes),
                int(s.kind))

    def read_expert_block(self, layer_index: int, expert_id: int) -> bytes:
        path, off, _db, pb, _k = self.expert_source(layer_index, expert_id)
        with open(path, "rb") as f:
            f.seek(off)
            return f.read(pb)

    def close(self):
        if getattr(self, "handle", None):
            lib().wh_model_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertLoader:
    """Streams a layer's FP4 expert blocks into one device arena.

    threads: reader threads (each with two pinned staging buffers); direct_io:
    O_DIRECT reads where the file system allows them."""

    def __init__(self, ctx: Context, manifest: ModelManifest, threads: int = 8,
                 direct_io: bool = False):
        self.ctx = ctx
        self.manifest = manifest
        h = C.c_void_p()
        _check(lib().wh_expert_loader_create(ctx.handle, manifest.handle, threads,
                                             int(bool(direct_io)), C.byref(h)))
        self.handle = h

    def arena_bytes(self, layer_index: int, expert_ids: Sequence[int]) -> int:
        ids = (C.c_uint32 * len(expert_ids))(*expert_ids)
        out = C.c_size_t()
        _check(lib().wh_expert_arena_bytes(self.manifest.handle, layer_index,
                                           C.cast(ids, C.c_void_p), len(expert_ids),
                                           C.byref(out)))
        return int(out.value)

    def load(self, layer_index: int, expert_ids: Sequence[int], arena=None, stream=None):
        """Returns (arena, [DeepSeekV4Fp4Expert per id]); work queued on `stream`
        (default: the current torch stream) after this call sees the weights."""
        import torch

        n = len(expert_ids)
        if arena is None:
            arena = torch.empty(max(self.arena_bytes(layer_index, expert_ids), 1),
                                dtype=torch.uint8, device=f"cuda:{self.ctx.device}")
        ids = (C.c_uint32 * max(n, 1))(*expert_ids)
        specs = (Fp4ExpertSpec * max(n, 1))()
        _check(lib().wh_expert_loader_load(self.handle, layer_index, C.cast(ids, C.c_void_p), n,
                                           arena.data_ptr(), arena.numel(), specs,
                                           _stream(stream)))
        return arena, [_expert_from_spec(specs[i], arena) for i in range(n)]

    def close(self):
        if getattr(self, "handle", None):
            lib().wh_expert_loader_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------
# Writing (the reference converter's layout, byte for byte)
@dataclass
class BlockTensor:
    name: str
    dtype_original: int
    quant_format: int
    role: int
    shape: tuple
    data: bytes
    scale: float = 1.0
    zero_point: float = 0.0


def checksum64(data: bytes) -> int:
    """The converter's block checksum: BLAKE2b with an 8-byte digest, little-endian."""
    return int.from_bytes(hashlib.blake2b(data, digest_size=8).digest(), "little")


def align_up(v: int, a: int = ALIGN_2MB) -> int:
    return (v + a - 1) // a * a


def pack_block(tensors: Sequence[BlockTensor],
               quant_format: int = QUANT_DEEPSEEK_RAW_MIXED) -> bytes:
    """A ZCBLK01 block: [header][records][names][data in order][shapes in order],
    the layout write_raw_block_payload writes (tools/stream_convert_deepseek_v4.py)."""
    n = len(tensors)
    names, name_offsets = bytearray(), []
    for t in tensors:
        raw = t.name.encode("utf-8")
        if len(raw) > 65535:
            raise ValueError(f"tensor name is too long: {t.name}")
        name_offsets.append(len(names))
        names += struct.pack("<H", len(raw)) + raw
    rto = _BLOCK_HEADER.size
    nmo = rto + n * _RECORD.size
    pos = nmo + len(names)
    data_offsets = []
    for t in tensors:
        data_offsets.append(pos)
        pos += len(t.data)
    shapes, shape_offsets = bytearray(), []
    for t in tensors:
        shape_offsets.append(pos + len(shapes))
        shapes += struct.pack("<I", len(t.shape)) + b"".join(struct.pack("<Q", d) for d in t.shape)
    out = bytearray(_BLOCK_HEADER.pack(QUANT_BLOCK_MAGIC, 1, n, quant_format, 0, rto, nmo))
    for t, no, do, so in zip(tensors, name_offsets, data_offsets, shape_offsets):
        out += _RECORD.pack(min(t.dtype_original, 65535), min(t.quant_format, 65535),
                            len(t.shape), t.role, no, so, do, len(t.data), t.scale, t.zero_point)
    out += names
    for t in tensors:
        out += t.data
    out += shapes
    return bytes(out)


def deepseek_fp4_expert_tensors(prefix: str, w1, s1, w3, s3, w2, s2) -> list:
    """The six tensors of a DeepSeek-V4 routed expert (`prefix` such as
    "layers.3.ffn.experts.17"), named, typed and ordered as the converter
    writes them: I8 packed E2M1 weights [rows, cols/2] and F8_E8M0 scales
    [rows, cols/32], sorted by name.  Arguments are 2-D uint8 arrays."""
    import numpy as np

    out = []
    for w, (wt, sc), role in (("w1", (w1, s1), ROLE_GATE_PROJ), ("w2", (w2, s2), ROLE_DOWN_PROJ),
                              ("w3", (w3, s3), ROLE_UP_PROJ)):
        sc = np.ascontiguousarray(sc, dtype=np.uint8)
        wt = np.ascontiguousarray(wt, dtype=np.uint8)
        out.append(BlockTensor(f"{prefix}.{w}.scale", DTYPE_F8_E8M0, QUANT_DEEPSEEK_UE8M0_SCALE,
                               role, tuple(sc.shape), sc.tobytes()))
        out.append(BlockTensor(f"{prefix}.{w}.weight", DTYPE_INT8, QUANT_DEEPSEEK_FP4_E2M1_PACKED,
                               role, tuple(wt.shape), wt.tobytes()))
    return out


def _with_extension(path: Path, ext: str) -> Path:
    name = path.name
    stem = name[:name.rfind(".")] if "." in name[1:] else name
    return path.with_name(stem + "." + ext)


@dataclass
class LayerSpec:
    layer_id: int
    dense: Sequence[BlockTensor]
    experts: dict  # expert_id -> [BlockTensor]


def write_model(out_path, layers: Sequence[LayerSpec], *, hidden_size: int,
                global_tensors: Optional[Sequence[BlockTensor]] = None,
                num_attention_heads: int = 0, num_kv_heads: int = 0,
                active_experts_per_token: int = 6, experts_dir: Optional[Path] = None,
                pack: bool = False) -> dict:
    """Write a ZCINF01 model as the reference's DeepSeek converter does
    (execute_conversion, tools/stream_convert_deepseek_v4.py): the model file
    with the optional global auxiliary block and one dense block per layer,
    one ZCBLK01 shard per expert under `experts_dir` and MODEL.shards.json.
    pack=True writes the experts into MODEL.experts_pack.bin with
    MODEL.experts_pack.index.json instead of shard files, which is what
    tools/build_experts_pack.py leaves behind.  Returns the layer and expert
    plans."""
    out_path = Path(out_path)
    experts_dir = Path(experts_dir) if experts_dir else out_path.parent / "experts"
    out_path.parent.mkdir(parents=True, exist_ok=True)
    n_layers = len(layers) + (1 if global_tensors else 0)
    n_experts = sum(len(L.experts) for L in layers)
    manifest_size = _MANIFEST_HEADER.size + n_layers * _LAYER_DESC.size + \
        n_experts * _EXPERT_DESC.size
    layer_plans, expert_plans, shard_plans = [], [], []
    pack_path = _with_extension(out_path, "experts_pack.bin")
    pack_entries = []
    pack_f = open(pack_path, "wb") if pack else None

    def aligned_block(f, payload: bytes):
        off = align_up(f.tell())
        f.write(b"\0" * (off - f.tell()))
        f.write(payload)
        disk = align_up(len(payload))
        f.write(b"\0" * (disk - len(payload)))
        return off, disk

    try:
        with open(out_path, "wb") as f:
            f.write(b"\0" * _ENGINE_HEADER.size)
            manifest_offset = align_up(f.tell())
            f.write(b"\0" * (manifest_offset - f.tell()))
            f.write(b"\0" * manifest_size)
            if global_tensors:
                payload = pack_block(global_tensors)
                off, disk = aligned_block(f, payload)
                layer_plans.append(dict(layer_id=0, dense_offset=off, dense_disk_bytes=disk,
                                        dense_payload_bytes=len(payload),
                                        dense_dequant_bytes=sum(len(t.data) for t in global_tensors),
                                        first_expert_index=0, num_experts=0,
                                        checksum=checksum64(payload), block_type=1))
            for L in layers:
                payload = pack_block(L.dense)
                off, disk = aligned_block(f, payload)
                first = len(expert_plans)
                for eid in sorted(L.experts):
                    ts = L.experts[eid]
                    blk = pack_block(ts)
                    disk_e = align_up(len(blk))
                    name = f"layer{L.layer_id}_expert{eid}.zcblk"
                    if pack_f is not None:
                        pack_entries.append(dict(layer_id=L.layer_id, expert_id=eid,
                                                 offset=pack_f.tell(), disk_bytes=disk_e,
                                                 payload_bytes=len(blk)))
                        pack_f.write(blk)
                        pack_f.write(b"\0" * (disk_e - len(blk)))
                    else:
                        experts_dir.mkdir(parents=True, exist_ok=True)
                        with open(experts_dir / name, "wb") as g:
                            g.write(blk)
                            g.write(b"\0" * (disk_e - len(blk)))
                    dq = sum(len(t.data) for t in ts)
                    ck = checksum64(blk)
                    expert_plans.append(dict(layer_id=L.layer_id, expert_id=eid, disk_offset=0,
                                             disk_bytes=disk_e, payload_bytes=len(blk),
                                             dequant_bytes=dq,
                                             quant_format=QUANT_DEEPSEEK_RAW_MIXED,
                                             route_rank_hint=eid, checksum=ck))
                    try:
                        rel = (experts_dir / name).relative_to(out_path.parent)
                    except ValueError:
                        rel = experts_dir / name
                    shard_plans.append(dict(layer_id=L.layer_id, expert_id=eid,
                                            path=str(rel).replace("\\", "/"), disk_bytes=disk_e,
                                            payload_bytes=len(blk), dequant_bytes=dq,
                                            quant_format=QUANT_DEEPSEEK_RAW_MIXED, checksum=ck))
                layer_plans.append(dict(layer_id=L.layer_id, dense_offset=off,
                                        dense_disk_bytes=disk,
                                        dense_payload_bytes=len(payload),
                                        dense_dequant_bytes=sum(len(t.data) for t in L.dense),
                                        first_expert_index=first, num_experts=len(L.experts),
                                        checksum=checksum64(payload), block_type=0))
            file_size = f.tell()
            manifest = bytearray(_MANIFEST_HEADER.pack(
                len(layer_plans), len(expert_plans), 0, 0, _MANIFEST_HEADER.size,
                _MANIFEST_HEADER.size + len(layer_plans) * _LAYER_DESC.size,
                _MANIFEST_HEADER.size + len(layer_plans) * _LAYER_DESC.size +
                len(expert_plans) * _EXPERT_DESC.size))
            for p in layer_plans:
                manifest += _LAYER_DESC.pack(p["layer_id"], p["block_type"], p["dense_offset"],
                                             p["dense_disk_bytes"], p["dense_payload_bytes"],
                                             p["dense_dequant_bytes"], 0, 0,
                                             p["first_expert_index"], p["num_experts"],
                                             QUANT_DEEPSEEK_RAW_MIXED, CHECKSUM_BLAKE2B64,
                                             p["checksum"])
            for e in expert_plans:
                manifest += _EXPERT_DESC.pack(e["layer_id"], e["expert_id"], e["disk_offset"],
                                              e["disk_bytes"], e["payload_bytes"],
                                              e["dequant_bytes"], e["quant_format"],
                                              e["route_rank_hint"], e["checksum"])
            header = _ENGINE_HEADER.pack(
                MODEL_MAGIC, 1, 0, file_size, manifest_offset, len(manifest), 0, 0, 0, 0, 2, 2,
                len(layer_plans), hidden_size, num_attention_heads, num_kv_heads,
                max((len(L.experts) for L in layers), default=0), active_experts_per_token,
                ALIGN_2MB, QUANT_DEEPSEEK_RAW_MIXED, checksum64(bytes(manifest)), 0)
            f.seek(0)
            f.write(header)
            f.seek(manifest_offset)
            f.write(manifest)
    finally:
        if pack_f is not None:
            pack_f.close()
    shard_map = {"format": "wohper-sharded-experts", "version": 1, "core_file": str(out_path),
                 "experts_dir": str(experts_dir),
                 "layers_in_core": [L.layer_id for L in layers],
                 "alignment": ALIGN_2MB, "quant_format": QUANT_DEEPSEEK_RAW_MIXED,
                 "dense_layers": layer_plans, "experts": shard_plans}
    _with_extension(out_path, "shards.json").write_text(json.dumps(shard_map, indent=2))
    if pack:
        index = {"format": "wohper-experts-pack", "version": 1, "pack_file": pack_path.name,
                 "entries": pack_entries}
        _with_extension(out_path, "experts_pack.index.json").write_text(json.dumps(index))
    return {"layers": layer_plans, "experts": expert_plans}


def build_experts_pack(model_path, keep_shards: bool = False) -> Path:
    """Consolidate the shard files named by MODEL.shards.json into
    MODEL.experts_pack.bin + MODEL.experts_pack.index.json, in shard-map order,
    as tools/build_experts_pack.py does."""
    model_path = Path(model_path)
    base = model_path.parent
    shards = json.loads(_with_extension(model_path, "shards.json").read_text())
    pack_path = _with_extension(model_path, "experts_pack.bin")
    entries, off = [], 0
    with open(pack_path, "wb") as out:
        for e in shards["experts"]:
            data = (base / e["path"]).read_bytes()
            if len(data) != e["disk_bytes"]:
                raise RuntimeError(f"size mismatch {e['path']}: {len(data)} != {e['disk_bytes']}")
            out.write(data)
            entries.append(dict(layer_id=e["layer_id"], expert_id=e["expert_id"], offset=off,
                                disk_bytes=e["disk_bytes"], payload_bytes=e["payload_bytes"]))
            off += len(data)
    if not keep_shards:
        for e in shards["experts"]:
            os.remove(base / e["path"])
    _with_extension(model_path, "experts_pack.index.json").write_text(json.dumps(
        {"format": "wohper-experts-pack", "version": 1, "pack_file": pack_path.name,
         "entries": entries}))
    return pack_path
