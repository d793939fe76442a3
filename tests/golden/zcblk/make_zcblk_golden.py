#!/usr/bin/env python3
"""Generate tests/golden/zcblk/ from the reference's own format writers.

Run in the build container, where the read-only reference checkout exists:

    python tests/golden/zcblk/make_zcblk_golden.py [--reference /path/to/reference]

Steps:
1. Write a tiny synthetic DeepSeek-V4-style checkpoint (two safetensors shards,
   their index and a config.json): two layers of four routed FP4 experts
   (I8-packed E2M1 + F8_E8M0 scales, hidden 64, intermediate 32), per-layer
   router gate / bias / tid2eid table, an FP8 shared expert and norms, plus
   global embed / norm / head tensors.  Seeded random bytes.
2. Convert it with the reference converter's functions
   (tools/stream_convert_deepseek_v4.py: build_tensor_items, group_items,
   plan_payload, execute_conversion), which write the ZCINF01 model file,
   one ZCBLK01 shard per expert and the shard map.
3. Consolidate the shards into an experts pack with the reference's
   tools/build_experts_pack.py, which writes the pack and its index and
   deletes the shard files (each is a byte-identical slice of the pack; the
   tests cut them back out to exercise the shard-file path).
4. Store the output tree as deepseek_tiny.tar.gz (sorted members, zero
   mtimes) and, in expected.json, what the reference's converter assigned to
   every tensor (dtype code, quant format, role code, shape, block) with the
   sha256 of its source bytes.
"""
from __future__ import annotations

import argparse
import hashlib
import io
import json
import struct
import subprocess
import sys
import tarfile
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
HIDDEN, INTER, EXPERTS, LAYERS, VOCAB, TOPK = 64, 32, 4, 2, 16, 2


def tensors(rng):
    """name -> (safetensors dtype, shape, bytes)."""
    out = {}

    def put(name, dtype, shape, data):
        out[name] = (dtype, list(shape), bytes(data))

    def scales(shape):
        return rng.integers(118, 132, size=shape, dtype=np.uint8).tobytes()

    for L in range(LAYERS):
        for e in range(EXPERTS):
            p = f"layers.{L}.ffn.experts.{e}"
            for w, (r, c) in (("w1", (INTER, HIDDEN)), ("w3", (INTER, HIDDEN)),
                              ("w2", (HIDDEN, INTER))):
                put(f"{p}.{w}.weight", "I8", (r, c // 2),
                    rng.integers(0, 256, size=r * c // 2, dtype=np.uint8))
                put(f"{p}.{w}.scale", "F8_E8M0", (r, c // 32), scales((r, c // 32)))
        g = f"layers.{L}.ffn"
        put(f"{g}.gate.weight", "BF16", (EXPERTS, HIDDEN),
            rng.integers(0, 1 << 16, size=EXPERTS * HIDDEN, dtype=np.uint16).tobytes())
        put(f"{g}.gate.bias", "F32", (EXPERTS,),
            rng.standard_normal(EXPERTS).astype(np.float32).tobytes())
        if L == 0:
            put(f"{g}.gate.tid2eid", "I64", (VOCAB, TOPK),
                rng.integers(0, EXPERTS, size=VOCAB * TOPK, dtype=np.int64).tobytes())
        for w, (r, c) in (("w1", (INTER, HIDDEN)), ("w3", (INTER, HIDDEN)),
                          ("w2", (HIDDEN, INTER))):
            put(f"{g}.shared_experts.{w}.weight", "F8_E4M3", (r, c),
                rng.integers(0, 256, size=r * c, dtype=np.uint8))
            put(f"{g}.shared_experts.{w}.scale", "F8_E8M0", (1, 1), scales((1, 1)))
        put(f"layers.{L}.ffn_norm.weight", "BF16", (HIDDEN,),
            rng.integers(0, 1 << 16, size=HIDDEN, dtype=np.uint16).tobytes())
    put("embed.weight", "BF16", (VOCAB, HIDDEN),
        rng.integers(0, 1 << 16, size=VOCAB * HIDDEN, dtype=np.uint16).tobytes())
    put("norm.weight", "BF16", (HIDDEN,),
        rng.integers(0, 1 << 16, size=HIDDEN, dtype=np.uint16).tobytes())
    put("head.weight", "BF16", (VOCAB, HIDDEN),
        rng.integers(0, 1 << 16, size=VOCAB * HIDDEN, dtype=np.uint16).tobytes())
    return out


def write_safetensors(path: Path, items: dict):
    header, blobs, off = {}, [], 0
    for name in sorted(items):
        dtype, shape, data = items[name]
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)
    path.write_bytes(struct.pack("<Q", len(raw)) + raw + b"".join(blobs))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the reference checkout (the Wohper repository root)")
    args = ap.parse_args()
    tools = Path(args.reference) / "tools"
    sys.path.insert(0, str(tools))
    import stream_convert_deepseek_v4 as sc  # the reference converter

    items = tensors(np.random.default_rng(20261202))
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        ckpt = tmp / "ckpt"
        ckpt.mkdir()
        shard_of = {n: ("model-00001-of-00002.safetensors"
                        if not n.startswith("layers.1.") else "model-00002-of-00002.safetensors")
                    for n in items}
        for shard in sorted(set(shard_of.values())):
            write_safetensors(ckpt / shard, {n: v for n, v in items.items() if shard_of[n] == shard})
        (ckpt / "model.safetensors.index.json").write_text(json.dumps({"weight_map": shard_of}))
        config = {"hidden_size": HIDDEN, "num_attention_heads": 2, "num_key_value_heads": 1,
                  "num_hidden_layers": LAYERS, "num_experts_per_tok": TOPK}
        (ckpt / "config.json").write_text(json.dumps(config))

        out = tmp / "out"
        ti = sc.build_tensor_items(ckpt)
        dense, experts, glob = sc.group_items(ti, list(range(LAYERS)), None, "all")
        est = sc.plan_payload(dense, experts, glob)
        ns = argparse.Namespace(out=out / "dense_core.bin", experts_dir=None, shard_index_out=None,
                                progress=tmp / "progress.json", model_dir=ckpt, chunk_mb=8)
        sc.execute_conversion(ns, config, dense, experts, glob, est)
        subprocess.run([sys.executable, str(tools / "build_experts_pack.py"), "--base", str(out)],
                       check=True, stdout=subprocess.DEVNULL)

        # expected: what the converter assigned to each tensor, block by block
        blocks = {"global_aux": [it.name for it in glob]}
        for L, refs in dense.items():
            blocks[f"dense_layer_{L}"] = [it.name for it in refs]
        for L, by_e in experts.items():
            for e, refs in sorted(by_e.items()):
                blocks[f"layer{L}_expert{e}"] = [it.name for it in refs]
        expected = {
            "hidden": HIDDEN, "inter": INTER, "experts_per_layer": EXPERTS, "layers": LAYERS,
            "blocks": blocks,
            "tensors": {it.name: {"dtype_original": sc.dtype_code(it),
                                  "quant_format": sc.tensor_quant_format(it),
                                  "role": sc.tensor_role_code(it), "shape": list(it.shape),
                                  "sha256": hashlib.sha256(items[it.name][2]).hexdigest()}
                        for it in ti.values()},
        }
        (HERE / "expected.json").write_text(json.dumps(expected, indent=1, sort_keys=True) + "\n")

        buf = io.BytesIO()
        with tarfile.open(fileobj=buf, mode="w:gz", compresslevel=9) as tar:
            for p in sorted(out.rglob("*")):
                if p.is_file():
                    info = tar.gettarinfo(str(p), arcname=str(p.relative_to(out)))
                    info.mtime, info.uid, info.gid, info.uname, info.gname = 0, 0, 0, "", ""
                    with p.open("rb") as fh:
                        tar.addfile(info, fh)
        (HERE / "deepseek_tiny.tar.gz").write_bytes(buf.getvalue())
        print(f"wrote {HERE / 'deepseek_tiny.tar.gz'} ({len(buf.getvalue())} bytes)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
