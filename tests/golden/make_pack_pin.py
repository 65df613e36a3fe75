"""Pin the DS41PK01 pack layout against the reference's own packer (tools/pack_exl3.py).

Builds two small seeded layers (6 routed experts, hidden 256, inter 128, EXL3 K3), writes their
routed experts as a synthetic safetensors checkpoint with the tensor names the reference packer
parses (layers.L.ffn.experts.E.{w1,w2,w3}.{suh,svh,trellis,mul1}; tools/pack_exl3.py:30-46), runs the
reference packer on it unmodified except for its layer / expert counts (module constants N_LAYERS,
N_EXPERTS; the packer itself is fixed to 40 x 384) and records what it wrote: the header, every
index slot and the SHA-256 of every record's padded bytes. tests/test_pack.py rebuilds the same
layers and checks eva_b200.pack.write_pack against that record: same header, the same index fields
apart from the record offset (the reference packs records right after the index, this writer at the
next 4096-byte boundary), the same record bytes.

Needs a checkout of the reference (first argument or EVA_REFERENCE). The fixture is small and
committed; the tests never read the reference.

Usage: python tests/golden/make_pack_pin.py [/path/to/reference]
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import struct
import sys
import tempfile
from pathlib import Path

OUT = Path(__file__).resolve().parent
ROOT = OUT.parent.parent

CFG = dict(name="pack-pin", hidden=256, inter=128, n_experts=6, topk=2, router="softmax", bits=3)
SEEDS = (1, 2)
MUL1 = 0x83DCD12D - (1 << 32)          # the codebook multiplier as the int32 a checkpoint stores
PROJ_OF = {"w1": "gate", "w2": "down", "w3": "up"}


def pin_layers():
    sys.path.insert(0, str(ROOT))
    from eva_b200.config import MoEConfig
    from eva_b200.experts import make_layer
    cfg = MoEConfig(**CFG)
    return cfg, [make_layer(cfg, "cpu", seed=s) for s in SEEDS]


def write_checkpoint(d: Path, cfg, layers) -> None:
    """One safetensors shard + model.safetensors.index.json holding the layers' routed experts."""
    from eva_b200.experts import record_layout
    offs, _, shapes = record_layout(cfg.hidden, cfg.inter, cfg.bits)
    header, blobs, pos = {}, [], 0
    for li, lay in enumerate(layers):
        raw = lay.storage.numpy().tobytes()
        for e in range(cfg.n_experts):
            base = e * lay.record_bytes
            for w, proj in PROJ_OF.items():
                fin, fout = shapes[proj]
                items = [("suh", "F16", [fin]), ("svh", "F16", [fout]),
                         ("trellis", "I16", [fin // 16, fout // 16, 16 * cfg.bits])]
                for kind, dtype, shape in items:
                    o, nb = offs[(proj, kind)]
                    blobs.append(raw[base + o: base + o + nb])
                    header[f"layers.{li}.ffn.experts.{e}.{w}.{kind}"] = {
                        "dtype": dtype, "shape": shape, "data_offsets": [pos, pos + nb]}
                    pos += nb
                blobs.append(struct.pack("<i", MUL1))
                header[f"layers.{li}.ffn.experts.{e}.{w}.mul1"] = {"dtype": "I32", "shape": [],
                                                                   "data_offsets": [pos, pos + 4]}
                pos += 4
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(d / "shard.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    json.dump({"weight_map": {name: "shard.safetensors" for name in header}},
              open(d / "model.safetensors.index.json", "w"))


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EVA_REFERENCE")
    if not ref:
        sys.exit("pass the reference checkout's root as the first argument or set EVA_REFERENCE")
    ref = Path(ref)
    cfg, layers = pin_layers()
    with tempfile.TemporaryDirectory() as tmp:
        ckpt, out = Path(tmp) / "ckpt", Path(tmp) / "pack"
        ckpt.mkdir()
        write_checkpoint(ckpt, cfg, layers)
        spec = importlib.util.spec_from_file_location("ref_pack_exl3", ref / "tools" / "pack_exl3.py")
        packer = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(packer)
        packer.BASE, packer.OUT_DIR = str(ckpt), str(out)
        packer.N_LAYERS, packer.N_EXPERTS = len(layers), cfg.n_experts
        packer.main()
        raw = (out / "experts.bin").read_bytes()
    slot = struct.Struct("<QIHH" + "HHHHIIIiIII" * 3)
    n = len(layers) * cfg.n_experts
    slots = [list(slot.unpack_from(raw, 24 + i * 128)) for i in range(n)]
    pin = {
        "config": CFG, "seeds": list(SEEDS),
        "header": list(struct.unpack("<IIII", raw[8:24])), "magic": raw[:8].decode(),
        "slots": slots,
        "record_sha256": [hashlib.sha256(raw[s[0]: s[0] + s[1]]).hexdigest() for s in slots],
        "file_bytes": len(raw),
    }
    (OUT / "pack_ref_pin.json").write_text(json.dumps(pin, indent=1) + "\n")
    print(f"wrote pack_ref_pin.json ({n} records, reference pack of {len(raw)} bytes)")


if __name__ == "__main__":
    main()
