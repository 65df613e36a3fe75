"""DS41PK01 expert packs: the reference's on-disk format for routed EXL3 experts.

Format (writer tools/pack_exl3.py:13-17,77-112,188-199; reader runtime/ds41/cache.py:40-43,150-158,
1788-1797, paths within the Findddx/eva project):
  bytes 0-7     magic b"DS41PK01"
  bytes 8-23    <IIII: version 1, n_layers, n_experts, slot size 128
  index         n_layers * n_experts slots of 128 bytes, layer-major, each
                <QIHH: record offset in the file, padded record bytes, K of w1, 1
                then for w1 (gate), w2 (down), w3 (up): <HHHHIIIiIII: in features, out features, K, 0,
                suh bytes, svh bytes, trellis bytes, mul1 (the codebook multiplier as int32), and the
                suh / svh / trellis offsets inside the record
  records       per expert: for w1, w2, w3 the suh fp16[in], svh fp16[out], trellis int16
                [in/16][out/16][16K], padded to 4096 bytes; the same bytes an ExpertLayer holds per
                expert (eva_b200.experts.record_layout)

The reference writer starts the records right after the index; this writer starts them at the next
4096-byte boundary (the index gives every record's offset, so readers are unaffected, and every
record is then 4096-aligned for O_DIRECT reads). The reference reader accepts only 384 experts per
layer (its N_EXPERTS, cache.py:42); the format itself has no such limit. tests/golden/
make_pack_pin.py runs the reference writer on seeded experts: its header, index fields (record
offsets aside) and record bytes equal this writer's.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np
import torch

from .config import MoEConfig
from .experts import ALIGN, PACK_ORDER, ExpertLayer, _pointer_tables, record_layout

MAGIC = b"DS41PK01"
VERSION = 1
SLOT = 128
SLOT_FMT = struct.Struct("<QIHH" + "HHHHIIIiIII" * 3)
MUL1_MULT = 0x83DCD12D                      # mul1 codebook multiplier (EXL3 format)
MUL1_FIELD = MUL1_MULT - (1 << 32)          # as the int32 the pack stores

assert SLOT_FMT.size <= SLOT


def _align(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def slot_fields(rec_off: int, cfg: MoEConfig) -> tuple:
    """The 4 + 3 x 11 index fields of one routed expert record of `cfg` stored at `rec_off`."""
    offs, padded, shapes = record_layout(cfg.hidden, cfg.inter, cfg.bits)
    fields = [rec_off, padded, cfg.bits, 1]
    for proj in PACK_ORDER:
        fin, fout = shapes[proj]
        fields += [fin, fout, cfg.bits, 0, offs[(proj, "suh")][1], offs[(proj, "svh")][1], offs[(proj, "trellis")][1],
                   MUL1_FIELD, offs[(proj, "suh")][0], offs[(proj, "svh")][0], offs[(proj, "trellis")][0]]
    return tuple(fields)


def write_pack(path: str, layers) -> None:
    """Write the routed experts of `layers` (whole layers, same shape) as one DS41PK01 file."""
    layers = list(layers)
    if not layers:
        raise ValueError("no layers")
    cfg = layers[0].cfg
    E = cfg.n_experts
    for lay in layers:
        if lay.cfg.hidden != cfg.hidden or lay.cfg.inter != cfg.inter or lay.cfg.bits != cfg.bits or lay.n_local != E:
            raise ValueError("every layer must hold all experts of one shape")
        if lay.cfg.hidden > 0xFFFF or lay.cfg.inter > 0xFFFF:
            raise ValueError("the slot format stores feature counts in 16 bits")
    rec = layers[0].record_bytes
    payload = _align(8 + 16 + len(layers) * E * SLOT)
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<IIII", VERSION, len(layers), E, SLOT))
        index = bytearray()
        for li in range(len(layers)):
            for e in range(E):
                fields = slot_fields(payload + (li * E + e) * rec, cfg)
                index += SLOT_FMT.pack(*fields).ljust(SLOT, b"\x00")
        f.write(index)
        f.write(b"\x00" * (payload - f.tell()))
        for lay in layers:
            f.write(lay.storage[: E * rec].cpu().numpy().tobytes())


@dataclass
class Pack:
    """An open DS41PK01 file: header and index (record bytes are read on demand)."""
    path: str
    n_layers: int
    n_experts: int
    slots: list

    @classmethod
    def open(cls, path: str) -> "Pack":
        with open(path, "rb") as f:
            head = f.read(24)
            if head[:8] != MAGIC:
                raise ValueError(f"bad pack magic {head[:8]!r}")
            version, n_layers, n_experts, slot = struct.unpack("<IIII", head[8:24])
            if version != VERSION or slot != SLOT:
                raise ValueError(f"unsupported pack version {version} / slot {slot}")
            raw = f.read(n_layers * n_experts * SLOT)
        slots = [SLOT_FMT.unpack_from(raw, i * SLOT) for i in range(n_layers * n_experts)]
        return cls(path, n_layers, n_experts, slots)

    def fields(self, layer: int, expert: int) -> tuple:
        return self.slots[layer * self.n_experts + expert]

    def record(self, layer: int, expert: int) -> bytes:
        f = self.fields(layer, expert)
        with open(self.path, "rb") as fh:
            return os.pread(fh.fileno(), f[1], f[0])

    def check_shape(self, cfg: MoEConfig) -> None:
        """Raise unless every slot describes a record of cfg's routed-expert shape."""
        _, padded, shapes = record_layout(cfg.hidden, cfg.inter, cfg.bits)
        for f in self.slots:
            if f[1] != padded or f[2] != cfg.bits:
                raise ValueError("pack records do not match the config")
            for pi, proj in enumerate(PACK_ORDER):
                fin, fout, k = f[4 + 11 * pi: 7 + 11 * pi]
                if (fin, fout, k) != (*shapes[proj], cfg.bits):
                    raise ValueError(f"pack {proj} shape does not match the config")


def load_layer(pack: Pack, layer: int, template: ExpertLayer, device="cpu", experts=None) -> ExpertLayer:
    """A layer whose routed records come from the pack and whose shared expert and router come from
    `template` (the pack holds routed experts only, as in the reference)."""
    cfg = template.cfg
    if pack.n_experts != cfg.n_experts:
        raise ValueError("pack expert count differs from the config")
    pack.check_shape(cfg)
    ids = tuple(range(cfg.n_experts)) if experts is None else tuple(int(e) for e in experts)
    rec = template.record_bytes
    shared = template.storage[template.n_local * rec:].cpu()
    storage = torch.empty(len(ids) * rec + shared.numel(), dtype=torch.uint8)
    with open(pack.path, "rb") as fh:
        for i, e in enumerate(ids):
            off, nb = pack.fields(layer, e)[:2]
            storage[i * rec:(i + 1) * rec] = torch.from_numpy(np.frombuffer(os.pread(fh.fileno(), nb, off), np.uint8).copy())
    storage[len(ids) * rec:] = shared
    storage = storage.to(device)
    packed, sh = _pointer_tables(cfg, storage, rec, len(ids))
    dev = storage.device
    return ExpertLayer(cfg, storage, rec, packed.to(dev), None if sh is None else sh.to(dev),
                       template.router_w.to(dev), template.router_b.to(dev), ids)
