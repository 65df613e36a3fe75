"""EXL3 expert records and the pointer-table handles the MoE kernels read.

Record layout follows eva's DS41PK01 expert pack: per expert one record, projections in the
order w1 (gate), w2 (down), w3 (up), each stored as suh, svh, trellis, the record padded to
4096 bytes (tools/pack_exl3.py:77-112; read back by runtime/ds41/cache.py:1788-1797).

The handle is the reference's pointer table: int64 [9, E] of device addresses in the row order
[gate.trellis, gate.suh, gate.svh, up.trellis, up.suh, up.svh, down.trellis, down.suh, down.svh]
(runtime/ds41/cache.py:1864-1887), zero meaning unbound.

Tensors: trellis int16 [in/16, out/16, 16*K]; suh fp16 [in]; svh fp16 [out].

No EXL3 quantizer exists in the reference (tools/pack_exl3.py only repacks), so synthetic experts
use uniformly random trellis codes (every 16-bit state decodes to a valid codebook value with
about unit variance), suh = +-1 and svh = +-scale with a small magnitude jitter, which makes the
effective weight entries roughly N(0, scale^2).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .config import MoEConfig

ALIGN = 4096
PTR_ROWS = 9
# row index of each tensor in the pointer table
ROW = {("gate", "trellis"): 0, ("gate", "suh"): 1, ("gate", "svh"): 2,
       ("up", "trellis"): 3, ("up", "suh"): 4, ("up", "svh"): 5,
       ("down", "trellis"): 6, ("down", "suh"): 7, ("down", "svh"): 8}
PACK_ORDER = ("gate", "down", "up")   # w1, w2, w3


def _align(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def record_layout(hidden: int, inter: int, bits: int):
    """Byte offsets of every tensor inside one expert record, and the padded record size."""
    shapes = {"gate": (hidden, inter), "down": (inter, hidden), "up": (hidden, inter)}
    offs = {}
    rel = 0
    for proj in PACK_ORDER:
        fin, fout = shapes[proj]
        offs[(proj, "suh")] = (rel, fin * 2)
        rel += fin * 2
        offs[(proj, "svh")] = (rel, fout * 2)
        rel += fout * 2
        tb = fin * fout * bits // 8
        offs[(proj, "trellis")] = (rel, tb)
        rel += tb
    return offs, _align(rel), shapes


@dataclass
class ExpertLayer:
    """One layer's experts resident in a single uint8 allocation, plus routing parameters."""
    cfg: MoEConfig
    storage: torch.Tensor          # uint8, routed records then the shared record
    record_bytes: int
    packed: torch.Tensor           # int64 [9, E] device addresses (reference handle format)
    shared: torch.Tensor | None    # int64 [9] addresses of the shared expert
    router_w: torch.Tensor         # float32 [E, H]
    router_b: torch.Tensor         # float32 [E] (e_score_correction_bias / gate bias)
    experts: tuple = ()            # global ids of the routed records held, in table order

    @property
    def device(self):
        return self.storage.device

    @property
    def n_local(self) -> int:
        """Routed experts held (columns of `packed`); equals cfg.n_experts for a whole layer."""
        return len(self.experts)

    def tensor(self, expert: int, proj: str, kind: str) -> torch.Tensor:
        """View of one tensor of a routed expert (expert == -1: the shared expert)."""
        cfg = self.cfg
        if expert < 0:
            offs, _, shapes = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
            base = self.n_local * self.record_bytes
            bits = cfg.shared_bits
        else:
            offs, _, shapes = record_layout(cfg.hidden, cfg.inter, cfg.bits)
            base = expert * self.record_bytes
            bits = cfg.bits
        off, nb = offs[(proj, kind)]
        raw = self.storage[base + off: base + off + nb]
        fin, fout = shapes[proj]
        if kind == "trellis":
            return raw.view(torch.int16).view(fin // 16, fout // 16, 16 * bits)
        return raw.view(torch.float16)

    def host_copy(self, pinned: bool = False) -> "ExpertLayer":
        """Same experts in host memory (pointer tables re-based): for the CPU oracle, or page-locked
        (pinned=True) as the host side of an expert cache."""
        if pinned:
            storage = torch.empty(self.storage.numel(), dtype=torch.uint8, pin_memory=True)
            storage.copy_(self.storage)
        else:
            storage = self.storage.cpu()
        return _with_storage(self, storage)

    def to(self, device) -> "ExpertLayer":
        return _with_storage(self, self.storage.to(device), device)


def _pointer_tables(cfg: MoEConfig, storage: torch.Tensor, record_bytes: int, n_local: int):
    base = storage.data_ptr()
    offs, _, _ = record_layout(cfg.hidden, cfg.inter, cfg.bits)
    packed = torch.zeros(PTR_ROWS, n_local, dtype=torch.int64)
    for (proj, kind), row in ROW.items():
        off = offs[(proj, kind)][0]
        packed[row] = base + off + torch.arange(n_local, dtype=torch.int64) * record_bytes
    shared = None
    if cfg.shared_inter:
        soffs, _, _ = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
        sbase = base + n_local * record_bytes
        shared = torch.zeros(PTR_ROWS, dtype=torch.int64)
        for (proj, kind), row in ROW.items():
            shared[row] = sbase + soffs[(proj, kind)][0]
    return packed, shared


def _with_storage(layer: ExpertLayer, storage: torch.Tensor, device=None) -> ExpertLayer:
    packed, shared = _pointer_tables(layer.cfg, storage, layer.record_bytes, layer.n_local)
    dev = storage.device
    return ExpertLayer(layer.cfg, storage, layer.record_bytes, packed.to(dev),
                       None if shared is None else shared.to(dev),
                       layer.router_w.to(dev), layer.router_b.to(dev), layer.experts)


def _fill_record(storage, base, offs, shapes, gen, scale, device):
    for proj in PACK_ORDER:
        fin, fout = shapes[proj]
        off, nb = offs[(proj, "trellis")]
        n16 = nb // 2
        codes = torch.randint(-32768, 32768, (n16,), dtype=torch.int32, generator=gen, device=device)
        storage[base + off: base + off + nb].view(torch.int16).copy_(codes.to(torch.int16))
        for kind, n, mag in (("suh", fin, 1.0), ("svh", fout, scale)):
            o, b = offs[(proj, kind)]
            sign = torch.randint(0, 2, (n,), generator=gen, device=device).to(torch.float32) * 2 - 1
            jit = torch.rand((n,), generator=gen, device=device) * 0.5 + 0.75
            storage[base + o: base + o + b].view(torch.float16).copy_((sign * jit * mag).to(torch.float16))


def _record_seed(seed: int, index: int) -> int:
    return (seed * 1_000_003 + index + 1) & 0x7FFF_FFFF_FFFF_FFFF


def make_router(cfg: MoEConfig, device="cpu", seed: int = 0, router_scale: float = 0.02, bias_std: float | None = None):
    """The synthetic layer's router: FP32 weights [E, H] from `seed`, bias [E] from `seed + 2`."""
    rgen = torch.Generator(device="cpu")
    rgen.manual_seed(seed)
    router_w = (torch.randn(cfg.n_experts, cfg.hidden, generator=rgen) * router_scale).to(device)
    bgen = torch.Generator(device="cpu")
    bgen.manual_seed(seed + 2)
    if bias_std is None:
        bias_std = 0.01 if cfg.router != "softmax" else 0.0
    router_b = (torch.randn(cfg.n_experts, generator=bgen) * bias_std).to(device)
    return router_w, router_b


def make_layer(cfg: MoEConfig, device="cpu", seed: int = 0, svh_scale: float = 0.02,
               router_scale: float = 0.02, bias_std: float | None = None,
               n_fill: int | None = None, experts=None) -> ExpertLayer:
    """Synthetic layer: seeded EXL3 experts (+ shared expert), FP32 router weights and bias.

    Seeds: routed expert e from (seed, e), the shared expert from (seed, n_experts), router weights
    from `seed`, router bias from `seed + 2`. Each record has its own seed stream, so a layer built
    for a subset of experts (one expert-parallel rank) holds exactly the bytes of the whole layer.
    experts: global ids of the routed experts to hold, in table order (default: all).
    n_fill: fill only the first n_fill held experts with random data (the rest stay zero, a valid
    all-zero-state code); used to build multi-GB layers quickly.
    """
    device = torch.device(device)
    ids = tuple(range(cfg.n_experts)) if experts is None else tuple(int(e) for e in experts)
    if any(not 0 <= e < cfg.n_experts for e in ids) or len(set(ids)) != len(ids):
        raise ValueError("experts must be distinct ids in [0, n_experts)")
    _, rec, _ = record_layout(cfg.hidden, cfg.inter, cfg.bits)
    total = len(ids) * rec
    if cfg.shared_inter:
        _, srec, _ = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
        total += srec
    storage = torch.zeros(total, dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device)
    offs, _, shapes = record_layout(cfg.hidden, cfg.inter, cfg.bits)
    nf = len(ids) if n_fill is None else min(n_fill, len(ids))
    for i in range(nf):
        gen.manual_seed(_record_seed(seed, ids[i]))
        _fill_record(storage, i * rec, offs, shapes, gen, svh_scale, device)
    if cfg.shared_inter:
        soffs, _, sshapes = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
        gen.manual_seed(_record_seed(seed, cfg.n_experts))
        _fill_record(storage, len(ids) * rec, soffs, sshapes, gen, svh_scale, device)
    router_w, router_b = make_router(cfg, device, seed, router_scale, bias_std)
    packed, shared = _pointer_tables(cfg, storage, rec, len(ids))
    return ExpertLayer(cfg, storage, rec, packed.to(device), None if shared is None else shared.to(device),
                       router_w, router_b, ids)


def replicate_experts(layer: ExpertLayer, n_src: int) -> None:
    """Copy the first n_src routed records cyclically over the remaining experts (in place)."""
    rec = layer.record_bytes
    E = layer.n_local
    src = layer.storage[: n_src * rec]
    for e in range(n_src, E, n_src):
        n = min(n_src, E - e)
        layer.storage[e * rec: (e + n) * rec].copy_(src[: n * rec])
