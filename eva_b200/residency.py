"""Expert residency: a device budget of expert slots per layer, misses copied from pinned host memory
on a side stream, and the reference's pointer-table handle kept pointing at the resident copies.

Mirrors the reference's ExpertCache mechanics (paths within the Findddx/eva project):
  _blit    runtime/ds41/cache.py:1852-1862   H2D copy of one expert record into a device slot
  _bind    cache.py:1864-1887                 the 9 device addresses of the expert in the host table
  _unbind  cache.py:1889-1899                 zero column (unbound; a kernel that selects it flags it)
  _flush   cache.py:1901-1915                 host table -> device table, in stream order
  install  cache.py:1946-1996 (_install_if_absent)
  prefetch cache.py:2064-2080 (prefetch_gpu)  copies on a side stream while other work runs
Placement/promotion policy, NVMe tiers and the frozen tier are out of scope; eviction here is
least-recently-used among the experts the current step does not need.

The handle is int64 [9, n_local] in the row order [g.trellis, g.suh, g.svh, u.trellis, u.suh, u.svh,
d.trellis, d.suh, d.svh]; the shared expert stays resident.
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from .experts import ROW, ExpertLayer, record_layout


class SlotLRU:
    """Which expert holds which device slot; least-recently-used eviction."""

    def __init__(self, n_slots: int):
        if n_slots < 1:
            raise ValueError("at least one slot")
        self.n_slots = n_slots
        self.slot_of: dict[int, int] = {}
        self.lru: OrderedDict[int, None] = OrderedDict()
        self.free = list(range(n_slots - 1, -1, -1))

    def lookup(self, expert: int):
        slot = self.slot_of.get(expert)
        if slot is not None:
            self.lru.move_to_end(expert)
        return slot

    def assign(self, expert: int, protected) -> tuple[int, int | None]:
        """A slot for `expert` (not resident): a free one, else the least recently used expert's that is
        not in `protected`. Returns (slot, evicted expert or None)."""
        if expert in self.slot_of:
            raise ValueError("already resident")
        evicted = None
        if self.free:
            slot = self.free.pop()
        else:
            for cand in self.lru:
                if cand not in protected:
                    evicted = cand
                    break
            if evicted is None:
                raise RuntimeError("every slot holds an expert this step needs: budget too small")
            slot = self.slot_of.pop(evicted)
            del self.lru[evicted]
        self.slot_of[expert] = slot
        self.lru[expert] = None
        return slot, evicted


class ExpertResidency:
    """A layer's routed experts in pinned host memory, `n_slots` of them resident on the device."""

    def __init__(self, layer: ExpertLayer, n_slots: int, device, copy_stream=None):
        cfg = layer.cfg
        self.cfg, self.device = cfg, torch.device(device)
        self.n_local = layer.n_local
        self.experts = layer.experts
        rec = layer.record_bytes
        self.record_bytes = rec
        self.n_slots = min(n_slots, self.n_local)
        self.policy = SlotLRU(self.n_slots)
        src = layer.storage
        self.host = torch.empty(self.n_local * rec, dtype=torch.uint8, pin_memory=True)
        self.host.copy_(src[: self.n_local * rec])
        self.slots = torch.empty(self.n_slots * rec, dtype=torch.uint8, device=self.device)
        shared = src[self.n_local * rec:]
        self.shared_storage = shared.to(self.device) if shared.numel() else None
        offs, _, _ = record_layout(cfg.hidden, cfg.inter, cfg.bits)
        self._row_off = [0] * 9
        for (proj, kind), row in ROW.items():
            self._row_off[row] = offs[(proj, kind)][0]
        self.shared_addrs = None
        if self.shared_storage is not None:
            soffs, _, _ = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
            base = self.shared_storage.data_ptr()
            self.shared_addrs = [0] * 9
            for (proj, kind), row in ROW.items():
                self.shared_addrs[row] = base + soffs[(proj, kind)][0]
        self.host_ptrs = torch.zeros(9, self.n_local, dtype=torch.int64, pin_memory=True)
        self.packed = torch.zeros(9, self.n_local, dtype=torch.int64, device=self.device)
        self.copy_stream = copy_stream if copy_stream is not None else torch.cuda.Stream(self.device)
        self.last_use = None        # event after the last launch that read the slots / table
        self.flush_event = None     # event after the last host-table copy
        self.stats = {"hits": 0, "misses": 0, "h2d_bytes": 0}

    # -- the reference's steps ------------------------------------------------------------------------
    def _blit(self, expert: int, slot: int):
        rec = self.record_bytes
        self.slots[slot * rec:(slot + 1) * rec].copy_(self.host[expert * rec:(expert + 1) * rec], non_blocking=True)
        self.stats["h2d_bytes"] += rec

    def _bind(self, expert: int, slot: int):
        base = self.slots.data_ptr() + slot * self.record_bytes
        for row in range(9):
            self.host_ptrs[row, expert] = base + self._row_off[row]

    def _unbind(self, expert: int):
        self.host_ptrs[:, expert] = 0

    def _flush(self):
        self.packed.copy_(self.host_ptrs, non_blocking=True)
        self.flush_event = torch.cuda.Event()
        self.flush_event.record(torch.cuda.current_stream(self.device))

    def install(self, experts) -> torch.cuda.Event:
        """Make `experts` (local ids) resident; copies and the table update run on the copy stream after
        the last recorded use. Returns the event that completes them."""
        need = [int(e) for e in dict.fromkeys(experts)]
        if len(need) > self.n_slots:
            raise RuntimeError(f"{len(need)} experts needed at once, {self.n_slots} slots")
        missing = []
        for e in need:
            if not 0 <= e < self.n_local:
                raise ValueError(f"expert {e} outside [0, {self.n_local})")
            if self.policy.lookup(e) is None:
                missing.append(e)
            else:
                self.stats["hits"] += 1
        ev = torch.cuda.Event()
        with torch.cuda.stream(self.copy_stream):
            if missing:
                if self.last_use is not None:
                    self.copy_stream.wait_event(self.last_use)
                if self.flush_event is not None:
                    self.flush_event.synchronize()      # the pinned table is about to change
                protected = set(need)
                for e in missing:
                    slot, evicted = self.policy.assign(e, protected)
                    if evicted is not None:
                        self._unbind(evicted)
                    self._blit(e, slot)
                    self._bind(e, slot)
                    self.stats["misses"] += 1
                self._flush()
            ev.record(self.copy_stream)
        return ev

    def ensure(self, experts, stream=None) -> None:
        """install() and make `stream` (default: current) wait for it."""
        ev = self.install(experts)
        (stream or torch.cuda.current_stream(self.device)).wait_event(ev)

    def prefetch(self, experts) -> torch.cuda.Event:
        """install() without waiting: the copies overlap whatever the compute stream does next."""
        return self.install(experts)

    def mark_used(self, stream=None) -> None:
        """Record that launches reading the slots / table were issued on `stream` up to here."""
        self.last_use = torch.cuda.Event()
        self.last_use.record(stream or torch.cuda.current_stream(self.device))
