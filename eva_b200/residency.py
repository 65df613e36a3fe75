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
        if src.device.type == "cpu" and src.is_pinned():    # already page-locked: copy from it in place
            self.host = src[: self.n_local * rec]
        else:
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


# -------------------------------------------------------------------------------------------------
# Device-side expert cache (the default for expert-parallel stacks): no host synchronisation.

import ctypes  # noqa: E402

from . import _lib  # noqa: E402

_POOL_MAX_LOCAL = 1024


class ExpertPool:
    """Device record slots shared by the layers of one GPU (eva_pool_plan / eva_pool_copy).

    A layer added with add_layer() keeps its experts in pinned host memory; the experts its routes
    select are made resident on the device stream in two launches (plan: needed set, CLOCK slot
    choice, pointer-table updates; copy: records read from pinned host memory by the device), and a
    layer's predicted experts (its previous step's needed set) can be prefetched on the pool's copy
    stream while another layer runs. Every slot holds one record; n_slots must be at least the largest
    layer's local expert count, so that a layer's needed set always fits."""

    def __init__(self, device, n_slots: int, record_bytes: int, max_layers: int = 256, timing: bool = False):
        self.lib = _lib.load()
        self.timing = timing             # record CUDA events around every staging launch
        self._events = {"plan": [], "copy": [], "prefetch": []}
        self.device = torch.device(device)
        if record_bytes % 16:
            raise ValueError("record size must be a multiple of 16 bytes")
        self.n_slots, self.record_bytes, self.max_layers = int(n_slots), int(record_bytes), int(max_layers)
        self.slots = torch.empty(self.n_slots * self.record_bytes, dtype=torch.uint8, device=self.device)
        self.owner = torch.full((self.n_slots,), -1, dtype=torch.int32, device=self.device)
        self.stamp = torch.zeros(self.n_slots, dtype=torch.int64, device=self.device)
        # {hand, 0, status bits, 0, bytes copied (int64), plan counter (int64)}
        self.state = torch.zeros(8, dtype=torch.int32, device=self.device)
        self._layer_bytes = ctypes.sizeof(_lib.EvaPoolLayer)
        self.layers_dev = torch.zeros(self.max_layers * self._layer_bytes, dtype=torch.uint8, device=self.device)
        self.layers: list[PooledLayer] = []
        self.struct = _lib.EvaExpertPool(self.n_slots, 0, self.record_bytes, self.slots.data_ptr(),
                                         self.owner.data_ptr(), self.stamp.data_ptr(), self.state.data_ptr())
        self.copy_stream = torch.cuda.Stream(self.device)

    def add_layer(self, layer: ExpertLayer) -> "PooledLayer":
        if len(self.layers) >= self.max_layers:
            raise ValueError(f"at most {self.max_layers} layers per pool")
        if layer.record_bytes != self.record_bytes:
            raise ValueError("all layers of a pool have records of the pool's size")
        if layer.n_local > min(self.n_slots, _POOL_MAX_LOCAL):
            raise ValueError(f"a layer's {layer.n_local} local experts must fit the pool ({self.n_slots} slots, "
                             f"at most {_POOL_MAX_LOCAL})")
        pl = PooledLayer(self, len(self.layers), layer)
        self.layers.append(pl)
        raw = bytes(pl.struct)
        off = pl.index * self._layer_bytes
        self.layers_dev[off:off + len(raw)].copy_(torch.frombuffer(bytearray(raw), dtype=torch.uint8))
        return pl

    def bytes_copied(self) -> int:
        """Record bytes the copies moved so far (reads the device counter: synchronises)."""
        return int(self.state[4:6].cpu().view(torch.int64).item())

    def plan_counter(self) -> int:
        """Exact plans so far (the stamp of the latest one; reads the device counter: synchronises)."""
        return int(self.state[6:8].cpu().view(torch.int64).item())

    def status(self) -> int:
        return int(self.state[2].item())

    def staging_ms(self) -> dict:
        """Device time of the stagings issued since the last call (timing=True): 'plan' = exact plans
        (the stream that runs the layers), 'copy' = their copies, 'prefetch' = prefetch plans and copies
        (the pool's copy stream; with split plans the exact copies run there too). Synchronises."""
        torch.cuda.synchronize(self.device)
        out = {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self._events.items()}
        for v in self._events.values():
            v.clear()
        return out

    def _begin(self, stream):
        if not self.timing:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    def _end(self, start, stream, kind):
        if start is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            self._events[kind].append((start, ev))


class PooledLayer:
    """One layer's experts behind an ExpertPool, with the attributes EPMoE reads from a residency:
    `packed` (the reference's int64 [9, n_local] handle, kept bound to the resident copies by the
    device), `shared_addrs` (the shared expert, resident in its own device buffer), `device`."""

    def __init__(self, pool: ExpertPool, index: int, layer: ExpertLayer):
        cfg = layer.cfg
        self.pool, self.index, self.cfg = pool, index, cfg
        self.device = pool.device
        self.n_local, self.experts, self.record_bytes = layer.n_local, layer.experts, layer.record_bytes
        self.n_slots = pool.n_slots
        rec = self.record_bytes
        src = layer.storage
        if src.device.type == "cpu" and src.is_pinned():    # already page-locked: read in place
            self.host = src[: self.n_local * rec]
        else:
            self.host = torch.empty(self.n_local * rec, dtype=torch.uint8, pin_memory=True)
            self.host.copy_(src[: self.n_local * rec])
        if not pool.lib.eva_host_mapped(ctypes.c_void_p(self.host.data_ptr())):
            raise RuntimeError("pinned host records are not readable by the device at their address")
        shared = src[self.n_local * rec:]
        self.shared_storage = shared.to(self.device) if shared.numel() else None
        self.shared_addrs = None
        if self.shared_storage is not None:
            soffs, _, _ = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
            base = self.shared_storage.data_ptr()
            self.shared_addrs = [0] * 9
            for (proj, kind), row in ROW.items():
                self.shared_addrs[row] = base + soffs[(proj, kind)][0]
        offs, _, _ = record_layout(cfg.hidden, cfg.inter, cfg.bits)
        row_off = [0] * 9
        for (proj, kind), row in ROW.items():
            row_off[row] = offs[(proj, kind)][0]
        self.packed = torch.zeros(9, self.n_local, dtype=torch.int64, device=self.device)
        self.slot_of = torch.full((self.n_local,), -1, dtype=torch.int32, device=self.device)
        self.last_needed = torch.zeros((self.n_local + 31) // 32, dtype=torch.int32, device=self.device)
        self.jobs = torch.zeros(1 + 2 * self.n_local, dtype=torch.int32, device=self.device)
        self.pjobs = torch.zeros(1 + 2 * self.n_local, dtype=torch.int32, device=self.device)
        self.struct = _lib.EvaPoolLayer(index, self.n_local, self.host.data_ptr(), (ctypes.c_int64 * 9)(*row_off),
                                        self.slot_of.data_ptr(), self.last_needed.data_ptr(), self.packed.data_ptr())
        self._split = None                      # rw_hit / rw_miss buffers of split plans
        self.next: PooledLayer | None = None    # the layer to prefetch once this one is planned
        self.ready = None                       # event: this layer's prefetch is done

    def _call(self, fn, *args):
        _lib.check(fn(ctypes.byref(self.pool.struct), ctypes.c_void_p(self.pool.layers_dev.data_ptr()), self.index,
                      *args), fn.__name__)

    def plan(self, sel: torch.Tensor, rw: torch.Tensor, stream=None, split: bool = False):
        """Make the experts selected by sel / rw ([rows, topk], rw 0 = inactive) resident, after this
        layer's prefetch if one is in flight. The plan runs in stream order on `stream` (default:
        current). split=False: the copies follow it on the same stream; returns None. split=True: the
        copies run on the pool's copy stream and the call returns (rw_hit, rw_miss, copied): rw split
        into the routes of experts already resident and of those being copied, and the event after the
        copies, so that an experts launch over rw_hit overlaps them and one over rw_miss waits for
        `copied`."""
        s = stream or torch.cuda.current_stream(self.device)
        if self.ready is not None:
            s.wait_event(self.ready)
            self.ready = None
        rows, topk = sel.shape
        lib, pool = self.pool.lib, self.pool
        hit = miss = None
        if split:
            if self._split is None or self._split[0].shape != rw.shape:
                self._split = (torch.empty_like(rw), torch.empty_like(rw))
            hit, miss = self._split
        t = pool._begin(s)
        self._call(lib.eva_pool_plan, ctypes.c_void_p(sel.data_ptr()), int(sel.dtype == torch.int64),
                   ctypes.c_void_p(rw.data_ptr()), rows, topk, 0, ctypes.c_void_p(self.jobs.data_ptr()),
                   None if hit is None else ctypes.c_void_p(hit.data_ptr()),
                   None if miss is None else ctypes.c_void_p(miss.data_ptr()), ctypes.c_void_p(s.cuda_stream))
        pool._end(t, s, "plan")
        cs = pool.copy_stream if split else s
        if split:
            ev = torch.cuda.Event()
            ev.record(s)
            cs.wait_event(ev)
        t = pool._begin(cs)
        self._call(lib.eva_pool_copy, ctypes.c_void_p(self.jobs.data_ptr()), ctypes.c_void_p(cs.cuda_stream))
        pool._end(t, cs, "copy")
        if not split:
            return None
        copied = torch.cuda.Event()
        copied.record(cs)
        return hit, miss, copied

    def prefetch(self, after=None) -> None:
        """This layer's previous needed set made resident on the pool's copy stream, after the work
        already issued on `after` (default: the current stream), typically while another layer runs."""
        cs = self.pool.copy_stream
        ev = torch.cuda.Event()
        ev.record(after or torch.cuda.current_stream(self.device))
        cs.wait_event(ev)
        lib = self.pool.lib
        dummy = ctypes.c_void_p(self.jobs.data_ptr())
        t = self.pool._begin(cs)
        self._call(lib.eva_pool_plan, dummy, 0, dummy, 0, self.cfg.topk, 1, ctypes.c_void_p(self.pjobs.data_ptr()),
                   None, None, ctypes.c_void_p(cs.cuda_stream))
        self._call(lib.eva_pool_copy, ctypes.c_void_p(self.pjobs.data_ptr()), ctypes.c_void_p(cs.cuda_stream))
        self.pool._end(t, cs, "prefetch")
        self.ready = torch.cuda.Event()
        self.ready.record(cs)
