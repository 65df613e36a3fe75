"""Expert parallelism: the routed experts sharded over ranks (one process per GPU), token rows
exchanged with NCCL over NVLink.

The reference runs every expert on one GPU and has no exchange; its kernel only anticipates
sharding with a local-expert filter (runtime/ds41/csrc/moe_coop2048/vendor/exl3_moe_coop_kernel.cuh:
208-223) and shared-only/zero rows for tokens without a local expert (:573-610). `EPMoE.forward`
keeps the operator contract of `Block.experts` (runtime/ds41/model.py:454-499): BF16 hidden states
in, BF16 out, every token's output = shared expert + sum of its routed experts' weighted outputs.

One forward on every rank (all ranks call it together, each with its own tokens):
  1. route its tokens with the full router (replicated, 7.3 MB for DeepSeek-V3)
  2. dispatch: for each destination rank, the rows of the tokens that have at least one expert
     there, each row once, with the slots of other ranks' experts given weight 0
  3. exchange row counts (exact mode only; one host synchronisation) and the rows themselves
     (one grouped send/recv of x rows, expert ids and weights)
  4. routed experts on the received rows, with the shared expert of its own tokens (sent to itself,
     all of them, as one segment) in the same launch (the NCCL transport runs it separately)
  5. return the weighted partial sums to the tokens' ranks (all-to-all) and add them up in rank
     order on top of the shared output

Transports. "peers" (the default on GPUs): every rank maps every other rank's arena (CUDA IPC over
NVLink); the dispatch kernel stores each row straight into its destination's receive segment and
releases a per-source flag, the experts run on the received rows in place, and the combine kernel
reads the partial sums from the peers' arenas after their flags; nothing synchronises the host and
no collective library runs in the step (protocol: include/eva_moe.h, EvaEpPeers). "nccl": the same
plan with torch.distributed grouped send/recv and all-to-all, in a "fixed" mode (segments of
max_tokens rows) or an "exact" mode (row counts exchanged first, one host synchronisation); it is
the baseline, and the transport the multi-process CPU tests check the exchange logic with.

The device work is behind an ops object (`CudaEpOps`, the C ABI of libeva_moe.so).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .config import MoEConfig
from .experts import ExpertLayer

_BF16, _F32, _I32 = torch.bfloat16, torch.float32, torch.int32


@dataclass(frozen=True)
class ExpertPlacement:
    """Which rank holds each global expert, and its column in that rank's pointer tables."""
    owner: np.ndarray      # int32 [E]
    local_id: np.ndarray   # int32 [E]
    world: int

    @classmethod
    def from_owner(cls, owner, world: int) -> "ExpertPlacement":
        owner = np.asarray(owner, dtype=np.int32)
        if owner.ndim != 1 or owner.size == 0 or owner.min() < 0 or owner.max() >= world:
            raise ValueError("owner must give a rank in [0, world) for every expert")
        local = np.zeros_like(owner)
        for r in range(world):
            ids = np.flatnonzero(owner == r)
            local[ids] = np.arange(ids.size, dtype=np.int32)
        return cls(owner, local, world)

    @classmethod
    def contiguous(cls, n_experts: int, world: int) -> "ExpertPlacement":
        """Experts [r E/N, (r+1) E/N) on rank r."""
        per = -(-n_experts // world)
        return cls.from_owner(np.arange(n_experts) // per, world)

    @classmethod
    def balanced(cls, load, world: int) -> "ExpertPlacement":
        """Equal expert counts per rank, experts taken in decreasing expected load, each going to the
        least-loaded rank that still has room (for skewed, e.g. Zipf, routing)."""
        load = np.asarray(load, dtype=np.float64)
        E = load.size
        room = np.full(world, E // world, dtype=np.int64)
        room[: E % world] += 1
        acc = np.zeros(world)
        owner = np.empty(E, dtype=np.int32)
        for e in np.argsort(-load, kind="stable"):
            r = min((r for r in range(world) if room[r] > 0), key=lambda r: (acc[r], r))
            owner[e] = r
            acc[r] += load[e]
            room[r] -= 1
        return cls.from_owner(owner, world)

    def experts_of(self, rank: int) -> tuple:
        """Global ids held by `rank`, in table order."""
        return tuple(int(e) for e in np.flatnonzero(self.owner == rank))


class _CudaView:
    """__cuda_array_interface__ of raw device memory (a torch view of an arena region)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _device_view(ptr: int, shape, typestr: str, device) -> torch.Tensor:
    return torch.as_tensor(_CudaView(ptr, shape, typestr), device=device)


class CudaEpOps:
    """Device work of one rank through libeva_moe.so; no fallback."""

    def __init__(self, layer: ExpertLayer, placement: ExpertPlacement, max_tokens: int, max_recv: int,
                 residency=None):
        device = residency.device if residency is not None else layer.device
        if not torch.cuda.is_available() or device.type != "cuda":
            raise RuntimeError("CudaEpOps requires a CUDA device; there is no CPU fallback")
        cfg = layer.cfg
        self.lib = _lib.load()
        self.cfg, self.layer, self.device = cfg, layer, device
        self.residency = residency
        self._miss_part = None          # partial rows of the copied experts' launch (expert cache)
        self.router_w = layer.router_w.to(device)
        self.router_b = layer.router_b.to(device)
        self.world = placement.world
        self.route_shape = _lib.shape_of(cfg)
        self.local_shape = _lib.shape_of(cfg, shared=False, n_experts=layer.n_local)
        self.shared_shape = _lib.shape_of(cfg, n_experts=layer.n_local)
        self.ws_route = self._ws(self.route_shape, max_tokens)
        # the arena launch runs the own tokens' shared expert too: size for the shared shape
        self.ws_local = self._ws(self.shared_shape if layer.shared is not None else self.local_shape, max_recv)
        self.ws_shared = self._ws(self.shared_shape, max_tokens) if layer.shared is not None else None
        self.owner = torch.as_tensor(placement.owner, dtype=_I32, device=self.device)
        self.local_id = torch.as_tensor(placement.local_id, dtype=_I32, device=self.device)
        self.status = torch.zeros(1, dtype=_I32, device=self.device)
        if residency is not None:   # resident slots behind the same handle format
            self._rows = tuple(residency.packed.unbind(0))
            self._shared = _lib.shared_array(residency.shared_addrs)
        else:
            self._rows = tuple(layer.packed.unbind(0))
            self._shared = _lib.shared_array(layer.shared.tolist()) if layer.shared is not None else None
        self._tables = _lib.table_array(self._rows)
        self._zero_sel = torch.zeros(max_tokens, cfg.topk, dtype=_I32, device=self.device)
        self._zero_rw = torch.zeros(max_tokens, cfg.topk, dtype=_F32, device=self.device)

    @property
    def has_shared(self) -> bool:
        return self._shared is not None

    def _ws(self, shape, rows):
        n = self.lib.eva_moe_workspace_bytes(ctypes.byref(shape), max(rows, 1))
        if n == 0:
            raise ValueError("unsupported MoE shape")
        return torch.zeros(n, dtype=torch.uint8, device=self.device)

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def route(self, x):
        M = x.shape[0]
        idx = torch.empty(M, self.cfg.topk, dtype=_I32, device=self.device)
        w = torch.empty(M, self.cfg.topk, dtype=_F32, device=self.device)
        rc = self.lib.eva_moe_route(ctypes.byref(self.route_shape), x.data_ptr(), int(x.dtype == _BF16), M,
                                    self.router_w.data_ptr(), self.router_b.data_ptr(), None,
                                    idx.data_ptr(), w.data_ptr(), self.ws_route.data_ptr(), self.ws_route.numel(),
                                    self._stream())
        _lib.check(rc, "eva_moe_route")
        return idx, w

    def dispatch(self, x, idx, w, capacity, segment):
        M, H, k = x.shape[0], self.cfg.hidden, self.cfg.topk
        counts = torch.empty(self.world, dtype=_I32, device=self.device)
        pos = torch.empty(self.world, M, dtype=_I32, device=self.device)
        sx = torch.empty(capacity, H, dtype=x.dtype, device=self.device)
        ssel = torch.empty(capacity, k, dtype=_I32, device=self.device)
        srw = torch.empty(capacity, k, dtype=_F32, device=self.device)
        rc = self.lib.eva_ep_dispatch(H, k, self.cfg.n_experts, x.data_ptr(), x.element_size(), M, idx.data_ptr(),
                                      w.data_ptr(), self.world, self.owner.data_ptr(), self.local_id.data_ptr(),
                                      capacity, segment, counts.data_ptr(), pos.data_ptr(), sx.data_ptr(),
                                      ssel.data_ptr(), srw.data_ptr(), self.status.data_ptr(), self._stream())
        _lib.check(rc, "eva_ep_dispatch")
        return counts, pos, sx, ssel, srw

    def experts(self, x, sel, rw, out_f32):
        R = x.shape[0]
        if R == 0:
            return out_f32
        rc = self.lib.eva_moe_experts(ctypes.byref(self.local_shape), x.data_ptr(), int(x.dtype == _BF16), R,
                                      sel.data_ptr(), 0, rw.data_ptr(), self._tables, None, self.ws_local.data_ptr(),
                                      self.ws_local.numel(), out_f32.data_ptr(), None, self._stream())
        _lib.check(rc, "eva_moe_experts")
        return out_f32

    def shared(self, x):
        """Shared expert of this rank's own tokens (every routed slot inactive), or None."""
        if self.ws_shared is None:
            return None
        M = x.shape[0]
        out = torch.empty(M, self.cfg.hidden, dtype=_F32, device=self.device)
        rc = self.lib.eva_moe_experts(ctypes.byref(self.shared_shape), x.data_ptr(), int(x.dtype == _BF16), M,
                                      self._zero_sel.data_ptr(), 0, self._zero_rw.data_ptr(), self._tables,
                                      self._shared, self.ws_shared.data_ptr(), self.ws_shared.numel(),
                                      out.data_ptr(), None, self._stream())
        _lib.check(rc, "eva_moe_experts (shared)")
        return out

    def combine(self, back, pos, base, out_bf16, out_f32=None):
        M = pos.shape[1]
        rc = self.lib.eva_ep_combine(self.cfg.hidden, M, self.world, back.data_ptr(), pos.data_ptr(),
                                     _lib.ptr(base), _lib.ptr(out_f32), _lib.ptr(out_bf16), self._stream())
        _lib.check(rc, "eva_ep_combine")

    # -- exchange over NVLink peer memory -----------------------------------------------------------
    def setup_peers(self, group, rank: int, world: int, segment_rows: int):
        """Allocate this rank's arena, exchange CUDA IPC handles, map every peer's arena."""
        P = _lib.EvaEpPeers()
        P.world, P.rank, P.H, P.topk = world, rank, self.cfg.hidden, self.cfg.topk
        P.n_experts, P.segment_rows, P.x_elem_bytes = self.cfg.n_experts, segment_rows, 2
        _lib.check(self.lib.eva_ep_arena_layout(ctypes.byref(P)), "eva_ep_arena_layout")
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.eva_peer_alloc(P.bytes, ctypes.byref(own), handle), "eva_peer_alloc")
        self._own_arena = own.value
        self._opened = []
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        with torch.cuda.device(self.device):
            for r in range(world):
                if r == rank:
                    P.arena[r] = own.value
                    continue
                ptr = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                _lib.check(self.lib.eva_peer_open(buf, ctypes.byref(ptr)), "eva_peer_open")
                P.arena[r] = ptr.value
                self._opened.append(ptr.value)
        P.owner, P.local_id = self.owner.data_ptr(), self.local_id.data_ptr()
        self.peers = P
        self.segment_rows = segment_rows
        self._arena_rows = R = world * segment_rows
        base = own.value
        self.recv_sel = _device_view(base + P.off_sel, (R, self.cfg.topk), "<i4", self.device)
        self.recv_rw = _device_view(base + P.off_rw, (R, self.cfg.topk), "<f4", self.device)
        self.part = _device_view(base + P.off_part, (R, self.cfg.hidden), "<f4", self.device)

    def close_peers(self, group=None):
        """Unmap the peers' arenas, then (after every rank has) free this rank's own."""
        if getattr(self, "peers", None) is None:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                self.lib.eva_peer_close(ctypes.c_void_p(ptr))
        if dist.is_initialized() and self.peers.world > 1:
            dist.barrier(group)
        with torch.cuda.device(self.device):
            self.lib.eva_peer_free(ctypes.c_void_p(self._own_arena))
        self.peers = None

    def dispatch_peers(self, x, idx, w, all_to_self=False):
        M = x.shape[0]
        counts = torch.empty(self.world, dtype=_I32, device=self.device)
        pos = torch.empty(self.world, M, dtype=_I32, device=self.device)
        rc = self.lib.eva_ep_dispatch_peers(ctypes.byref(self.peers), x.data_ptr(), M, idx.data_ptr(), w.data_ptr(),
                                            int(all_to_self), counts.data_ptr(), pos.data_ptr(),
                                            self.status.data_ptr(), self._stream())
        _lib.check(rc, "eva_ep_dispatch_peers")
        return counts, pos

    def wait_rows(self):
        _lib.check(self.lib.eva_ep_wait_rows(ctypes.byref(self.peers), self.status.data_ptr(), self._stream()),
                   "eva_ep_wait_rows")

    def _experts_call(self, rw_ptr: int, out_ptr: int, own_rows: int = -1):
        """Experts of the arena rows; own_rows >= 0: this rank's own tokens (the first own_rows rows of
        its own segment) also get the shared expert, in the same launch."""
        P = self.peers
        base = self._own_arena
        if own_rows >= 0 and self._shared is not None:
            rc = self.lib.eva_moe_experts_window(ctypes.byref(self.shared_shape), base + P.off_x, 1, self._arena_rows,
                                                 base + P.off_sel, 0, rw_ptr, self._tables, self._shared,
                                                 self.peers.rank * self.segment_rows, own_rows,
                                                 self.ws_local.data_ptr(), self.ws_local.numel(), out_ptr, None,
                                                 self._stream())
        else:
            rc = self.lib.eva_moe_experts(ctypes.byref(self.local_shape), base + P.off_x, 1, self._arena_rows,
                                          base + P.off_sel, 0, rw_ptr, self._tables, None, self.ws_local.data_ptr(),
                                          self.ws_local.numel(), out_ptr, None, self._stream())
        _lib.check(rc, "eva_moe_experts (arena)")

    def experts_arena(self, own_rows: int = -1, mark=None):
        """Routed experts of every received row, from this rank's arena into its partial rows.

        With a PooledLayer (device-side expert cache), the experts the received rows select are made
        resident on the device stream without a host synchronisation, and the next layer's prefetch is
        issued. With an ExpertResidency (host-managed), the needed set is read on the host (a
        synchronisation), misses are copied from pinned host memory on the side stream, and when more
        are selected than there are slots they run in groups that fit, each group's slots masked into
        its own launch and the partial sums added."""
        P = self.peers
        base = self._own_arena
        res = self.residency
        if res is None:
            self._experts_call(base + P.off_rw, base + P.off_part, own_rows)
        elif hasattr(res, "plan"):
            # device-side expert cache: the plan in stream order; the misses' copies, then the next
            # layer's prefetch, on the pool's copy stream; the resident experts' launch overlaps the
            # copies and the copied experts' launch follows them
            hit, miss, copied = res.plan(self.recv_sel, self.recv_rw, split=True)
            if res.next is not None:
                res.next.prefetch()
            self._experts_call(hit.data_ptr(), base + P.off_part, own_rows)
            torch.cuda.current_stream(self.device).wait_event(copied)
            if self._miss_part is None:
                self._miss_part = torch.empty_like(self.part)
            self._experts_call(miss.data_ptr(), self._miss_part.data_ptr(), -1)
            self.part.add_(self._miss_part)
        else:
            active = self.recv_rw != 0
            needed = torch.unique(self.recv_sel[active]).tolist()      # host synchronisation
            groups = [needed[i:i + res.n_slots] for i in range(0, len(needed), res.n_slots)] or [[]]
            if len(groups) == 1:
                res.ensure(groups[0])
                self._experts_call(base + P.off_rw, base + P.off_part, own_rows)
                res.mark_used()
            else:
                keep = torch.zeros(self.layer.n_local, dtype=torch.bool, device=self.device)
                tmp = torch.empty_like(self.part)
                for gi, g in enumerate(groups):
                    res.ensure(g)
                    keep.zero_()
                    keep[torch.as_tensor(g, device=self.device)] = True
                    rw_g = torch.where(keep[self.recv_sel.long()], self.recv_rw, 0.0)
                    self._experts_call(rw_g.data_ptr(), (self.part if gi == 0 else tmp).data_ptr(),
                                       own_rows if gi == 0 else -1)
                    res.mark_used()
                    if gi:
                        self.part.add_(tmp)
        if mark is not None:
            mark("experts")
        # the partials are published by the combine launch (eva_ep_combine_peers), first thing

    def combine_peers(self, pos, base, out_bf16, out_f32=None):
        rc = self.lib.eva_ep_combine_peers(ctypes.byref(self.peers), pos.shape[1], pos.data_ptr(), _lib.ptr(base),
                                           _lib.ptr(out_f32), _lib.ptr(out_bf16), self.status.data_ptr(),
                                           self._stream())
        _lib.check(rc, "eva_ep_combine_peers")

    def read_status(self) -> int:
        st = int(self.status.item())
        for ws in (self.ws_route, self.ws_local, self.ws_shared):
            if ws is not None:
                v = ctypes.c_int32(0)
                _lib.check(self.lib.eva_moe_read_status(ws.data_ptr(), ctypes.byref(v), self._stream()), "status")
                st |= v.value
        return st


class EPMoE:
    """Expert-parallel MoE layer operator (one instance per rank, all ranks call forward together).

    layer:      this rank's experts (layer.experts == placement.experts_of(rank)) plus the shared
                expert and the full router
    max_tokens: most tokens one rank passes to one forward
    residency:  optional eva_b200.residency.ExpertResidency holding this rank's experts in pinned host
                memory with a device slot budget (then `layer` may live in host memory)
    transport:  "peers" (default with the CUDA ops: rows stored straight into the destinations' arenas
                over NVLink by this library's kernels, segments of max_tokens rows, no host
                synchronisation, no collective library in the step) or "nccl" (torch.distributed
                grouped send/recv and all-to-all; the only transport of the CPU checker)
    mode:       nccl transport only: "fixed" (segments of max_tokens rows, no host synchronisation),
                "exact" (counts exchanged first) or "auto" (fixed up to 64 tokens per rank)
    """

    def __init__(self, layer: ExpertLayer, placement: ExpertPlacement, *, max_tokens: int = 64,
                 mode: str = "auto", group=None, ops=None, transport: str = "auto", residency=None):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if placement.world != self.world:
            raise ValueError(f"placement is for {placement.world} ranks, the group has {self.world}")
        if tuple(layer.experts) != placement.experts_of(self.rank):
            raise ValueError("layer.experts must be placement.experts_of(rank)")
        if mode not in ("auto", "fixed", "exact"):
            raise ValueError("mode must be auto, fixed or exact")
        self.cfg: MoEConfig = layer.cfg
        self.layer, self.placement = layer, placement
        self.max_tokens = max_tokens
        self.mode = ("fixed" if max_tokens <= 64 else "exact") if mode == "auto" else mode
        self.max_recv = self.world * max_tokens
        self.capacity = self.world * max_tokens if self.mode == "fixed" else max_tokens * min(self.cfg.topk, self.world)
        self.ops = ops if ops is not None else CudaEpOps(layer, placement, max_tokens, self.max_recv, residency)
        self.device = getattr(self.ops, "device", layer.device)
        if transport == "auto":
            transport = "peers" if isinstance(self.ops, CudaEpOps) else "nccl"
        if transport not in ("peers", "nccl"):
            raise ValueError("transport must be peers, nccl or auto")
        if transport == "peers" and not hasattr(self.ops, "setup_peers"):
            raise ValueError("the peers transport needs CUDA ops")
        if getattr(self.ops, "residency", None) is not None and transport != "peers":
            raise ValueError("expert residency runs with the peers transport")
        self.transport = transport
        if dist.is_initialized() and self.world > 1:
            dist.barrier(group)   # communicator set up before the first grouped send/recv
        if transport == "peers":
            self.ops.setup_peers(group, self.rank, self.world, max_tokens)

    def close(self):
        """Release the peer-memory arenas (every rank calls it, before destroying the process group)."""
        if self.transport == "peers":
            self.ops.close_peers(self.group)

    # -- exchange helpers (torch.distributed; NCCL on GPUs, gloo for the CPU tests) ---------------------
    def _exchange_rows(self, send, send_counts, send_offs, recv, recv_counts, recv_offs):
        """Rows of each tensor in `send` go to every rank (grouped point-to-point; own rows copied)."""
        ops = []
        for r in range(self.world):
            if r == self.rank:
                for s, d in zip(send, recv):
                    n = send_counts[r]
                    if n:
                        d[recv_offs[r]: recv_offs[r] + n].copy_(s[send_offs[r]: send_offs[r] + n])
                continue
            gr = dist.get_global_rank(self.group, r) if self.group is not None else r
            if send_counts[r]:
                for s in send:
                    ops.append(dist.P2POp(dist.isend, s[send_offs[r]: send_offs[r] + send_counts[r]], gr, self.group))
            if recv_counts[r]:
                for d in recv:
                    ops.append(dist.P2POp(dist.irecv, d[recv_offs[r]: recv_offs[r] + recv_counts[r]], gr, self.group))
        return dist.batch_isend_irecv(ops) if ops else []

    def forward(self, x, *, out=None, out_f32=None, idx_out=None, w_out=None, phases=None):
        """x: BF16 [M, H] on this rank's device (M <= max_tokens); returns BF16 [M, H].

        phases: optional list that receives (name, CUDA event) after each phase of the peer-memory
        step, in stream order: route, dispatch (plan + pack stores into the peers' arenas), wait
        (until every peer's rows arrived), experts, combine (publish this rank's partials, wait until
        every peer's arrived, then the sum)."""
        cfg, ops = self.cfg, self.ops
        mark = None
        if phases is not None:
            def mark(name):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(torch.cuda.current_stream(self.device))
                phases.append((name, ev))
            mark("start")
        if x.dim() != 2 or x.shape[1] != cfg.hidden or x.dtype != _BF16:
            raise ValueError(f"x must be BF16 [M, {cfg.hidden}]")
        M = x.shape[0]
        if not 0 <= M <= self.max_tokens:
            raise ValueError(f"0..{self.max_tokens} tokens per rank")
        x = x.contiguous()
        idx, w = ops.route(x)
        if idx_out is not None:
            idx_out.copy_(idx)
        if w_out is not None:
            w_out.copy_(w)
        if out is None:
            out = torch.empty(M, cfg.hidden, dtype=_BF16, device=self.device)
        if self.transport == "peers":
            if mark is not None:
                mark("route")
            fuse = ops.has_shared
            _, pos = ops.dispatch_peers(x, idx, w, all_to_self=fuse)
            base = None
            if not fuse:
                base = ops.shared(x)
            if mark is not None:
                mark("dispatch")
            ops.wait_rows()
            if mark is not None:
                mark("wait")
            ops.experts_arena(own_rows=M if fuse else -1, mark=mark)   # own tokens' shared expert in the same launch
            ops.combine_peers(pos, base, out, out_f32)   # publishes this rank's partials, then waits for all
            if mark is not None:
                mark("combine")
            return out
        seg = self.max_tokens if self.mode == "fixed" else 0
        counts, pos, sx, ssel, srw = ops.dispatch(x, idx, w, self.capacity, seg)
        W = self.world
        if self.mode == "fixed":
            send_counts = recv_counts = [seg] * W
        else:
            rc = torch.empty_like(counts)
            if self.world > 1:
                dist.all_to_all_single(rc, counts, group=self.group)
            else:
                rc.copy_(counts)
            both = torch.cat([counts, rc]).cpu().tolist()     # the one host synchronisation
            send_counts, recv_counts = both[:W], both[W:]
        send_offs = np.concatenate([[0], np.cumsum(send_counts)[:-1]]).astype(int).tolist()
        recv_offs = np.concatenate([[0], np.cumsum(recv_counts)[:-1]]).astype(int).tolist()
        R = int(sum(recv_counts))
        if R > self.max_recv:
            raise RuntimeError(f"{R} received rows exceed max_recv {self.max_recv}")
        rx = torch.empty(R, cfg.hidden, dtype=x.dtype, device=self.device)
        rsel = torch.empty(R, cfg.topk, dtype=_I32, device=self.device)
        rrw = torch.empty(R, cfg.topk, dtype=_F32, device=self.device)
        works = self._exchange_rows((sx, ssel, srw), send_counts, send_offs, (rx, rsel, rrw), recv_counts, recv_offs)
        base = ops.shared(x)                      # overlaps the exchange
        for wk in works:
            wk.wait()
        part = torch.empty(R, cfg.hidden, dtype=_F32, device=self.device)
        ops.experts(rx, rsel, rrw, part)
        back = torch.empty(sx.shape[0], cfg.hidden, dtype=_F32, device=self.device)
        works = self._exchange_rows((part,), recv_counts, recv_offs, (back,), send_counts, send_offs)
        for wk in works:
            wk.wait()
        ops.combine(back, pos, base, out, out_f32)
        return out

    __call__ = forward

    def status(self) -> int:
        return self.ops.read_status()
