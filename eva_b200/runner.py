"""Host side of the MoE hot path: the reference's operator interfaces over the C ABI.

* `EvaMoERunner.run(x, sel, weights, packed, k, limit, *, check_bounds=True)` is a drop-in for the
  reference's runner boundary: runtime/ds41/moe_coop512.py:203-253 (`CoopRunner512.run`),
  moe_coop2048.py:255-307 and moe_coop3072.py (`CoopRunner2048/3072.run`), called from
  `ExpertCache._run_coop` (runtime/ds41/cache.py:2152-2225). Same argument meaning: Half x, int64
  routes, Half/BF16/Float route weights rounded to Half (zero = inactive slot), nine borrowed
  pointer tables in the cache's row order (or one int64 [9, n_local] tensor), EXL3 K and the SwiGLU
  limit. Returns Float[M, H] (routed experts only, like the reference runner). Same error
  behaviour: ValueError for bad arguments, RuntimeError for launch failures, and a failed runner
  refuses further calls.
* `EvaMoE` is the MoE-layer operator of `Block` (runtime/ds41/model.py:404-499): `route(x)` returns
  (weights, indices) as `Block.route`, `experts(x)` routes, runs the routed experts and the shared
  expert and returns the result in x's dtype (BF16 hidden states in and out).

Both run on the caller's current CUDA stream and never synchronise the host unless asked to
(`check_bounds=True` reads the device status word after the launch); the library call itself uses
the workspace fixed at construction, and only the returned tensors come from torch's allocator.
"""
from __future__ import annotations

import ctypes
import math
import threading

import torch

from . import _lib
from .config import MoEConfig
from .experts import ExpertLayer

_F16, _BF16, _F32, _I64 = torch.float16, torch.bfloat16, torch.float32, torch.int64


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, device, name: str):
    if not isinstance(t, torch.Tensor) or t.device != device:
        raise ValueError(f"{name} must be a tensor on {device}")


class EvaMoERunner:
    """Routed-expert runner with the reference runner's call shape (no shared expert)."""

    def __init__(self, device="cuda", topk=6, hidden=5120, inter=2304, max_rows=64, *, n_experts=384):
        if not torch.cuda.is_available():
            raise RuntimeError("EvaMoERunner requires CUDA; there is no CPU fallback")
        self.lib = _lib.load()
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("EvaMoERunner requires a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if type(topk) is not int or not 1 <= topk <= 32:
            raise ValueError("topk must be an int in 1..32")
        if type(max_rows) is not int or max_rows < 1:
            raise ValueError("max_rows must be a positive int")
        self.topk, self.hidden, self.inter, self.max_rows, self.n_experts = topk, hidden, inter, max_rows, n_experts
        self._lock, self._failed = threading.Lock(), False
        # like the reference runner (moe_coop2048.py:263-290): one owner thread, the construction stream
        self._owner_thread = threading.get_ident()
        self._owner_stream = torch.cuda.current_stream(self.device).cuda_stream
        self._ws = {}
        self.out = torch.empty(max_rows, hidden, device=self.device, dtype=_F32)
        self.rw = torch.empty(max_rows, topk, device=self.device, dtype=_F32)

    def _shape(self, k, limit, n_local) -> _lib.EvaMoeShape:
        return _lib.EvaMoeShape(self.hidden, self.inter, n_local, self.topk, int(k), 0, 3, 2, 1, 1, 1,
                                _lib.ACT_CLAMP_AFTER, _lib.ACT_CLAMP_BEFORE, 1.0, float(limit))

    def _workspace(self, shape) -> torch.Tensor:
        key = (shape.n_experts, shape.bits)
        ws = self._ws.get(key)
        if ws is None:
            n = self.lib.eva_moe_workspace_bytes(ctypes.byref(shape), self.max_rows)
            if n == 0:
                raise ValueError("unsupported shape (hidden % 256, inter % 128, K in 2..4)")
            ws = torch.zeros(n, dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    @staticmethod
    def _tables(packed):
        if isinstance(packed, torch.Tensor):
            if packed.ndim != 2 or packed.shape[0] != 9 or packed.dtype != _I64:
                raise ValueError("packed must be int64 [9, n_local] or nine int64 tables")
            packed = tuple(packed.unbind(0))
        if not isinstance(packed, (tuple, list)) or len(packed) != 9:
            raise ValueError("nine borrowed pointer tables required")
        n_local = packed[0].numel()
        for t in packed:
            if not isinstance(t, torch.Tensor) or t.dtype != _I64 or t.ndim != 1 or t.numel() != n_local:
                raise ValueError("pointer tables must be int64 [n_local] of equal length")
            if not t.is_contiguous():
                raise ValueError("pointer tables must be contiguous")
        return packed, n_local

    def run(self, x, sel, weights, packed, k, limit, *, check_bounds=True):
        """Routed experts of `rows` tokens: float32 [rows, hidden], an owned tensor.

        Same arguments and errors as the reference runner's run (moe_coop2048.py:255-305): ValueError
        for bad arguments; RuntimeError from another thread, on another stream than the construction
        stream, under graph capture, or while a call is in progress; any error after the arguments
        were accepted poisons the runner. check_bounds=True reads the device status word back (the
        reference's mandatory bounds check); False skips that host read (the kernels still skip and
        flag an out-of-range expert), which the reference does not offer.
        """
        if threading.get_ident() != self._owner_thread:
            raise RuntimeError("EvaMoERunner requires its owner thread")
        if self._failed:
            raise RuntimeError("EvaMoERunner launch failed earlier; discard this runner")
        if type(k) not in (int, float) or k not in (2, 3, 4):
            raise ValueError("EXL3 K must be 2, 3 or 4")
        if type(limit) not in (int, float) or not math.isfinite(limit) or not 0 <= limit <= 3.4028234663852886e38:
            raise ValueError("limit must be a finite nonnegative number")
        if type(check_bounds) is not bool:
            raise TypeError("check_bounds must be bool")
        if (not isinstance(x, torch.Tensor) or x.ndim != 2 or x.shape[1] != self.hidden
                or not 1 <= x.shape[0] <= self.max_rows or x.dtype not in (_F16, _BF16)):
            raise ValueError(f"x must be Half/BF16[1..{self.max_rows},{self.hidden}]")
        rows = x.shape[0]
        if (not isinstance(sel, torch.Tensor) or tuple(sel.shape) != (rows, self.topk) or sel.dtype != _I64
                or not isinstance(weights, torch.Tensor) or weights.shape != sel.shape
                or weights.dtype not in (_F16, _BF16, _F32)):
            raise ValueError(f"routes/weights require [rows,{self.topk}] Long and Half/BF16/Float")
        tables, n_local = self._tables(packed)
        for name, t in (("x", x), ("sel", sel), ("weights", weights), *(("packed", t) for t in tables)):
            _require_cuda(t, self.device, name)
        if torch.cuda.current_stream(self.device).cuda_stream != self._owner_stream:
            raise RuntimeError("EvaMoERunner requires its construction stream")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("EvaMoERunner does not support graph capture")
        if not self._lock.acquire(blocking=False):
            raise RuntimeError("EvaMoERunner is already in use")
        try:
            x, sel = x.contiguous(), sel.contiguous()
            rw = self.rw[:rows]
            # the reference rounds the routing weights to Half before the kernels (zero = inactive)
            rw.copy_(weights.to(_F16).to(_F32))
            shape = self._shape(k, limit, n_local)
            ws = self._workspace(shape)
            out = self.out[:rows]
            stream = _stream(self.device)
            if check_bounds:
                _lib.check(self.lib.eva_moe_clear_status(ws.data_ptr(), stream), "eva_moe_clear_status")
            rc = self.lib.eva_moe_experts(ctypes.byref(shape), x.data_ptr(), int(x.dtype == _BF16), rows,
                                          sel.data_ptr(), 1, rw.data_ptr(), _lib.table_array(tables), None,
                                          ws.data_ptr(), ws.numel(), out.data_ptr(), None, stream)
            _lib.check(rc, "eva_moe_experts")
            if check_bounds:
                st = ctypes.c_int32(0)
                _lib.check(self.lib.eva_moe_read_status(ws.data_ptr(), ctypes.byref(st), stream), "eva_moe_read_status")
                if st.value & _lib.STATUS_BAD_EXPERT:
                    raise ValueError("expert index outside pointer tables (or unbound pointer)")
                if st.value:
                    raise RuntimeError(f"device status {st.value:#x}")
            return out.clone()
        except BaseException:
            self._failed = True
            raise
        finally:
            self._lock.release()

    def prepare_routes(self, sel, weights, n_local, capacity=None):
        """The integer run table alone (reference `prepare_routes`), as an owned int32 tensor."""
        rows = sel.shape[0]
        capacity = self.max_rows if capacity is None else capacity
        if sel.dtype != _I64 or sel.ndim != 2 or sel.shape[1] != self.topk or not 1 <= rows <= capacity:
            raise ValueError("prepare requires Long [rows, topk] routes within capacity")
        shape = self._shape(3, 0.0, n_local)
        rw = weights.to(_F16).to(_F32).contiguous()
        runs = torch.zeros(2 + 2 * capacity * self.topk + 1, dtype=torch.int32, device=self.device)
        rc = self.lib.eva_moe_permute(ctypes.byref(shape), sel.contiguous().data_ptr(), 1, rw.data_ptr(), rows,
                                      capacity, runs.data_ptr(), None, _stream(self.device))
        _lib.check(rc, "eva_moe_permute")
        return runs


class EvaMoE:
    """MoE-layer operator: router + routed EXL3 experts + shared expert (Block.route/Block.experts).

    forward(x, out=...) issues only stream-ordered work and never synchronises the host, so it can be
    captured in a CUDA graph (torch.cuda.graph) and replayed with new inputs copied into the captured
    x; the workspace is the operator's own, so one captured graph per operator runs at a time."""

    def __init__(self, layer: ExpertLayer, max_rows: int = 64):
        if not torch.cuda.is_available() or layer.device.type != "cuda":
            raise RuntimeError("EvaMoE requires a CUDA-resident ExpertLayer; there is no CPU fallback")
        if layer.n_local != layer.cfg.n_experts:
            raise ValueError("EvaMoE needs every routed expert; use eva_b200.ep.EPMoE for an expert shard")
        self.lib = _lib.load()
        self.layer = layer
        self.cfg: MoEConfig = layer.cfg
        self.device = layer.device
        self.max_rows = max_rows
        self.shape = _lib.shape_of(self.cfg)
        n = self.lib.eva_moe_workspace_bytes(ctypes.byref(self.shape), max_rows)
        if n == 0:
            raise ValueError("unsupported MoE shape")
        self.workspace = torch.zeros(n, dtype=torch.uint8, device=self.device)
        self._tables = _lib.table_array(tuple(layer.packed.unbind(0)))
        self._packed_rows = tuple(layer.packed.unbind(0))   # keep the row views alive
        self._shared = _lib.shared_array(layer.shared.tolist()) if layer.shared is not None else None

    def _check_x(self, x):
        if (not isinstance(x, torch.Tensor) or x.device != self.device or x.dtype not in (_BF16, _F16)
                or x.shape[-1] != self.cfg.hidden):
            raise ValueError(f"x must be BF16/Half [..., {self.cfg.hidden}] on {self.device}")
        flat = x.reshape(-1, self.cfg.hidden).contiguous()
        if not 1 <= flat.shape[0] <= self.max_rows:
            raise ValueError(f"1..{self.max_rows} tokens per call")
        return flat

    def route(self, x, *, logits_out=None):
        """(weights float32 [M, topk], indices int64 [M, topk]) like Block.route."""
        flat = self._check_x(x)
        M = flat.shape[0]
        idx = torch.empty(M, self.cfg.topk, dtype=torch.int32, device=self.device)
        w = torch.empty(M, self.cfg.topk, dtype=_F32, device=self.device)
        rc = self.lib.eva_moe_route(ctypes.byref(self.shape), flat.data_ptr(), int(flat.dtype == _BF16), M,
                                    self.layer.router_w.data_ptr(), self.layer.router_b.data_ptr(),
                                    _lib.ptr(logits_out), idx.data_ptr(), w.data_ptr(), self.workspace.data_ptr(),
                                    self.workspace.numel(), _stream(self.device))
        _lib.check(rc, "eva_moe_route")
        return w, idx.to(_I64)

    def forward(self, x, *, out=None, out_f32=None, idx_out=None, w_out=None, logits_out=None):
        """Route + routed experts + shared expert; returns out (x's dtype, x's shape)."""
        flat = self._check_x(x)
        M = flat.shape[0]
        if out is None:
            out = torch.empty(M, self.cfg.hidden, dtype=_BF16, device=self.device)
        rc = self.lib.eva_moe_forward(ctypes.byref(self.shape), flat.data_ptr(), int(flat.dtype == _BF16), M,
                                      self.layer.router_w.data_ptr(), self.layer.router_b.data_ptr(), self._tables,
                                      self._shared, self.workspace.data_ptr(), self.workspace.numel(),
                                      _lib.ptr(out_f32), out.data_ptr(), _lib.ptr(logits_out), _lib.ptr(idx_out),
                                      _lib.ptr(w_out), _stream(self.device))
        _lib.check(rc, "eva_moe_forward")
        if x.dtype != _BF16:
            return out.to(x.dtype).view_as(x)
        return out.view_as(x)

    experts = forward

    def experts_given_routes(self, x, idx, w, *, out_f32=None, out=None, shared=True):
        """Experts + combine for externally computed routes (idx int32/int64 [M,k], w float32)."""
        flat = self._check_x(x)
        M = flat.shape[0]
        if out is None and out_f32 is None:
            out_f32 = torch.empty(M, self.cfg.hidden, dtype=_F32, device=self.device)
        shape = self.shape if shared else _lib.shape_of(self.cfg, shared=False)
        rc = self.lib.eva_moe_experts(ctypes.byref(shape), flat.data_ptr(), int(flat.dtype == _BF16), M,
                                      idx.contiguous().data_ptr(), int(idx.dtype == _I64),
                                      w.to(_F32).contiguous().data_ptr(), self._tables,
                                      self._shared if shared else None, self.workspace.data_ptr(),
                                      self.workspace.numel(), _lib.ptr(out_f32), _lib.ptr(out), _stream(self.device))
        _lib.check(rc, "eva_moe_experts")
        return out_f32 if out_f32 is not None else out

    def status(self) -> int:
        st = ctypes.c_int32(0)
        _lib.check(self.lib.eva_moe_read_status(self.workspace.data_ptr(), ctypes.byref(st), _stream(self.device)),
                   "eva_moe_read_status")
        return st.value

    def clear_status(self) -> None:
        _lib.check(self.lib.eva_moe_clear_status(self.workspace.data_ptr(), _stream(self.device)), "eva_moe_clear_status")
