"""ctypes binding of libeva_moe.so (the C ABI declared in include/eva_moe.h).

There is no fallback: if the library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

from .config import MoEConfig

LIB_PATH = Path(__file__).resolve().parent / "libeva_moe.so"

EVA_OK, EVA_ERR_INVALID, EVA_ERR_CUDA, EVA_ERR_WORKSPACE = 0, 1, 2, 3
STATUS_BAD_EXPERT, STATUS_TIMEOUT, STATUS_CAPACITY = 1, 2, 4
ACT_CLAMP_AFTER, ACT_CLAMP_BEFORE = 0, 1

# every symbol include/eva_moe.h declares
EXPORTS = ("eva_moe_workspace_bytes", "eva_moe_clear_status", "eva_moe_read_status", "eva_moe_route",
           "eva_moe_topk", "eva_moe_permute", "eva_moe_permute_ws", "eva_moe_experts", "eva_moe_forward", "eva_exl3_dequant",
           "eva_moe_arch", "eva_moe_experts_noalloc", "eva_moe_experts_decode", "eva_moe_experts_prefill",
           "eva_ep_dispatch", "eva_ep_combine", "eva_ep_arena_layout", "eva_peer_alloc", "eva_peer_open",
           "eva_peer_close", "eva_peer_free", "eva_ep_dispatch_peers", "eva_ep_wait_rows", "eva_ep_signal_partials",
           "eva_ep_combine_peers", "eva_rmsnorm_residual", "eva_moe_experts_window", "eva_decode_microbench",
           "eva_tc_selftest", "eva_pool_plan", "eva_pool_copy", "eva_host_mapped")
EP_MAX_WORLD = 32
NOALLOC_SCRATCH_BYTES = 16 << 20


class EvaMoeShape(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("n_experts", ctypes.c_int32),
                ("topk", ctypes.c_int32), ("bits", ctypes.c_int32), ("shared_inter", ctypes.c_int32),
                ("shared_bits", ctypes.c_int32), ("router", ctypes.c_int32), ("n_group", ctypes.c_int32),
                ("topk_group", ctypes.c_int32), ("norm_topk", ctypes.c_int32), ("act_routed", ctypes.c_int32),
                ("act_shared", ctypes.c_int32), ("route_scale", ctypes.c_float), ("swiglu_limit", ctypes.c_float)]


def shape_of(cfg: MoEConfig, *, shared: bool = True, bits: int | None = None, limit: float | None = None,
             act_routed: int = ACT_CLAMP_AFTER, act_shared: int = ACT_CLAMP_BEFORE,
             n_experts: int | None = None) -> EvaMoeShape:
    return EvaMoeShape(cfg.hidden, cfg.inter, cfg.n_experts if n_experts is None else n_experts, cfg.topk,
                       cfg.bits if bits is None else bits, cfg.shared_inter if shared else 0, cfg.shared_bits,
                       cfg.router_code, cfg.n_group, cfg.topk_group, int(cfg.norm_topk), act_routed, act_shared,
                       float(cfg.route_scale), float(cfg.swiglu_limit if limit is None else limit))


class EvaExpertPool(ctypes.Structure):
    _fields_ = [("n_slots", ctypes.c_int32), ("reserved", ctypes.c_int32), ("record_bytes", ctypes.c_int64),
                ("slots", ctypes.c_void_p), ("owner", ctypes.c_void_p), ("stamp", ctypes.c_void_p),
                ("state", ctypes.c_void_p)]


class EvaPoolLayer(ctypes.Structure):
    _fields_ = [("layer", ctypes.c_int32), ("n_local", ctypes.c_int32), ("host_records", ctypes.c_void_p),
                ("row_off", ctypes.c_int64 * 9), ("slot_of", ctypes.c_void_p), ("last_needed", ctypes.c_void_p),
                ("table", ctypes.c_void_p)]


class EvaEpPeers(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("H", ctypes.c_int32), ("topk", ctypes.c_int32),
                ("n_experts", ctypes.c_int32), ("segment_rows", ctypes.c_int32), ("x_elem_bytes", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("off_x", ctypes.c_uint64), ("off_sel", ctypes.c_uint64),
                ("off_rw", ctypes.c_uint64), ("off_part", ctypes.c_uint64), ("bytes", ctypes.c_uint64),
                ("arena", ctypes.c_void_p * EP_MAX_WORLD), ("owner", ctypes.c_void_p), ("local_id", ctypes.c_void_p)]


_lib = None


def load(build_if_missing: bool = True):
    """Load libeva_moe.so (building it with nvcc first when it is missing and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() and build_if_missing and not os.environ.get("EVA_NO_BUILD"):
        from .build import build
        build()
    if not LIB_PATH.exists():
        raise RuntimeError(f"libeva_moe.so not found at {LIB_PATH}; run `python -m eva_b200.build`")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, i32, sz, P = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t, ctypes.POINTER
    shp = P(EvaMoeShape)
    L.eva_moe_workspace_bytes.restype = sz
    L.eva_moe_workspace_bytes.argtypes = [shp, i32]
    L.eva_moe_clear_status.restype = ctypes.c_int
    L.eva_moe_clear_status.argtypes = [vp, vp]
    L.eva_moe_read_status.restype = ctypes.c_int
    L.eva_moe_read_status.argtypes = [vp, P(i32), vp]
    L.eva_moe_route.restype = ctypes.c_int
    L.eva_moe_route.argtypes = [shp, vp, i32, i32, vp, vp, vp, vp, vp, vp, sz, vp]
    L.eva_moe_topk.restype = ctypes.c_int
    L.eva_moe_topk.argtypes = [shp, vp, i32, vp, vp, vp, vp]
    L.eva_moe_permute.restype = ctypes.c_int
    L.eva_moe_permute.argtypes = [shp, vp, i32, vp, i32, i32, vp, vp, vp]
    L.eva_moe_permute_ws.restype = ctypes.c_int
    L.eva_moe_permute_ws.argtypes = [shp, vp, i32, vp, i32, i32, vp, vp, vp, sz, vp]
    L.eva_moe_experts.restype = ctypes.c_int
    L.eva_moe_experts.argtypes = [shp, vp, i32, i32, vp, i32, vp, P(vp), P(ctypes.c_int64), vp, sz, vp, vp, vp]
    for name in ("eva_moe_experts_decode", "eva_moe_experts_prefill"):
        fn = getattr(L, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [shp, vp, i32, i32, vp, i32, vp, P(vp), P(ctypes.c_int64), vp, sz, vp, vp, vp]
    L.eva_moe_forward.restype = ctypes.c_int
    L.eva_moe_forward.argtypes = [shp, vp, i32, i32, vp, vp, P(vp), P(ctypes.c_int64), vp, sz, vp, vp,
                                  vp, vp, vp, vp]
    L.eva_exl3_dequant.restype = ctypes.c_int
    L.eva_exl3_dequant.argtypes = [vp, i32, i32, i32, vp, vp]
    L.eva_moe_experts_noalloc.restype = ctypes.c_int
    L.eva_moe_experts_noalloc.argtypes = [shp, vp, i32, i32, vp, i32, vp, P(vp), P(ctypes.c_int64), vp, vp, vp, vp]
    L.eva_ep_dispatch.restype = ctypes.c_int
    L.eva_ep_dispatch.argtypes = [i32, i32, i32, vp, i32, i32, vp, vp, i32, vp, vp, i32, i32, vp, vp, vp, vp, vp, vp, vp]
    L.eva_ep_combine.restype = ctypes.c_int
    L.eva_ep_combine.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, vp]
    pp = P(EvaEpPeers)
    for name, args in (("eva_ep_arena_layout", [pp]), ("eva_peer_alloc", [sz, P(vp), vp]), ("eva_peer_open", [vp, P(vp)]),
                       ("eva_peer_close", [vp]), ("eva_peer_free", [vp]),
                       ("eva_ep_dispatch_peers", [pp, vp, i32, vp, vp, i32, vp, vp, vp, vp]),
                       ("eva_ep_wait_rows", [pp, vp, vp]), ("eva_ep_signal_partials", [pp, vp]),
                       ("eva_ep_combine_peers", [pp, i32, vp, vp, vp, vp, vp, vp])):
        fn = getattr(L, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args
    L.eva_moe_experts_window.restype = ctypes.c_int
    L.eva_moe_experts_window.argtypes = [shp, vp, i32, i32, vp, i32, vp, P(vp), P(ctypes.c_int64), i32, i32, vp, sz,
                                         vp, vp, vp]
    L.eva_rmsnorm_residual.restype = ctypes.c_int
    L.eva_rmsnorm_residual.argtypes = [i32, i32, vp, vp, vp, i32, ctypes.c_float, vp, vp]
    L.eva_decode_microbench.restype = ctypes.c_int
    L.eva_decode_microbench.argtypes = [i32, i32, i32, P(ctypes.c_double), vp]
    L.eva_tc_selftest.restype = ctypes.c_int
    L.eva_tc_selftest.argtypes = [i32, vp, vp, vp, vp, vp]
    L.eva_pool_plan.restype = ctypes.c_int
    L.eva_pool_plan.argtypes = [P(EvaExpertPool), vp, i32, vp, i32, vp, i32, i32, i32, vp, vp, vp, vp]
    L.eva_pool_copy.restype = ctypes.c_int
    L.eva_pool_copy.argtypes = [P(EvaExpertPool), vp, i32, vp, vp]
    L.eva_host_mapped.restype = ctypes.c_int
    L.eva_host_mapped.argtypes = [vp]
    L.eva_moe_arch.restype = i32
    L.eva_moe_arch.argtypes = []
    _lib = L
    return L


def check(rc: int, what: str) -> None:
    if rc == EVA_OK:
        return
    if rc == EVA_ERR_INVALID:
        raise ValueError(f"{what}: invalid argument (shape, pointer, alignment or unsupported K)")
    if rc == EVA_ERR_WORKSPACE:
        raise ValueError(f"{what}: workspace too small")
    raise RuntimeError(f"{what}: CUDA launch failed (rc={rc})")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def table_array(tables) -> ctypes.Array:
    arr = (ctypes.c_void_p * 9)()
    for i, t in enumerate(tables):
        arr[i] = t.data_ptr() if hasattr(t, "data_ptr") else int(t)
    return arr


def shared_array(addrs) -> ctypes.Array | None:
    if addrs is None:
        return None
    arr = (ctypes.c_int64 * 9)()
    for i, a in enumerate(addrs):
        arr[i] = int(a)
    return arr
