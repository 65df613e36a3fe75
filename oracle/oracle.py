"""CPU oracle for the DeepSeek MoE hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this
module. The product (eva_b200) never imports it and has no CPU fallback.

Restated from the reference (paths within Findddx/eva):
  * routers ........ sqrtsoftplus: runtime/ds41/model.py:404-416 (Block.route).
                     softmax (DeepSeek-V2-Lite) and sigmoid + bias, group-limited (DeepSeek-V3) are
                     NOT in the reference; they follow the published DeepSeek gating, checked
                     against transformers 5.5.0's DeepSeek-V2/V3 routing functions
                     (tests/golden/make_route_pins.py).
  * run table ...... runtime/ds41/moe_coop2048.py:69-111 (reference_runs / reference_table),
                     generalised to any top-k / capacity.
  * EXL3 experts ... oracle/exl3_oracle.c (C restatement, see its header).
  * CPU baseline ... oracle/cpu_fast.c: the same layer in float32 with dequantization fused into the
                     GEMV, timed by bench.py as the CPU baseline (moe_forward_fast); checked against
                     moe_forward, never used as the parity reference.
  * RMSNorm ........ runtime/ds41/model.py:968-970 rms(x, weight, eps) (mean square in FP32).

Score functions are evaluated in float64 and rounded once to float32, so a GPU kernel that does
the same agrees bit for bit given the same float32 logits; the reference's own float32 torch ops
may differ from that by one ulp, which only matters for near-exact ties.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    srcs = [HERE / "exl3_oracle.c", HERE / "cpu_fast.c"]
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(f.stat().st_mtime for f in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        u16, u32, i32, dbl = ctypes.c_uint16, ctypes.c_uint32, ctypes.c_int, ctypes.c_double
        vp = ctypes.c_void_p
        L.eo_mul1_decode.restype = u16
        L.eo_mul1_decode.argtypes = [u32]
        L.eo_mul1_integer.restype = i32
        L.eo_mul1_integer.argtypes = [u32]
        L.eo_tile_state.restype = u32
        L.eo_tile_state.argtypes = [vp, i32, i32]
        L.eo_tile_state_fast.restype = u32
        L.eo_tile_state_fast.argtypes = [vp, i32, i32]
        L.eo_dequant.restype = None
        L.eo_dequant.argtypes = [vp, i32, i32, i32, vp]
        L.eo_f16_from_double.restype = u16
        L.eo_f16_from_double.argtypes = [dbl]
        L.eo_linear.restype = None
        L.eo_linear.argtypes = [vp, i32, i32, i32, vp, vp, vp, i32, vp]
        L.eo_act.restype = dbl
        L.eo_act.argtypes = [dbl, dbl, dbl, i32]
        L.eo_moe_forward.restype = i32
        L.eo_moe_forward.argtypes = [vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, i32, vp, i32, i32,
                                     dbl, vp, vp, i32]
        L.cf_moe_forward.restype = i32
        L.cf_moe_forward.argtypes = [vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, i32, vp, i32, i32,
                                     dbl, vp, i32]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ------------------------------------------------------------------------------------------------
# EXL3 decode


def mul1_decode(states) -> np.ndarray:
    """fp16 bit patterns of the mul1 codebook for an array of 16-bit states."""
    L = lib()
    s = np.asarray(states, dtype=np.uint32).ravel()
    return np.array([L.eo_mul1_decode(int(v)) for v in s], dtype=np.uint16)


def mul1_table() -> np.ndarray:
    """All 65536 codebook values as fp16 bit patterns."""
    return mul1_decode(np.arange(65536, dtype=np.uint32))


def tile_state(tile_words: np.ndarray, K: int, p: int, fast: bool = False) -> int:
    L = lib()
    t = np.ascontiguousarray(tile_words, dtype=np.uint32)
    return (L.eo_tile_state_fast if fast else L.eo_tile_state)(_ptr(t), K, p)


def tile_pos(p: int):
    """(k, n) of trellis position p inside a 16x16 tile."""
    lane, j = p >> 3, p & 7
    return 2 * (lane & 3) + (j & 1) + 8 * ((j >> 1) & 1), (lane >> 2) + 8 * (j >> 2)


def dequant(trellis: np.ndarray, K: int) -> np.ndarray:
    """trellis int16 [in/16, out/16, 16K] -> fp16 bit patterns [in, out]."""
    t = np.ascontiguousarray(trellis, dtype=np.int16)
    kt, nt, w = t.shape
    assert w == 16 * K
    out = np.empty((kt * 16, nt * 16), dtype=np.uint16)
    lib().eo_dequant(_ptr(t), kt * 16, nt * 16, K, _ptr(out))
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def linear(x: np.ndarray, suh: np.ndarray, svh: np.ndarray, w16: np.ndarray, round_in: bool = True) -> np.ndarray:
    """One EXL3 linear in float64: y = had(fp16(had(x * suh)) @ W') * svh."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    M, fin = x.shape
    fout = w16.shape[1]
    y = np.empty((M, fout), dtype=np.float64)
    su = np.ascontiguousarray(suh, dtype=np.uint16)
    sv = np.ascontiguousarray(svh, dtype=np.uint16)
    w = np.ascontiguousarray(w16, dtype=np.uint16)
    lib().eo_linear(_ptr(x), M, fin, fout, _ptr(su), _ptr(sv), _ptr(w), int(round_in), _ptr(y))
    return y


def hadamard128(v: np.ndarray) -> np.ndarray:
    """Blockwise natural-order Sylvester Hadamard / sqrt(128) along the last axis."""
    v = np.asarray(v, dtype=np.float64)
    shp = v.shape
    a = v.reshape(-1, shp[-1] // 128, 128).copy()
    h = 1
    while h < 128:
        a = a.reshape(a.shape[0], a.shape[1], -1, 2, h)
        x, y = a[..., 0, :].copy(), a[..., 1, :].copy()
        a[..., 0, :], a[..., 1, :] = x + y, x - y
        a = a.reshape(a.shape[0], a.shape[1], 128)
        h *= 2
    return (a / np.sqrt(128.0)).reshape(shp)


# ------------------------------------------------------------------------------------------------
# Routers (float32 outputs; scores via float64 then one rounding)


def router_logits(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """FP32 router logits x @ w.T, accumulated in float64 then rounded (model.py:404-406)."""
    return (np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64).T).astype(np.float32)


def _topk_desc(v: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest per row, descending; equal values: lower index first."""
    order = np.lexsort((np.broadcast_to(np.arange(v.shape[-1]), v.shape), -v.astype(np.float64)), axis=-1)
    return order[..., :k]


def scores(logits: np.ndarray, router: str) -> np.ndarray:
    l = np.asarray(logits, dtype=np.float32).astype(np.float64)
    if router == "sigmoid":
        return (1.0 / (1.0 + np.exp(-l))).astype(np.float32)
    if router == "softmax":
        m = l.max(axis=-1, keepdims=True)
        e = np.exp(l - m)
        return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    if router == "sqrtsoftplus":
        # torch softplus (beta 1, threshold 20), rounded to float32, then float32 sqrt
        sp = np.where(l > 20.0, l, np.log1p(np.exp(np.minimum(l, 20.0)))).astype(np.float32)
        return np.sqrt(sp.astype(np.float64)).astype(np.float32)
    raise ValueError(router)


def route(logits: np.ndarray, bias: np.ndarray, cfg) -> tuple[np.ndarray, np.ndarray]:
    """Top-k expert ids (int32 [M, k], descending by selection score) and float32 weights.

    sqrtsoftplus: model.py:404-416. sigmoid: DeepSeek-V3 noaux_tc (group score = sum of the top-2
    biased scores of a group, top `topk_group` groups kept, others -inf). softmax: DeepSeek-V2-Lite
    greedy top-k. Weights are the unbiased scores, renormalised over the selection when
    cfg.norm_topk (sum + 1e-20), times cfg.route_scale. Equal scores go to the lower expert id.
    The sigmoid and softmax forms are checked against transformers 5.5.0
    DeepseekV3MoE.route_tokens_to_experts and DeepseekV2Moe.route_tokens_to_experts ("greedy")
    by tests/golden/make_route_pins.py.
    """
    s = scores(logits, cfg.router)
    M, E = s.shape
    if cfg.router == "softmax":
        choice = np.asarray(logits, dtype=np.float32)   # softmax is monotonic in the logits
    else:
        choice = (s + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    if cfg.n_group > 1:
        g = choice.reshape(M, cfg.n_group, E // cfg.n_group)
        top2 = -np.sort(-g, axis=-1)[..., :2]
        gscore = (top2[..., 0] + top2[..., 1]).astype(np.float32)
        keep = _topk_desc(gscore, cfg.topk_group)
        mask = np.zeros((M, cfg.n_group), dtype=bool)
        np.put_along_axis(mask, keep, True, axis=-1)
        choice = np.where(np.repeat(mask, E // cfg.n_group, axis=-1), choice, -np.inf).astype(np.float32)
    idx = _topk_desc(choice, cfg.topk).astype(np.int32)
    w = np.take_along_axis(s, idx, axis=-1).astype(np.float32)
    if cfg.norm_topk:
        w = (w / (w.sum(axis=-1, keepdims=True, dtype=np.float32) + np.float32(1e-20))).astype(np.float32)
    w = (w * np.float32(cfg.route_scale)).astype(np.float32)
    return idx, w


# ------------------------------------------------------------------------------------------------
# Permutation: the reference's int32 run table (moe_coop2048.py:91-111), any top-k / capacity


RUN_ROWS = 8


def run_table(sel: np.ndarray, rw: np.ndarray | None, capacity: int) -> list[int]:
    """[n_runs, 0, run_start[S+1], order[S]] with S = capacity * topk: active slots (rw != 0)
    sorted by (expert, slot) and cut into runs of at most 8 slots of one expert; unused entries 0."""
    sel = np.asarray(sel)
    M, topk = sel.shape
    S = capacity * topk
    if rw is None:
        rw = np.ones(sel.shape, dtype=np.float32)
    active = sorted((int(sel[m, k]), m * topk + k) for m in range(M) for k in range(topk) if rw[m, k] != 0)
    runs = []
    for e, s in active:
        if not runs or runs[-1][0] != e or len(runs[-1][1]) == RUN_ROWS:
            runs.append((e, []))
        runs[-1][1].append(s)
    table = [0] * (2 + S + 1 + S)
    table[0] = len(runs)
    pos = 0
    for r, (_, slots) in enumerate(runs):
        table[2 + r] = pos
        for s in slots:
            table[2 + S + 1 + pos] = s
            pos += 1
    table[2 + len(runs)] = pos
    return table


def expert_offsets(sel: np.ndarray, rw: np.ndarray | None, n_experts: int) -> np.ndarray:
    """Exclusive prefix of active-slot counts per expert: int32 [E + 1]."""
    sel = np.asarray(sel).ravel()
    act = np.ones(sel.shape, bool) if rw is None else (np.asarray(rw).ravel() != 0)
    cnt = np.bincount(sel[act], minlength=n_experts)
    return np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)


# ------------------------------------------------------------------------------------------------
# Full MoE layer from host-resident EXL3 experts


def moe_forward(x_bits: np.ndarray, sel: np.ndarray, rw: np.ndarray, layer, threads: int = 0,
                with_shared: bool = True, x_is_f16: bool = False) -> np.ndarray:
    """Routed experts + shared expert, float32 [M, H]. `layer` is an ExpertLayer in host memory;
    x_bits are bf16 bit patterns (or fp16 with x_is_f16)."""
    cfg = layer.cfg
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, H = x.shape
    sel32 = np.ascontiguousarray(sel, dtype=np.int32)
    rw32 = np.ascontiguousarray(rw, dtype=np.float32)
    assert str(layer.packed.device) == "cpu"
    ptrs = np.ascontiguousarray(layer.packed.numpy().T, dtype=np.int64)   # [E, 9]
    sh = None
    if with_shared and layer.shared is not None:
        sh = np.ascontiguousarray(layer.shared.numpy(), dtype=np.int64)
    out = np.empty((M, H), dtype=np.float32)
    n_tab = ptrs.shape[0]
    st = lib().eo_moe_forward(_ptr(x), int(x_is_f16), M, H, cfg.inter, cfg.topk, n_tab, _ptr(sel32), _ptr(rw32),
                              _ptr(ptrs), cfg.bits, None if sh is None else _ptr(sh),
                              cfg.shared_inter if sh is not None else 0, cfg.shared_bits,
                              float(cfg.swiglu_limit), _ptr(out), None, int(threads))
    if st:
        raise RuntimeError(f"oracle moe_forward status {st}")
    return out


def moe_forward_fast(x_bits: np.ndarray, sel: np.ndarray, rw: np.ndarray, layer, threads: int = 0,
                     with_shared: bool = True, x_is_f16: bool = False) -> np.ndarray:
    """moe_forward in float32 with the dequantization fused into the GEMV (cpu_fast.c): the CPU
    baseline bench.py times. Same arguments and result as moe_forward."""
    cfg = layer.cfg
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, H = x.shape
    sel32 = np.ascontiguousarray(sel, dtype=np.int32)
    rw32 = np.ascontiguousarray(rw, dtype=np.float32)
    assert str(layer.packed.device) == "cpu"
    ptrs = np.ascontiguousarray(layer.packed.numpy().T, dtype=np.int64)   # [E, 9]
    sh = None
    if with_shared and layer.shared is not None:
        sh = np.ascontiguousarray(layer.shared.numpy(), dtype=np.int64)
    out = np.empty((M, H), dtype=np.float32)
    st = lib().cf_moe_forward(_ptr(x), int(x_is_f16), M, H, cfg.inter, cfg.topk, ptrs.shape[0], _ptr(sel32),
                              _ptr(rw32), _ptr(ptrs), cfg.bits, None if sh is None else _ptr(sh),
                              cfg.shared_inter if sh is not None else 0, cfg.shared_bits,
                              float(cfg.swiglu_limit), _ptr(out), int(threads))
    if st:
        raise RuntimeError(f"cpu_fast moe_forward status {st}")
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rms(x, weight, eps) = weight * x * rsqrt(mean(x^2) + eps), evaluated in float64 (float32 result)."""
    x64 = np.asarray(x, np.float64)
    inv = 1.0 / np.sqrt((x64 * x64).mean(axis=-1, keepdims=True) + eps)
    return (np.asarray(w, np.float64) * x64 * inv).astype(np.float32)


def layer_forward(x_bf16: np.ndarray, layer, threads: int = 0):
    """Router (FP32 logits) + routed experts + shared: returns (out f32, idx, w, logits)."""
    cfg = layer.cfg
    x = bf16_to_f32(x_bf16)
    logits = router_logits(x, layer.router_w.numpy())
    idx, w = route(logits, layer.router_b.numpy(), cfg)
    return moe_forward(x_bf16, idx, w, layer, threads), idx, w, logits
