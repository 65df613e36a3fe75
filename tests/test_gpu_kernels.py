"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle and the reference's golden
vectors. Needs a B200: run with -m gpu.

Bars: EXL3 dequant, router indices (given identical FP32 logits) and the permutation table are
bit-exact; MoE outputs are within max|err| / max|ref| <= 2e-2 and cosine >= 0.9999 (the north
star's BF16 bar), and in practice ~1e-3 for the FP32 output.
"""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from eva_b200 import _lib
from eva_b200 import config as C
from eva_b200.experts import make_layer

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"

REL_TOL = 2e-2
COS_TOL = 0.9999


def close(out, ref, rel=REL_TOL, cos=COS_TOL):
    out = np.asarray(out, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    c = float(out @ ref / (np.linalg.norm(out) * np.linalg.norm(ref) + 1e-300))
    assert err <= rel and c >= cos, f"max-rel-err {err:.3e} cosine {c:.7f}"
    return err, c


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def stream():
    return torch.cuda.current_stream().cuda_stream


# ------------------------------------------------------------------------------------------------
# EXL3 dequant: bit-exact


@pytest.mark.parametrize("K", [2, 3, 4])
@pytest.mark.parametrize("fin,fout", [(128, 256), (2048, 1408)])
def test_dequant_bit_exact(lib, oracle, K, fin, fout):
    g = torch.Generator().manual_seed(K * 7 + fin)
    tr = torch.randint(-32768, 32768, (fin // 16, fout // 16, 16 * K), generator=g, dtype=torch.int32).to(torch.int16)
    ref = oracle.dequant(tr.numpy(), K)
    w = torch.empty(fin, fout, dtype=torch.int16, device=DEV)
    trd = tr.to(DEV)
    _lib.check(lib.eva_exl3_dequant(trd.data_ptr(), fin, fout, K, w.data_ptr(), stream()), "dequant")
    torch.cuda.synchronize()
    assert np.array_equal(w.cpu().numpy().view(np.uint16), ref)


# ------------------------------------------------------------------------------------------------
# Router


def _topk_gpu(lib, cfg, logits, bias):
    sh = _lib.shape_of(cfg)
    M = logits.shape[0]
    ld = torch.tensor(logits, device=DEV)
    bd = torch.tensor(bias, device=DEV)
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=DEV)
    w = torch.empty(M, cfg.topk, dtype=torch.float32, device=DEV)
    _lib.check(lib.eva_moe_topk(ctypes.byref(sh), ld.data_ptr(), M, bd.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                stream()), "topk")
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("cfg", [C.V2_LITE, C.V3, C.REF_NATIVE], ids=lambda c: c.name)
def test_topk_bit_exact_given_logits(lib, oracle, cfg):
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal((97, cfg.n_experts)) * 1.7).astype(np.float32)
    bias = (rng.standard_normal(cfg.n_experts) * 0.01).astype(np.float32)
    if cfg.router == "softmax":
        bias[:] = 0
    idx, w = _topk_gpu(lib, cfg, logits, bias)
    ridx, rw = oracle.route(logits, bias, cfg)
    assert np.array_equal(idx, ridx)
    assert np.allclose(w, rw, rtol=2e-6, atol=1e-7)


def test_topk_matches_reference_block_route(lib):
    """Identical FP32 logits from the reference's Block.route fixture -> identical indices."""
    g = np.load(GOLDEN / "route_sqrtsoftplus.npz")
    idx, w = _topk_gpu(lib, C.REF_NATIVE, g["logits"], g["gate_b"])
    assert np.array_equal(idx.astype(np.int64), g["indices"])
    assert np.allclose(w, g["weights"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("fixture,cfg", [("route_v3_sigmoid.npz", C.V3), ("route_v2lite_softmax.npz", C.V2_LITE)],
                         ids=["v3", "v2-lite"])
def test_topk_matches_transformers_gating(lib, fixture, cfg):
    """FP32 logits routed by transformers' DeepSeek-V3 / V2 gating (make_route_pins.py) -> the same
    expert sets; compared in ascending expert order because transformers leaves the top-k unsorted."""
    g = np.load(GOLDEN / fixture)
    bias = g["bias"] if "bias" in g.files else np.zeros(cfg.n_experts, np.float32)
    idx, w = _topk_gpu(lib, cfg, g["logits"], bias)
    order = np.argsort(idx, axis=-1, kind="stable")
    assert np.array_equal(np.take_along_axis(idx, order, -1).astype(np.int64), g["indices"])
    assert np.allclose(np.take_along_axis(w, order, -1), g["weights"], rtol=2e-6, atol=1e-7)


def test_group_limited_ties_and_masking(lib, oracle):
    cfg = C.V3
    logits = np.zeros((4, cfg.n_experts), np.float32)       # all ties: lowest indices / groups win
    bias = np.zeros(cfg.n_experts, np.float32)
    idx, _ = _topk_gpu(lib, cfg, logits, bias)
    ridx, _ = oracle.route(logits, bias, cfg)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(idx[0], np.arange(8))


# bf16 activations at every size; fp16 ones at one size per kernel path (GEMV, SIMT GEMM)
ROUTER_CASES = [(M, torch.bfloat16) for M in (1, 5, 32, 33, 128, 200, 1000)] + [(5, torch.float16), (200, torch.float16)]


@pytest.mark.parametrize("M,x_dtype", ROUTER_CASES,
                         ids=[f"{m}-{'bf16' if d == torch.bfloat16 else 'f16'}" for m, d in ROUTER_CASES])
@pytest.mark.parametrize("cfg", [C.V3, C.V2_LITE], ids=lambda c: c.name)
def test_router_logits_and_indices(lib, oracle, cfg, M, x_dtype):
    """M <= 32: k-sliced GEMV; larger bf16 batches: the tensor-core GEMM (three bf16 parts of each
    FP32 weight, k slices summed by the top-k kernel); larger fp16 batches: the SIMT GEMM.
    V2-Lite at 128 tokens is the router half of the FP32 CPU case: dense N(0, 0.02) router weights
    from seed 0, N(0, 1) hidden states, softmax top-6."""
    layer = make_layer(cfg.with_(n_experts=cfg.n_experts), "cpu", seed=0, n_fill=0)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(M, cfg.hidden, generator=g).to(torch.bfloat16).to(x_dtype)
    xd = x.to(DEV)
    W = layer.router_w.to(DEV)
    b = layer.router_b.to(DEV)
    sh = _lib.shape_of(cfg)
    ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(sh), M), dtype=torch.uint8, device=DEV)
    logits = torch.empty(M, cfg.n_experts, device=DEV)
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=DEV)
    w = torch.empty(M, cfg.topk, device=DEV)
    _lib.check(lib.eva_moe_route(ctypes.byref(sh), xd.data_ptr(), int(x_dtype == torch.bfloat16), M, W.data_ptr(),
                                 b.data_ptr(), logits.data_ptr(), idx.data_ptr(), w.data_ptr(), ws.data_ptr(), ws.numel(),
                                 stream()), "route")
    torch.cuda.synchronize()
    ref_logits = oracle.router_logits(x.float().numpy(), layer.router_w.numpy())
    assert np.allclose(logits.cpu().numpy(), ref_logits, rtol=1e-4, atol=1e-4)
    # FP32-level accuracy: error within 2^-16 of the dot product's absolute sum (a weight rounded to
    # one bf16 part would be off by up to 2^-9 of it)
    abs_sum = np.abs(x.float().numpy().astype(np.float64)) @ np.abs(layer.router_w.numpy().astype(np.float64)).T
    assert np.all(np.abs(logits.cpu().numpy() - ref_logits) <= abs_sum * 2.0**-16 + 1e-30)
    # given the kernel's own logits the selection is bit-exact
    ridx, rw = oracle.route(logits.cpu().numpy(), layer.router_b.numpy(), cfg)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    # end-to-end agreement with logits from the FP64 oracle
    e2e, _ = oracle.route(ref_logits, layer.router_b.numpy(), cfg)
    agree = np.mean(np.sort(e2e, -1) == np.sort(idx.cpu().numpy(), -1))
    assert agree >= 0.99


# ------------------------------------------------------------------------------------------------
# Permutation: bit-exact run table


def _permute_gpu(lib, topk, n_local, sel, rw, capacity, with_ws=False):
    cfg = C.MoEConfig("p", hidden=256, inter=128, n_experts=n_local, topk=topk, router="softmax")
    sh = _lib.shape_of(cfg, shared=False)
    seld = torch.tensor(np.asarray(sel, dtype=np.int64), device=DEV)
    rwd = torch.tensor(np.asarray(rw, dtype=np.float32), device=DEV)
    runs = torch.full((2 + 2 * capacity * topk + 1,), -7, dtype=torch.int32, device=DEV)
    est = torch.empty(n_local + 1, dtype=torch.int32, device=DEV)
    if with_ws:
        ws = torch.full((lib.eva_moe_workspace_bytes(ctypes.byref(sh), max(len(sel), 1)),), 0x5A, dtype=torch.uint8,
                        device=DEV)
        _lib.check(lib.eva_moe_permute_ws(ctypes.byref(sh), seld.data_ptr(), 1, rwd.data_ptr(), len(sel), capacity,
                                          runs.data_ptr(), est.data_ptr(), ws.data_ptr(), ws.numel(), stream()),
                   "permute_ws")
    else:
        _lib.check(lib.eva_moe_permute(ctypes.byref(sh), seld.data_ptr(), 1, rwd.data_ptr(), len(sel), capacity,
                                       runs.data_ptr(), est.data_ptr(), stream()), "permute")
    torch.cuda.synchronize()
    return runs.cpu().tolist(), est.cpu().numpy()


def test_permute_matches_reference_tables(lib):
    data = json.loads((GOLDEN / "run_tables.json").read_text())
    n = 0
    for c in data["cases"]:
        if c["table"] is None:
            continue
        runs, _ = _permute_gpu(lib, 6, 384, c["indices"], c["weights"], c["capacity"])
        assert runs == c["table"], c["module"]
        n += 1
    assert n >= 10


@pytest.mark.parametrize("M,topk,E,zero", [(1, 8, 256, 0.0), (64, 8, 256, 0.1), (300, 8, 16, 0.0),
                                           (4096, 8, 256, 0.02), (7, 6, 1024, 0.3)])
def test_permute_matches_oracle(lib, oracle, M, topk, E, zero):
    rng = np.random.default_rng(M + E)
    sel = np.stack([rng.choice(E, topk, replace=False) for _ in range(M)])
    rw = rng.random((M, topk)).astype(np.float32) + 0.01
    rw[rng.random((M, topk)) < zero] = 0
    runs, est = _permute_gpu(lib, topk, E, sel, rw, M)
    assert runs == oracle.run_table(sel, rw, M)
    assert np.array_equal(est, oracle.expert_offsets(sel, rw, E))


@pytest.mark.parametrize("M,topk,E,zero,cap_extra", [(257, 8, 256, 0.0, 0), (300, 8, 16, 0.05, 7), (1000, 6, 64, 0.2, 0),
                                                     (4096, 8, 256, 0.02, 0), (5000, 8, 1024, 0.0, 33),
                                                     (640, 12, 32, 0.5, 0)])
def test_permute_multi_cta_matches_oracle(lib, oracle, M, topk, E, zero, cap_extra):
    """Batches above 256 tokens with a workspace take the three-launch form (per-chunk counts, one
    scan, per-chunk stable scatter): the same table as the one-CTA kernel and the oracle, bit for bit,
    including ragged last chunks, inactive slots, spare capacity and top-k above 8 (two sub-chunks)."""
    rng = np.random.default_rng(M + E + topk)
    sel = np.stack([rng.choice(E, topk, replace=False) for _ in range(M)])
    rw = rng.random((M, topk)).astype(np.float32) + 0.01
    rw[rng.random((M, topk)) < zero] = 0
    cap = M + cap_extra
    runs, est = _permute_gpu(lib, topk, E, sel, rw, cap, with_ws=True)
    runs1, est1 = _permute_gpu(lib, topk, E, sel, rw, cap)
    assert runs == runs1 and np.array_equal(est, est1)
    assert runs == oracle.run_table(sel, rw, cap)
    assert np.array_equal(est, oracle.expert_offsets(sel, rw, E))


# ------------------------------------------------------------------------------------------------
# Fused experts vs the oracle

SMALL = C.MoEConfig("small", hidden=512, inter=256, n_experts=16, topk=4, router="sigmoid", n_group=4,
                    topk_group=2, route_scale=2.5, norm_topk=True, shared_inter=384, bits=3, shared_bits=4)


def _routes(cfg, M, rng, dup_heavy=False, zero=0.0):
    pool = 3 if dup_heavy else cfg.n_experts
    sel = []
    for _ in range(M):
        base = rng.choice(max(pool, cfg.topk), cfg.topk, replace=False)
        sel.append(base)
    sel = np.array(sel, dtype=np.int64)
    rw = (rng.random((M, cfg.topk)) + 0.1).astype(np.float32)
    rw[rng.random((M, cfg.topk)) < zero] = 0
    return sel, rw


def _run_experts(lib, cfg, layer_d, x, sel, rw, shared=True, limit=None, act_routed=0):
    sh = _lib.shape_of(cfg, shared=shared, limit=limit, act_routed=act_routed)
    M = x.shape[0]
    ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(sh), M), dtype=torch.uint8, device=DEV)
    out = torch.full((M, cfg.hidden), float("nan"), device=DEV)
    outb = torch.empty(M, cfg.hidden, dtype=torch.bfloat16, device=DEV)
    tables = _lib.table_array(tuple(layer_d.packed.unbind(0)))
    shared_a = _lib.shared_array(layer_d.shared.tolist()) if shared else None
    seld = torch.tensor(sel, device=DEV)
    rwd = torch.tensor(rw, device=DEV)
    xd = x.to(DEV)
    rc = lib.eva_moe_experts(ctypes.byref(sh), xd.data_ptr(), 1, M, seld.data_ptr(), 1, rwd.data_ptr(), tables,
                             shared_a, ws.data_ptr(), ws.numel(), out.data_ptr(), outb.data_ptr(), stream())
    _lib.check(rc, "experts")
    st = ctypes.c_int32(0)
    _lib.check(lib.eva_moe_read_status(ws.data_ptr(), ctypes.byref(st), stream()), "status")
    return out.cpu().numpy(), outb.float().cpu().numpy(), st.value


@pytest.mark.parametrize("bits,shared_bits", [(2, 4), (3, 4), (4, 4), (2, 2), (3, 3)])
@pytest.mark.parametrize("M", [1, 3, 8, 13])
def test_experts_small(lib, oracle, bits, shared_bits, M):
    """Routed and shared trellis widths: the ring's stages are sized for the widest of the launch
    (5 stages when both are K <= 3, 4 with a K = 4 projection)."""
    cfg = SMALL.with_(bits=bits, shared_bits=shared_bits)
    layer = make_layer(cfg, "cpu", seed=bits)
    layer_d = layer.to(DEV)
    rng = np.random.default_rng(M * 10 + bits)
    sel, rw = _routes(cfg, M, rng)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
    out, outb, st = _run_experts(lib, cfg, layer_d, x, sel, rw)
    assert st == 0
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rw, layer)
    err, _ = close(out, ref, rel=3e-3, cos=0.99999)
    close(outb, ref)


def test_experts_duplicates_inactive_and_no_shared(lib, oracle):
    cfg = SMALL
    layer = make_layer(cfg, "cpu", seed=9)
    layer_d = layer.to(DEV)
    rng = np.random.default_rng(2)
    M = 37                                   # runs longer than 8 rows (3 hot experts), ragged tail
    sel, rw = _routes(cfg, M, rng, dup_heavy=True, zero=0.2)
    rw[5, :] = 0                             # a token with no active slot
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    for shared in (True, False):
        out, _, st = _run_experts(lib, cfg, layer_d, x, sel, rw, shared=shared)
        assert st == 0
        ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rw, layer, with_shared=shared)
        close(out, ref, rel=3e-3, cos=0.99999)
        if not shared:
            assert np.all(out[5] == 0)


def test_experts_swiglu_limit_modes(lib, oracle):
    cfg = SMALL.with_(swiglu_limit=0.5)      # small limit so the clamps are exercised
    layer = make_layer(cfg, "cpu", seed=11, svh_scale=0.2)
    layer_d = layer.to(DEV)
    rng = np.random.default_rng(7)
    sel, rw = _routes(cfg, 6, rng)
    x = torch.randn(6, cfg.hidden, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    out, _, _ = _run_experts(lib, cfg, layer_d, x, sel, rw)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rw, layer)
    close(out, ref, rel=3e-3, cos=0.99999)


def test_experts_bad_expert_flags_status(lib, oracle):
    cfg = SMALL
    layer = make_layer(cfg, "cpu", seed=3)
    layer_d = layer.to(DEV)
    rng = np.random.default_rng(1)
    sel, rw = _routes(cfg, 4, rng)
    sel[1, 2] = cfg.n_experts + 5            # out of range: flagged, treated as inactive
    x = torch.randn(4, cfg.hidden, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    out, _, st = _run_experts(lib, cfg, layer_d, x, sel, rw)
    assert st & _lib.STATUS_BAD_EXPERT
    rw2 = rw.copy()
    rw2[1, 2] = 0
    sel2 = sel.copy()
    sel2[1, 2] = 0
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel2, rw2, layer)
    close(out, ref, rel=3e-3, cos=0.99999)


@pytest.mark.parametrize("cfg,M", [(C.V2_LITE, 4), (C.V3, 2), (C.REF_NATIVE, 3)], ids=lambda v: getattr(v, "name", str(v)))
def test_layer_forward_full_shapes(lib, oracle, cfg, M):
    """Router + experts + shared at the BASELINE shapes against the oracle (its own routing)."""
    from eva_b200.runner import EvaMoE
    layer_d = make_layer(cfg, DEV, seed=0)      # GB-sized: generated on the device
    layer = layer_d.host_copy()
    moe = EvaMoE(layer_d, max_rows=max(M, 8))
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    logits = torch.empty(M, cfg.n_experts, device=DEV)
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=DEV)
    w = torch.empty(M, cfg.topk, device=DEV)
    out32 = torch.empty(M, cfg.hidden, device=DEV)
    y = moe.forward(x.to(DEV), out_f32=out32, idx_out=idx, w_out=w, logits_out=logits)
    torch.cuda.synchronize()
    assert moe.status() == 0
    # oracle on the kernel's own routing (selection is bit-exact given the logits)
    ridx, rw = oracle.route(logits.cpu().numpy(), layer.router_b.numpy(), cfg)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), ridx, rw, layer)
    close(out32.cpu().numpy(), ref, rel=3e-3, cos=0.99999)
    close(y.float().cpu().numpy(), ref)


def test_runner_dropin_matches_oracle(oracle):
    """EvaMoERunner.run with the reference runner's arguments (Half x, Long routes, nine tables)."""
    from eva_b200.runner import EvaMoERunner
    cfg = C.MoEConfig("rn", hidden=1024, inter=512, n_experts=24, topk=6, router="sqrtsoftplus", bits=3,
                      swiglu_limit=10.0)
    layer = make_layer(cfg, "cpu", seed=5)
    layer_d = layer.to(DEV)
    runner = EvaMoERunner(DEV, topk=6, hidden=1024, inter=512, max_rows=16, n_experts=24)
    rng = np.random.default_rng(3)
    sel, rw = _routes(cfg, 9, rng)
    x = torch.randn(9, 1024, generator=torch.Generator().manual_seed(2)).to(torch.float16)
    y = runner.run(x.to(DEV), torch.tensor(sel, device=DEV), torch.tensor(rw, device=DEV).half(),
                   tuple(layer_d.packed.unbind(0)), 3, 10.0)
    rwh = torch.tensor(rw).half().float().numpy()
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rwh, layer, with_shared=False,
                             x_is_f16=True)
    close(y.cpu().numpy(), ref, rel=3e-3, cos=0.99999)
    # the table view equals the reference layout
    table = runner.prepare_routes(torch.tensor(sel, device=DEV), torch.tensor(rwh, device=DEV), 24, capacity=16)
    assert table.cpu().tolist() == oracle.run_table(sel, rwh, 16)
    bad = sel.copy()
    bad[0, 0] = 99
    with pytest.raises(ValueError):
        runner.run(x.to(DEV), torch.tensor(bad, device=DEV), torch.tensor(rw, device=DEV),
                   tuple(layer_d.packed.unbind(0)), 3, 10.0)
