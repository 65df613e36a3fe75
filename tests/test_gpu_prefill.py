"""The tensor-core (tcgen05) prefill path of the fused experts against the CPU oracle and against the
register-decode kernel on the same inputs. Needs a B200: -m gpu."""
import ctypes

import numpy as np
import pytest
import torch

from eva_b200 import _lib
from eva_b200 import config as C
from eva_b200.experts import make_layer

pytestmark = pytest.mark.gpu
DEV = "cuda"

SMALL = C.MoEConfig("small", hidden=512, inter=256, n_experts=16, topk=4, router="sigmoid", n_group=4,
                    topk_group=2, route_scale=2.5, norm_topk=True, shared_inter=384, bits=3, shared_bits=4)


def close(out, ref, rel, cos):
    out = np.asarray(out, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    c = float(out @ ref / (np.linalg.norm(out) * np.linalg.norm(ref)))
    assert err <= rel and c >= cos, f"max-rel-err {err:.3e} cosine {c:.7f}"
    return err


def run(lib, fn, cfg, layer_d, x, sel, rw, shared=True):
    sh = _lib.shape_of(cfg, shared=shared)
    M = x.shape[0]
    ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(sh), M), dtype=torch.uint8, device=DEV)
    out = torch.full((M, cfg.hidden), float("nan"), device=DEV)
    tables = _lib.table_array(tuple(layer_d.packed.unbind(0)))
    shared_a = _lib.shared_array(layer_d.shared.tolist()) if shared else None
    seld = torch.as_tensor(sel, device=DEV)
    rwd = torch.as_tensor(rw, device=DEV)
    rc = getattr(lib, fn)(ctypes.byref(sh), x.data_ptr(), int(x.dtype == torch.bfloat16), M, seld.data_ptr(),
                          int(seld.dtype == torch.int64), rwd.data_ptr(), tables, shared_a, ws.data_ptr(), ws.numel(),
                          out.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, fn)
    st = ctypes.c_int32(0)
    _lib.check(lib.eva_moe_read_status(ws.data_ptr(), ctypes.byref(st), torch.cuda.current_stream().cuda_stream), "st")
    assert st.value == 0
    return out.cpu().numpy()


def routes(cfg, M, rng, skew=False, zero=0.0):
    if skew:   # a few hot experts with many rows: multi-tile experts and many small ones
        p = 1.0 / np.arange(1, cfg.n_experts + 1) ** 1.1
        p /= p.sum()
        sel = np.stack([rng.choice(cfg.n_experts, cfg.topk, replace=False, p=p) for _ in range(M)])
    else:
        sel = np.stack([rng.choice(cfg.n_experts, cfg.topk, replace=False) for _ in range(M)])
    rw = (rng.random((M, cfg.topk)) + 0.1).astype(np.float32)
    rw[rng.random((M, cfg.topk)) < zero] = 0
    return sel.astype(np.int64), rw


@pytest.mark.parametrize("bits,M,skew", [(3, 200, False), (4, 300, True), (2, 130, True), (3, 40, False)])
def test_prefill_small_vs_oracle(oracle, bits, M, skew):
    lib = _lib.load()
    cfg = SMALL.with_(bits=bits)
    layer = make_layer(cfg, "cpu", seed=bits)
    layer_d = layer.to(DEV)
    rng = np.random.default_rng(M)
    sel, rw = routes(cfg, M, rng, skew=skew, zero=0.05)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
    out = run(lib, "eva_moe_experts_prefill", cfg, layer_d, x.to(DEV), sel, rw)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rw, layer)
    close(out, ref, 3e-3, 0.99999)


@pytest.mark.parametrize("cfg,M", [(C.V2_LITE, 512), (C.V3, 256)], ids=lambda v: getattr(v, "name", str(v)))
def test_prefill_matches_decode_kernel(oracle, cfg, M):
    lib = _lib.load()
    layer_d = make_layer(cfg, DEV, seed=1)
    rng = np.random.default_rng(1)
    sel, rw = routes(cfg, M, rng, skew=True)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(DEV)
    pre = run(lib, "eva_moe_experts_prefill", cfg, layer_d, x, sel, rw)
    dec = run(lib, "eva_moe_experts_decode", cfg, layer_d, x, sel, rw)
    close(pre, dec, 3e-3, 0.99999)
    # first rows against the FP64 oracle as well
    host = layer_d.host_copy()
    n = 3
    ref = oracle.moe_forward(x[:n].cpu().view(torch.int16).numpy().view(np.uint16), sel[:n], rw[:n], host)
    close(pre[:n], ref, 3e-3, 0.99999)


def test_forward_dispatches_prefill_for_large_batches(oracle):
    """eva_moe_forward at 300 rows routes through the tensor-core path; check against the oracle on
    the kernel's own routing (first rows)."""
    from eva_b200.runner import EvaMoE
    cfg = SMALL
    layer = make_layer(cfg, "cpu", seed=7)
    layer_d = layer.to(DEV)
    M = 300
    moe = EvaMoE(layer_d, max_rows=M)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    logits = torch.empty(M, cfg.n_experts, device=DEV)
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=DEV)
    w = torch.empty(M, cfg.topk, device=DEV)
    out = torch.empty(M, cfg.hidden, device=DEV)
    moe.forward(x.to(DEV), out_f32=out, idx_out=idx, w_out=w, logits_out=logits)
    torch.cuda.synchronize()
    assert moe.status() == 0
    ridx, rwt = oracle.route(logits.cpu().numpy(), layer.router_b.numpy(), cfg)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), ridx, rwt, layer)
    close(out.cpu().numpy(), ref, 3e-3, 0.99999)


def routes_with_counts(counts, M, topk, rng):
    """Routes in which expert e is selected by exactly counts[e] of the M rows (topk distinct experts
    per row): each row takes the topk experts with the most selections left."""
    left = np.array(counts, dtype=np.int64)
    assert left.sum() == M * topk and left.max() <= M
    sel = np.empty((M, topk), dtype=np.int64)
    for m in range(M):
        pick = np.argsort(-left, kind="stable")[:topk]
        assert (left[pick] > 0).all()
        left[pick] -= 1
        sel[m] = rng.permutation(pick)
    return sel[rng.permutation(M)]


def test_prefill_tile_heights_vs_oracle(oracle):
    """Experts whose row counts straddle the tile boundaries: 1, 63, 64, 65, 127, 128 rows (one
    half-height tile; the second CTA of the pair holds no rows, one row, or up to 64), 129, 255 (one
    full tile), 257 (a full tile and a half-height tail), and the shared expert's 320 rows (a full
    tile and a 64-row tail), against the FP64 oracle."""
    lib = _lib.load()
    cfg = SMALL
    M = 320
    counts = [1, 63, 64, 65, 127, 128, 129, 255, 257, 0, 2, 30, 31, 33, 95, 0]
    rng = np.random.default_rng(11)
    sel = routes_with_counts(counts, M, cfg.topk, rng)
    assert [int((sel == e).sum()) for e in range(cfg.n_experts)] == counts
    rw = (rng.random((M, cfg.topk)) + 0.1).astype(np.float32)
    layer = make_layer(cfg, "cpu", seed=5)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    out = run(lib, "eva_moe_experts_prefill", cfg, layer.to(DEV), x.to(DEV), sel, rw)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rw, layer)
    close(out, ref, 3e-3, 0.99999)
