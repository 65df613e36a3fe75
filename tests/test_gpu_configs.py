"""Parity at the configurations bench.py measures, against the FP64 oracle. Needs a B200: -m gpu.

* Config 3 (DeepSeek-V3 shape, EXL3 K3, 4.24 GB of experts): router + experts + shared through
  EvaMoE.forward at decode batches 1, 8, 16, 32 and 64 (the bench's headline line is batch 8).
* Config 2 (DeepSeek-V2-Lite shape, EXL3 K4): batches 1 and 16 (4 is in test_gpu_kernels.py).
* Skewed decode batches in which one expert is chosen by more rows than one run holds (8), so an
  expert is streamed as several runs, with ragged run lengths.

The oracle reads a host copy of the experts the step selected (a few hundred MB to 3.6 GB), not the
whole layer. Bars: router indices bit-exact given the kernel's logits; FP32 output max-rel-err
<= 3e-3 and cosine >= 0.99999; BF16 output max-rel-err <= 2e-2 and cosine >= 0.9999.
"""
import ctypes
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from eva_b200 import _lib
from eva_b200 import config as C
from eva_b200.experts import ROW, make_layer, record_layout

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(out, ref, rel, cos):
    out = np.asarray(out, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    c = float(out @ ref / (np.linalg.norm(out) * np.linalg.norm(ref) + 1e-300))
    assert err <= rel and c >= cos, f"max-rel-err {err:.3e} cosine {c:.7f}"
    return err, c


def host_subset(layer_d, experts):
    """The routed records `experts` (global ids of a whole-layer ExpertLayer) and the shared record
    copied to host memory, as the layer view the oracle reads: its pointer table holds host
    addresses for those experts and zero for every other column."""
    cfg = layer_d.cfg
    rec = layer_d.record_bytes
    ids = sorted({int(e) for e in np.asarray(experts).ravel()})
    E = layer_d.n_local
    sh_bytes = layer_d.storage.numel() - E * rec
    store = torch.empty(len(ids) * rec + sh_bytes, dtype=torch.uint8).pin_memory()
    for i, e in enumerate(ids):
        store[i * rec:(i + 1) * rec].copy_(layer_d.storage[e * rec:(e + 1) * rec])
    if sh_bytes:
        store[len(ids) * rec:].copy_(layer_d.storage[E * rec:])
    base = store.data_ptr()
    offs, _, _ = record_layout(cfg.hidden, cfg.inter, cfg.bits)
    packed = torch.zeros(9, E, dtype=torch.int64)
    for (proj, kind), row in ROW.items():
        for i, e in enumerate(ids):
            packed[row, e] = base + i * rec + offs[(proj, kind)][0]
    shared = None
    if cfg.shared_inter:
        soffs, _, _ = record_layout(cfg.hidden, cfg.shared_inter, cfg.shared_bits)
        shared = torch.zeros(9, dtype=torch.int64)
        for (proj, kind), row in ROW.items():
            shared[row] = base + len(ids) * rec + soffs[(proj, kind)][0]
    return SimpleNamespace(cfg=cfg, packed=packed, shared=shared, storage=store, router_b=layer_d.router_b.cpu())


@pytest.fixture(scope="module")
def v3_layer():
    layer = make_layer(C.V3, DEV, seed=0)        # 4.24 GB, generated on the device
    yield layer
    del layer
    torch.cuda.empty_cache()


@pytest.fixture(scope="module")
def v2l_layer():
    return make_layer(C.V2_LITE, DEV, seed=0)


def _forward_vs_oracle(oracle, layer_d, M, seed):
    from eva_b200.runner import EvaMoE
    cfg = layer_d.cfg
    moe = EvaMoE(layer_d, max_rows=M)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
    logits = torch.empty(M, cfg.n_experts, device=DEV)
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=DEV)
    w = torch.empty(M, cfg.topk, device=DEV)
    out32 = torch.empty(M, cfg.hidden, device=DEV)
    y = moe.forward(x.to(DEV), out_f32=out32, idx_out=idx, w_out=w, logits_out=logits)
    torch.cuda.synchronize()
    assert moe.status() == 0
    ridx, rw = oracle.route(logits.cpu().numpy(), layer_d.router_b.cpu().numpy(), cfg)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    host = host_subset(layer_d, ridx)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), ridx, rw, host)
    e32, c32 = close(out32.cpu().numpy(), ref, rel=3e-3, cos=0.99999)
    e16, c16 = close(y.float().cpu().numpy(), ref, rel=2e-2, cos=0.9999)
    print(f"{cfg.name} M={M}: {len(np.unique(ridx))} experts, fp32 {e32:.2e}/{c32:.7f}, bf16 {e16:.2e}/{c16:.7f}")


@pytest.mark.parametrize("M", [1, 8, 16, 32, 64])
def test_v3_decode_matches_oracle(oracle, v3_layer, M):
    """Config 3: DeepSeek-V3 layer, EXL3 K3 routed + shared experts, sigmoid group-limited router."""
    _forward_vs_oracle(oracle, v3_layer, M, seed=100 + M)


@pytest.mark.parametrize("M", [1, 16])
def test_v2lite_decode_matches_oracle(oracle, v2l_layer, M):
    """Config 2: DeepSeek-V2-Lite layer, EXL3 K4 routed experts, softmax top-6, 2816-wide shared MLP."""
    _forward_vs_oracle(oracle, v2l_layer, M, seed=200 + M)


def _skewed_routes(cfg, M, hot, rng):
    """Routes in which expert hot[i][0] is chosen by the first hot[i][1] rows, the remaining slots
    of every row filled with distinct random experts."""
    sel = np.zeros((M, cfg.topk), dtype=np.int64)
    hot_ids = {e for e, _ in hot}
    for m in range(M):
        chosen = [e for e, n in hot if m < n]
        rest = [e for e in rng.permutation(cfg.n_experts) if e not in hot_ids][: cfg.topk - len(chosen)]
        row = np.array(chosen + rest)
        sel[m] = row[rng.permutation(cfg.topk)]
    rw = (rng.random((M, cfg.topk)) + 0.1).astype(np.float32)
    return sel, rw


@pytest.mark.parametrize("M,hot", [(40, ((3, 40), (7, 13), (200, 9))), (64, ((11, 64), (12, 33), (250, 17))),
                                   (9, ((5, 9),))], ids=["M40", "M64", "M9"])
def test_v3_skewed_runs_match_oracle(oracle, v3_layer, M, hot):
    """An expert chosen by more than 8 rows is split into several runs (40 rows: 5 runs of one
    expert; 13 rows: 8 + 5; 9 rows: 8 + 1), each streamed by the decode kernel."""
    cfg = C.V3
    rng = np.random.default_rng(M)
    sel, rw = _skewed_routes(cfg, M, hot, rng)
    for e, n in hot:
        assert (sel == e).sum() == n
    layer_d = v3_layer
    sh = _lib.shape_of(cfg)
    lib = _lib.load()
    ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(sh), M), dtype=torch.uint8, device=DEV)
    out = torch.full((M, cfg.hidden), float("nan"), device=DEV)
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
    xd, seld, rwd = x.to(DEV), torch.tensor(sel, device=DEV), torch.tensor(rw, device=DEV)
    rc = lib.eva_moe_experts(ctypes.byref(sh), xd.data_ptr(), 1, M, seld.data_ptr(), 1, rwd.data_ptr(),
                             _lib.table_array(tuple(layer_d.packed.unbind(0))), _lib.shared_array(layer_d.shared.tolist()),
                             ws.data_ptr(), ws.numel(), out.data_ptr(), None,
                             torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "experts")
    st = ctypes.c_int32(0)
    _lib.check(lib.eva_moe_read_status(ws.data_ptr(), ctypes.byref(st), torch.cuda.current_stream().cuda_stream),
               "status")
    assert st.value == 0
    host = host_subset(layer_d, sel)
    ref = oracle.moe_forward(x.view(torch.int16).numpy().view(np.uint16), sel, rw, host)
    close(out.cpu().numpy(), ref, rel=3e-3, cos=0.99999)
