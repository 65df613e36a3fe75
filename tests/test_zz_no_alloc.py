"""eva_moe_experts_noalloc: the expert path for callers that cannot allocate device memory.

Such callers (a serving runtime that has already reserved the GPU's memory in its own pool, a
plugin host that hands over only input and output buffers, a latency-critical loop that must not
call cudaMalloc) get the same computation as eva_moe_experts with the scratch taken from a fixed
16 MiB device array inside the library. The GPU tests call both entry points through the C ABI on
the same inputs and check that they agree, on two calls in a row (the second call finds the first
call's leftovers in the shared array), for the DeepSeek-V2-Lite shape and for the DeepSeek-V3 shape
at its largest accepted batch. The host test pins the documented row limits: the size check runs
before any device call, so it needs no GPU. The file name makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from eva_b200 import _lib
from eva_b200 import config as C
from eva_b200.experts import make_layer

DEV = "cuda"
# largest accepted rows per call (documented in include/eva_moe.h beside the entry point)
MAX_ROWS = {"v3": 27, "v2-lite": 90, "ref-native": 47}


def _close(out, ref, rel=3e-3, cos=0.99999):
    out = np.asarray(out, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    c = float(out @ ref / (np.linalg.norm(out) * np.linalg.norm(ref)))
    assert err <= rel and c >= cos, f"max-rel-err {err:.3e} cosine {c:.7f}"


@pytest.mark.parametrize("cfg", [C.V3, C.V2_LITE, C.REF_NATIVE], ids=lambda c: c.name)
def test_noalloc_row_limit_is_checked_before_device_work(cfg):
    """At the documented maximum the size check passes and the null x is then rejected as an
    argument error; one row more is rejected as too large for the scratch. Neither reaches the
    device, so this runs without a GPU."""
    lib = _lib.load()
    shape = _lib.shape_of(cfg)
    tables = (ctypes.c_void_p * 9)(*([256] * 9))
    shared = (ctypes.c_int64 * 9)(*([256] * 9))
    m = MAX_ROWS[cfg.name]
    args = (256, 0, 256, tables, shared, 256, None, None, None)   # sel, sel_is_i64, rw, ..., out_f32, ..., stream
    assert lib.eva_moe_experts_noalloc(ctypes.byref(shape), None, 1, m, *args) == _lib.EVA_ERR_INVALID
    assert lib.eva_moe_experts_noalloc(ctypes.byref(shape), None, 1, m + 1, *args) == _lib.EVA_ERR_WORKSPACE


def _compare(lib, cfg, layer, Ms, seed):
    shape = _lib.shape_of(cfg)
    tables = _lib.table_array(tuple(layer.packed.unbind(0)))
    shared = _lib.shared_array(layer.shared.tolist())
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(seed)
    for call, M in enumerate(Ms):
        sel = torch.tensor(np.stack([rng.choice(cfg.n_experts, cfg.topk, replace=False) for _ in range(M)]),
                           dtype=torch.int32, device=DEV)
        rw = torch.tensor(rng.random((M, cfg.topk)) + 0.05, dtype=torch.float32, device=DEV)
        x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(seed + call)).to(torch.bfloat16).to(DEV)
        # existing entry point, caller-provided workspace
        ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(shape), M), dtype=torch.uint8, device=DEV)
        ref = torch.empty(M, cfg.hidden, device=DEV)
        _lib.check(lib.eva_moe_experts(ctypes.byref(shape), x.data_ptr(), 1, M, sel.data_ptr(), 0, rw.data_ptr(),
                                       tables, shared, ws.data_ptr(), ws.numel(), ref.data_ptr(), None, stream),
                   "eva_moe_experts")
        # allocation-free entry point
        out = torch.full((M, cfg.hidden), float("nan"), device=DEV)
        status = torch.full((1,), -1, dtype=torch.int32, device=DEV)
        _lib.check(lib.eva_moe_experts_noalloc(ctypes.byref(shape), x.data_ptr(), 1, M, sel.data_ptr(), 0,
                                               rw.data_ptr(), tables, shared, out.data_ptr(), None,
                                               status.data_ptr(), stream), "eva_moe_experts_noalloc")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        _close(out.cpu().numpy(), ref.cpu().numpy())


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point():
    lib = _lib.load()
    _compare(lib, C.V2_LITE, make_layer(C.V2_LITE, DEV, seed=21), (7, 3), seed=21)


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_v3_at_its_limit():
    """DeepSeek-V3 shape (the bench's): the largest accepted batch, then a batch of 8."""
    lib = _lib.load()
    layer = make_layer(C.V3, DEV, seed=22)
    _compare(lib, C.V3, layer, (MAX_ROWS["v3"], 8), seed=22)
    del layer
    torch.cuda.empty_cache()


@pytest.mark.gpu
def test_noalloc_rejects_calls_beyond_its_scratch():
    lib = _lib.load()
    cfg = C.V3
    shape = _lib.shape_of(cfg)
    dummy = (ctypes.c_void_p * 9)(*([256] * 9))
    sh = (ctypes.c_int64 * 9)(*([256] * 9))
    rc = lib.eva_moe_experts_noalloc(ctypes.byref(shape), 256, 1, 512, 256, 0, 256, dummy, sh, 256, None, None,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.EVA_ERR_WORKSPACE
