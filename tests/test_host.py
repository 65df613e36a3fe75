"""Host logic without a GPU: configs, expert records and handles, routers, permutation oracle,
the C ABI library's exports. CPU only."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from eva_b200 import config as C
from eva_b200 import experts as X

ROOT = Path(__file__).resolve().parent.parent


def test_config_validation():
    with pytest.raises(ValueError):
        C.MoEConfig("bad", hidden=100, inter=128, n_experts=8, topk=2, router="softmax")
    with pytest.raises(ValueError):
        C.MoEConfig("bad", hidden=256, inter=128, n_experts=8, topk=2, router="nope")
    with pytest.raises(ValueError):
        C.MoEConfig("bad", hidden=256, inter=128, n_experts=8, topk=2, router="sigmoid", n_group=3)
    assert C.V3.expert_bytes() == 16_515_072 + 6 * (7168 + 2048)


def test_record_layout_matches_pack_format():
    offs, rec, shapes = X.record_layout(256, 128, 3)
    # w1 (gate), w2 (down), w3 (up); each suh, svh, trellis (tools/pack_exl3.py:93-107)
    order = sorted(offs.items(), key=lambda kv: kv[1][0])
    assert [k for k, _ in order] == [("gate", "suh"), ("gate", "svh"), ("gate", "trellis"),
                                     ("down", "suh"), ("down", "svh"), ("down", "trellis"),
                                     ("up", "suh"), ("up", "svh"), ("up", "trellis")]
    assert rec % 4096 == 0
    assert all(o % 16 == 0 for o, _ in offs.values())


def test_pointer_tables_address_the_tensors():
    cfg = C.MoEConfig("t", hidden=256, inter=128, n_experts=4, topk=2, router="softmax", shared_inter=256, bits=2)
    layer = X.make_layer(cfg, "cpu", seed=1)
    for e in range(4):
        for (proj, kind), row in X.ROW.items():
            assert int(layer.packed[row, e]) == layer.tensor(e, proj, kind).data_ptr()
    for (proj, kind), row in X.ROW.items():
        assert int(layer.shared[row]) == layer.tensor(-1, proj, kind).data_ptr()
    t = layer.tensor(2, "down", "trellis")
    assert tuple(t.shape) == (128 // 16, 256 // 16, 32)
    suh = layer.tensor(0, "gate", "suh").float()
    assert torch.all(suh.abs() >= 0.74) and torch.all(suh.abs() <= 1.26)


def test_sigmoid_group_limited_route_properties(oracle):
    cfg = C.V3
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((64, cfg.n_experts)).astype(np.float32) * 1.7
    bias = (rng.standard_normal(cfg.n_experts) * 0.01).astype(np.float32)
    idx, w = oracle.route(logits, bias, cfg)
    groups = idx // (cfg.n_experts // cfg.n_group)
    assert all(len(set(g)) <= cfg.topk_group for g in groups)
    assert np.allclose(w.sum(-1), cfg.route_scale, rtol=1e-5)
    assert all(len(set(r)) == cfg.topk for r in idx)
    # without grouping it is plain biased top-k
    flat = cfg.with_(n_group=1, topk_group=1)
    idx2, _ = oracle.route(logits, bias, flat)
    s = oracle.scores(logits, "sigmoid") + bias
    assert np.array_equal(np.sort(idx2, -1), np.sort(np.argsort(-s, -1, kind="stable")[:, :cfg.topk], -1))


def test_softmax_route_unnormalised(oracle):
    cfg = C.V2_LITE
    rng = np.random.default_rng(1)
    logits = rng.standard_normal((16, cfg.n_experts)).astype(np.float32)
    idx, w = oracle.route(logits, np.zeros(cfg.n_experts, np.float32), cfg)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    assert np.allclose(w, np.take_along_axis(p, idx, -1), rtol=1e-6)
    assert np.array_equal(idx, np.argsort(-logits, -1, kind="stable")[:, :cfg.topk])


def test_run_table_edge_cases(oracle):
    # all inactive
    t = oracle.run_table(np.array([[3, 4]]), np.array([[0.0, 0.0]], np.float32), 2)
    assert t[0] == 0 and all(v == 0 for v in t)
    # one expert picked by 20 slots -> runs of 8, 8, 4
    sel = np.array([[5, i] for i in range(20)])[:, :1].repeat(2, 1)
    sel[:, 1] = np.arange(20) + 6
    t = oracle.run_table(sel, None, 20)
    S = 40
    starts = t[2:2 + t[0] + 1]
    assert t[0] == 3 + 20 and starts[:4] == [0, 8, 16, 20]
    order = t[2 + S + 1: 2 + S + 1 + 40]
    assert order[:20] == [2 * i for i in range(20)]


def test_c_abi_exports_every_declared_symbol():
    from eva_b200 import _lib
    L = _lib.load()
    header = (ROOT / "include" / "eva_moe.h").read_text()
    declared = set(re.findall(r"\b(eva_[a-z0-9_]+)\s*\(", header))
    assert declared == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(L, name)
    assert L.eva_moe_arch() == 100
    for cfg in (C.V3, C.V2_LITE, C.REF_NATIVE):
        sh = _lib.shape_of(cfg)
        assert L.eva_moe_workspace_bytes(ctypes.byref(sh), 64) > 0
    bad = _lib.shape_of(C.V3)
    bad.bits = 5
    assert L.eva_moe_workspace_bytes(ctypes.byref(bad), 64) == 0
    # argument errors are reported without touching a GPU
    assert L.eva_exl3_dequant(None, 16, 16, 3, None, None) == _lib.EVA_ERR_INVALID


def test_ctypes_bindings_match_the_header_prototypes():
    """Every binding that declares argtypes passes as many arguments as the header's prototype takes:
    a parameter added to or removed from include/eva_moe.h without the binding fails here, on CPU."""
    from eva_b200 import _lib
    L = _lib.load()
    header = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "eva_moe.h").read_text(), flags=re.S)
    protos = dict(re.findall(r"\b(eva_[a-z0-9_]+)\s*\(([^()]*)\)\s*;", header))
    assert set(protos) == set(_lib.EXPORTS)
    checked = 0
    for name, params in protos.items():
        argtypes = getattr(L, name).argtypes
        if argtypes is None:
            continue
        params = params.strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert len(argtypes) == n, f"{name}: header takes {n} arguments, the binding passes {len(argtypes)}"
        checked += 1
    assert checked >= 20, checked


def test_library_has_no_torch_dependency():
    import subprocess
    out = subprocess.run(["ldd", str(ROOT / "eva_b200" / "libeva_moe.so")], capture_output=True, text=True).stdout
    deps = [ln.split()[0] for ln in out.splitlines() if ln.strip()]
    assert not [d for d in deps if "torch" in d or "c10" in d], out


def test_workspace_grows_with_the_row_count():
    """A workspace sized for max_rows must serve every call with fewer rows: the size is
    non-decreasing in the row count (the router's k-split and the permutation's chunk count both
    depend on the row count; their regions are sized for the worst case up to max_rows)."""
    from eva_b200 import _lib
    L = _lib.load()
    for cfg in (C.V3, C.V2_LITE, C.REF_NATIVE):
        sh = _lib.shape_of(cfg)
        rows = list(range(1, 300)) + list(range(300, 9000, 37))
        sizes = [L.eva_moe_workspace_bytes(ctypes.byref(sh), m) for m in rows]
        assert all(b >= a for a, b in zip(sizes, sizes[1:])), cfg.name


def test_argument_errors_are_reported_without_a_gpu():
    """Entry points validate their arguments and the workspace size before touching a device."""
    from eva_b200 import _lib
    L = _lib.load()
    sh = _lib.shape_of(C.V3)
    fake = 256   # never dereferenced: every call below fails its checks first
    # permutation with a workspace: missing workspace, workspace too small for the rows
    assert L.eva_moe_permute_ws(ctypes.byref(sh), fake, 1, fake, 300, 300, fake, None, None, 0, None) == _lib.EVA_ERR_INVALID
    assert L.eva_moe_permute_ws(ctypes.byref(sh), fake, 1, fake, 300, 300, fake, None, fake, 1024, None) == \
        _lib.EVA_ERR_WORKSPACE
    # capacity below the row count
    assert L.eva_moe_permute(ctypes.byref(sh), fake, 1, fake, 300, 299, fake, None, None) == _lib.EVA_ERR_INVALID
    # routing: workspace too small for the rows (the router's slice partials and weight planes)
    n = L.eva_moe_workspace_bytes(ctypes.byref(sh), 64)
    assert L.eva_moe_route(ctypes.byref(sh), fake, 1, 65, fake, None, None, fake, fake, fake, n, None) == \
        _lib.EVA_ERR_WORKSPACE
    assert L.eva_moe_route(ctypes.byref(sh), fake, 1, 64, fake, None, None, fake, fake, None, n, None) == \
        _lib.EVA_ERR_INVALID


def test_empty_batches_return_before_any_device_work():
    """M = 0 is a valid call for every per-token entry point: arguments are checked, nothing is
    launched (the library is called here with no GPU and never-dereferenced aligned addresses)."""
    from eva_b200 import _lib
    L = _lib.load()
    sh = _lib.shape_of(C.V3)
    a = 1 << 20                                   # 16-byte aligned, never dereferenced
    tables = _lib.table_array([a] * 9)
    shared = _lib.shared_array([a] * 9)
    n = L.eva_moe_workspace_bytes(ctypes.byref(sh), 8)
    ok = _lib.EVA_OK
    assert L.eva_moe_topk(ctypes.byref(sh), a, 0, None, a, a, None) == ok
    assert L.eva_moe_route(ctypes.byref(sh), a, 1, 0, a, None, None, a, a, a, n, None) == ok
    for name in ("eva_moe_experts", "eva_moe_experts_decode", "eva_moe_experts_prefill"):
        assert getattr(L, name)(ctypes.byref(sh), a, 1, 0, a, 1, a, tables, shared, a, n, a, None, None) == ok
    assert L.eva_moe_experts_window(ctypes.byref(sh), a, 1, 0, a, 1, a, tables, shared, 0, 0, a, n, a, None,
                                    None) == ok
    assert L.eva_moe_forward(ctypes.byref(sh), a, 1, 0, a, None, tables, shared, a, n, None, a, None, None, None,
                             None) == ok
    assert L.eva_moe_experts_noalloc(ctypes.byref(sh), a, 1, 0, a, 1, a, tables, shared, None, a, None, None) == ok
    assert L.eva_rmsnorm_residual(C.V3.hidden, 0, a, None, a, 1, 1e-6, a, None) == ok
    # the same calls with a negative row count are argument errors
    assert L.eva_moe_topk(ctypes.byref(sh), a, -1, None, a, a, None) == _lib.EVA_ERR_INVALID
    assert L.eva_moe_experts(ctypes.byref(sh), a, 1, -1, a, 1, a, tables, shared, a, n, a, None, None) == \
        _lib.EVA_ERR_INVALID


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour on a machine without CUDA")
def test_operators_fail_loudly_without_cuda():
    """No CPU fallback: every operator of the product refuses to run without a CUDA device."""
    from eva_b200.ep import EPMoE, ExpertPlacement
    from eva_b200.runner import EvaMoE, EvaMoERunner
    cfg = C.MoEConfig("t", hidden=256, inter=128, n_experts=4, topk=2, router="softmax", bits=3)
    layer = X.make_layer(cfg, "cpu", seed=0)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        EvaMoERunner("cpu", topk=2, hidden=256, inter=128, max_rows=4, n_experts=4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        EvaMoE(layer)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        EPMoE(layer, ExpertPlacement.contiguous(cfg.n_experts, 1), max_tokens=4)


def test_runner_owner_thread_and_poisoning_checks_come_first():
    """EvaMoERunner.run refuses calls from a thread other than its owner and from a poisoned runner
    before looking at its arguments, as the reference runner does (moe_coop2048.py:263-266)."""
    import threading
    from eva_b200.runner import EvaMoERunner
    r = EvaMoERunner.__new__(EvaMoERunner)      # no CUDA here: only the host-side checks run
    r._owner_thread, r._failed = threading.get_ident() + 1, False
    with pytest.raises(RuntimeError, match="owner thread"):
        r.run(None, None, None, None, 3, 0.0)
    r._owner_thread, r._failed = threading.get_ident(), True
    with pytest.raises(RuntimeError, match="discard"):
        r.run(None, None, None, None, 3, 0.0)
    r._failed = False
    with pytest.raises(ValueError, match="K must be"):
        r.run(None, None, None, None, 5, 0.0)
