"""The eva_b200 kernels against the reference's OWN GPU kernels on the same B200 and inputs.

oracle/_ref/libref_coop.so is compiled from the reference checkout by oracle/build_ref.py (the
vendored ExLlamaV3 dq_dispatch decoder and MoE coop rot/A/B kernels, launched by our harness). The
tests skip when that library was not built. Needs a GPU: -m gpu.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from eva_b200 import _lib
from eva_b200 import config as C
from eva_b200.experts import make_layer

pytestmark = pytest.mark.gpu
DEV = "cuda"
REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_coop.so"


@pytest.fixture(scope="module")
def ref():
    if not REF.exists():
        pytest.skip("oracle/_ref/libref_coop.so not built (needs the reference checkout)")
    L = ctypes.CDLL(str(REF))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    L.ref_dequant.restype = i32
    L.ref_dequant.argtypes = [vp, i32, i32, i32, vp, vp]
    L.ref_coop_ctr_len.restype = ctypes.c_longlong
    L.ref_coop_ctr_len.argtypes = [i32, i32, i32, i32]
    L.ref_coop_run.restype = i32
    L.ref_coop_run.argtypes = [vp, vp, vp, i32, i32, i32, i32, ctypes.POINTER(vp), i32, vp, vp, vp, vp, vp, vp,
                               vp, i32, vp, i32, ctypes.c_float, vp]
    return L


def stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("K", [2, 3, 4])
def test_dequant_bit_exact_vs_reference_kernel(ref, oracle, K):
    """The reference's dq_dispatch<K, mul1> == our CPU decoder == our GPU decoder, bit for bit."""
    fin, fout = 512, 384
    g = torch.Generator().manual_seed(100 + K)
    tr = torch.randint(-32768, 32768, (fin // 16, fout // 16, 16 * K), generator=g, dtype=torch.int32).to(torch.int16)
    trd = tr.to(DEV)
    wr = torch.empty(fin, fout, dtype=torch.int16, device=DEV)
    we = torch.empty(fin, fout, dtype=torch.int16, device=DEV)
    assert ref.ref_dequant(trd.data_ptr(), fin, fout, K, wr.data_ptr(), stream()) == 0
    lib = _lib.load()
    _lib.check(lib.eva_exl3_dequant(trd.data_ptr(), fin, fout, K, we.data_ptr(), stream()), "dequant")
    torch.cuda.synchronize()
    w_ref = wr.cpu().numpy().view(np.uint16)
    assert np.array_equal(w_ref, oracle.dequant(tr.numpy(), K))
    assert np.array_equal(we.cpu().numpy().view(np.uint16), w_ref)


def ref_coop(ref, layer_d, x16, sel, rw16, K, limit, capacity=None):
    cfg = layer_d.cfg
    M, topk, H, I = x16.shape[0], sel.shape[1], cfg.hidden, cfg.inter
    cap = capacity or M
    slots = cap * topk
    o = dict(device=DEV)
    had_g = torch.empty(slots, H, dtype=torch.float16, **o)
    had_u = torch.empty_like(had_g)
    gu_g = torch.empty(slots, I, dtype=torch.float16, **o)
    gu_u = torch.empty_like(gu_g)
    act = torch.empty_like(gu_g)
    d_out = torch.empty(slots, H, dtype=torch.float32, **o)
    ctr = torch.zeros(ref.ref_coop_ctr_len(cap, topk, I, H), dtype=torch.int32, **o)
    out = torch.empty(cap, H, dtype=torch.float32, **o)
    tabs = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in layer_d.packed.unbind(0)])
    rc = ref.ref_coop_run(x16.data_ptr(), sel.data_ptr(), rw16.data_ptr(), M, topk, H, I, tabs, cfg.n_experts,
                          had_g.data_ptr(), had_u.data_ptr(), gu_g.data_ptr(), gu_u.data_ptr(), act.data_ptr(),
                          d_out.data_ptr(), ctr.data_ptr(), cap, out.data_ptr(), K, float(limit), stream())
    assert rc == 0
    return out[:M]


def eva_routed(layer_d, x16, sel, rw, limit):
    from eva_b200.runner import EvaMoERunner
    cfg = layer_d.cfg
    r = EvaMoERunner(DEV, topk=cfg.topk, hidden=cfg.hidden, inter=cfg.inter, max_rows=x16.shape[0],
                     n_experts=cfg.n_experts)
    return r.run(x16, sel, rw, tuple(layer_d.packed.unbind(0)), cfg.bits, limit)


CASES = [
    C.MoEConfig("small", hidden=512, inter=256, n_experts=16, topk=6, router="sqrtsoftplus", bits=3),
    C.MoEConfig("v2l-routed", hidden=2048, inter=1408, n_experts=64, topk=6, router="softmax", bits=4),
    C.MoEConfig("ref-native-routed", hidden=5120, inter=2304, n_experts=384, topk=6, router="sqrtsoftplus",
                bits=3, swiglu_limit=10.0),
    C.MoEConfig("v3-routed-k2", hidden=7168, inter=2048, n_experts=256, topk=8, router="sigmoid", bits=2),
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
@pytest.mark.parametrize("M", [1, 5])
def test_moe_matches_reference_kernels(ref, oracle, cfg, M):
    """Same x, routes, Half route weights and expert tables through the reference's coop kernels and
    through eva_moe_experts; both against the FP64 oracle. The reference accumulates in fp16, so it
    sits ~1e-3 from the oracle; ours sits closer."""
    layer_d = make_layer(cfg, DEV, seed=M)
    rng = np.random.default_rng(M)
    sel = np.stack([rng.choice(cfg.n_experts, cfg.topk, replace=False) for _ in range(M)]).astype(np.int64)
    rw = (rng.random((M, cfg.topk)) + 0.1).astype(np.float32)
    x16 = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(M)).to(torch.float16).to(DEV)
    seld = torch.tensor(sel, device=DEV)
    rw16 = torch.tensor(rw, device=DEV).half()
    y_ref = ref_coop(ref, layer_d, x16, seld, rw16, cfg.bits, cfg.swiglu_limit).cpu().numpy()
    y_eva = eva_routed(layer_d, x16, seld, rw16, cfg.swiglu_limit).cpu().numpy()
    torch.cuda.synchronize()
    # oracle on the selected experts only (host copy of the few records used)
    host = layer_d.host_copy()
    ref64 = oracle.moe_forward(x16.cpu().view(torch.int16).numpy().view(np.uint16), sel,
                               rw16.float().cpu().numpy(), host, with_shared=False, x_is_f16=True)
    scale = np.abs(ref64).max()
    e_ref = np.abs(y_ref - ref64).max() / scale
    e_eva = np.abs(y_eva - ref64).max() / scale
    e_cross = np.abs(y_eva - y_ref).max() / scale
    cos = float((y_eva.ravel() @ y_ref.ravel()) / (np.linalg.norm(y_eva) * np.linalg.norm(y_ref)))
    print(f"{cfg.name} M={M}: ref-vs-oracle {e_ref:.2e}, eva-vs-oracle {e_eva:.2e}, eva-vs-ref {e_cross:.2e}, cos {cos:.7f}")
    assert e_cross <= 2e-2 and cos >= 0.9999
    assert e_eva <= 3e-3


def test_speed_vs_reference_kernels(ref, capsys):
    """Routed experts of the DeepSeek-V3 decode step (batch 8, K3, 4.24 GB of experts): the reference's
    prepare/rot/A/B launches vs eva_moe_experts, same routes, CUDA events, a different batch every
    iteration (working set larger than L2). Prints both times and checks that the two outputs of the
    last batch agree (max-rel-err <= 2e-2, cosine >= 0.9999)."""
    cfg = C.V3.with_(shared_inter=0)
    layer_d = make_layer(cfg, DEV, seed=0)
    M, iters = 8, 20
    rng = np.random.default_rng(0)
    sels = [torch.tensor(np.stack([rng.choice(cfg.n_experts, cfg.topk, replace=False) for _ in range(M)]),
                         device=DEV) for _ in range(iters + 3)]
    rw16 = torch.full((M, cfg.topk), 0.125, device=DEV).half()
    xs = [torch.randn(M, cfg.hidden, device=DEV).half() for _ in range(iters + 3)]
    from eva_b200.runner import EvaMoERunner
    r = EvaMoERunner(DEV, topk=cfg.topk, hidden=cfg.hidden, inter=cfg.inter, max_rows=M, n_experts=cfg.n_experts)
    times, outs = {}, {}
    for name in ("reference", "eva"):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for i in range(iters + 3):
            if i == 3:
                torch.cuda.synchronize()
                ev[0].record()
            if name == "reference":
                y = ref_coop(ref, layer_d, xs[i], sels[i], rw16, cfg.bits, 0.0)
            else:
                y = r.run(xs[i], sels[i], rw16, tuple(layer_d.packed.unbind(0)), cfg.bits, 0.0, check_bounds=False)
        ev[1].record()
        torch.cuda.synchronize()
        times[name] = ev[0].elapsed_time(ev[1]) / iters
        outs[name] = y.double().cpu().numpy().ravel()
    a, b = outs["eva"], outs["reference"]
    err = np.abs(a - b).max() / np.abs(b).max()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    with capsys.disabled():
        print(f"\nV3 decode routed experts, batch {M}, K3: reference {times['reference']:.3f} ms/step, "
              f"eva {times['eva']:.3f} ms/step, speed-up {times['reference'] / times['eva']:.2f}x; "
              f"eva vs reference max-rel-err {err:.2e}, cosine {cos:.7f}")
    assert times["reference"] > 0 and times["eva"] > 0
    assert err <= 2e-2 and cos >= 0.9999


def test_prefill_speed_vs_reference_kernels(ref, capsys):
    """Routed experts of a DeepSeek-V3 prefill step (4096 tokens, K3, expert load skewed as rank^-1.1):
    the reference's coop kernels, which take at most 2048 slots per call (256 tokens at top-8), called
    16 times, vs one eva_moe_experts call (tensor-core path), same routes and fp16 inputs, CUDA
    events. Prints both times and checks the two outputs agree (max-rel-err, cosine)."""
    cfg = C.V3.with_(shared_inter=0)
    layer_d = make_layer(cfg, DEV, seed=0)
    M, chunk, iters = 4096, 256, 3
    E, k = cfg.n_experts, cfg.topk
    rng = np.random.default_rng(0)
    pz = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    pz /= pz.sum()
    perm = rng.permutation(E)
    sel = torch.tensor(np.stack([perm[rng.choice(E, k, replace=False, p=pz)] for _ in range(M)]), device=DEV)
    x16 = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(5)).half().to(DEV)
    rw16 = torch.full((M, k), 0.125, device=DEV).half()
    from eva_b200.runner import EvaMoERunner
    r = EvaMoERunner(DEV, topk=k, hidden=cfg.hidden, inter=cfg.inter, max_rows=M, n_experts=E)
    packed = tuple(layer_d.packed.unbind(0))

    def run_ref():
        return torch.cat([ref_coop(ref, layer_d, x16[i:i + chunk], sel[i:i + chunk], rw16[i:i + chunk], cfg.bits, 0.0)
                          for i in range(0, M, chunk)])

    def run_eva():
        return r.run(x16, sel, rw16, packed, cfg.bits, 0.0, check_bounds=False)

    times, outs = {}, {}
    for name, fn in (("reference", run_ref), ("eva", run_eva)):
        outs[name] = fn()                       # warm-up
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for _ in range(iters):
            fn()
        ev[1].record()
        torch.cuda.synchronize()
        times[name] = ev[0].elapsed_time(ev[1]) / iters
    a, b = outs["eva"].double().cpu().numpy().ravel(), outs["reference"].double().cpu().numpy().ravel()
    err = np.abs(a - b).max() / np.abs(b).max()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    with capsys.disabled():
        print(f"\nV3 prefill routed experts, {M} tokens, K3: reference {times['reference']:.3f} ms "
              f"({M // chunk} calls of {chunk} tokens), eva {times['eva']:.3f} ms, speed-up "
              f"{times['reference'] / times['eva']:.2f}x; eva vs reference max-rel-err {err:.2e}, cosine {cos:.7f}")
    assert err <= 2e-2 and cos >= 0.9999


def test_shared_expert_matches_reference_kernels(ref, oracle):
    """The shared expert's three EXL3 linears (exllamav3 LinearEXL3 in the reference, runtime/ds41/
    exl3_linear.py:135-151, not installed here) checked through the reference's own coop kernels, which
    run the same EXL3 linear: a table whose 6 columns all hold the DeepSeek-V3 shared expert, every token
    routed to all 6 with weight 1, gives 6 x the shared expert's output (swiglu limit 0, where the two
    activation clamp orders agree). Ours: eva_moe_experts with every routed slot inactive and the shared
    expert on (its virtual-slot path)."""
    cfg = C.V3.with_(n_experts=6, topk=6, n_group=1, topk_group=1)
    layer_d = make_layer(cfg, DEV, seed=4, n_fill=0)      # routed records unused; the shared one is filled
    M, H, I, K = 5, cfg.hidden, cfg.shared_inter, cfg.shared_bits
    x16 = torch.randn(M, H, generator=torch.Generator().manual_seed(7)).to(torch.float16).to(DEV)
    sel = torch.arange(6, device=DEV, dtype=torch.int64).repeat(M, 1)
    # the reference: 6 identical columns pointing at the shared expert's tensors
    cols = [torch.full((6,), int(a), dtype=torch.int64, device=DEV) for a in layer_d.shared.tolist()]
    slots = M * 6
    o = dict(device=DEV)
    had_g = torch.empty(slots, H, dtype=torch.float16, **o)
    had_u = torch.empty_like(had_g)
    gu_g = torch.empty(slots, I, dtype=torch.float16, **o)
    gu_u = torch.empty_like(gu_g)
    act = torch.empty_like(gu_g)
    d_out = torch.empty(slots, H, dtype=torch.float32, **o)
    ctr = torch.zeros(ref.ref_coop_ctr_len(M, 6, I, H), dtype=torch.int32, **o)
    out = torch.empty(M, H, dtype=torch.float32, **o)
    tabs = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in cols])
    rw16 = torch.ones(M, 6, device=DEV).half()
    assert ref.ref_coop_run(x16.data_ptr(), sel.data_ptr(), rw16.data_ptr(), M, 6, H, I, tabs, 6, had_g.data_ptr(),
                            had_u.data_ptr(), gu_g.data_ptr(), gu_u.data_ptr(), act.data_ptr(), d_out.data_ptr(),
                            ctr.data_ptr(), M, out.data_ptr(), K, 0.0, stream()) == 0
    y_ref = (out / 6).cpu().numpy()
    # ours: shared expert only
    lib = _lib.load()
    sh = _lib.shape_of(cfg)
    ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(sh), M), dtype=torch.uint8, device=DEV)
    y = torch.full((M, H), float("nan"), device=DEV)
    rw0 = torch.zeros(M, 6, device=DEV)
    _lib.check(lib.eva_moe_experts(ctypes.byref(sh), x16.data_ptr(), 0, M, sel.data_ptr(), 1, rw0.data_ptr(),
                                   _lib.table_array(tuple(layer_d.packed.unbind(0))),
                                   _lib.shared_array(layer_d.shared.tolist()), ws.data_ptr(), ws.numel(), y.data_ptr(),
                                   None, stream()), "experts")
    st = ctypes.c_int32(0)
    _lib.check(lib.eva_moe_read_status(ws.data_ptr(), ctypes.byref(st), stream()), "status")
    assert st.value == 0
    y_eva = y.cpu().numpy()
    host = layer_d.host_copy()
    ref64 = oracle.moe_forward(x16.cpu().view(torch.int16).numpy().view(np.uint16), sel.cpu().numpy(),
                               rw0.cpu().numpy(), host, with_shared=True, x_is_f16=True)
    scale = np.abs(ref64).max()
    e_ref = np.abs(y_ref - ref64).max() / scale
    e_eva = np.abs(y_eva - ref64).max() / scale
    e_cross = np.abs(y_eva - y_ref).max() / scale
    cos = float((y_eva.ravel() @ y_ref.ravel()) / (np.linalg.norm(y_eva) * np.linalg.norm(y_ref)))
    print(f"V3 shared expert M={M}: ref-vs-oracle {e_ref:.2e}, eva-vs-oracle {e_eva:.2e}, eva-vs-ref {e_cross:.2e}, "
          f"cos {cos:.7f}")
    assert e_cross <= 2e-2 and cos >= 0.9999
    assert e_eva <= 3e-3
