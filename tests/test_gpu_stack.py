"""Layer-stack glue, expert residency and DS41PK01 packs on a B200: the residual + RMSNorm kernel
against the oracle, EPMoE with a device slot budget smaller than the experts a step selects (grouped
launches, misses copied from pinned host memory) against the whole layer, a 3-layer stack against
the oracle, and a layer loaded from a pack against the layer it was written from. Needs a GPU."""
import numpy as np
import pytest
import torch

from eva_b200 import _lib
from eva_b200 import config as C
from eva_b200.ep import EPMoE, ExpertPlacement
from eva_b200.experts import make_layer
from eva_b200.residency import ExpertResidency
from eva_b200.runner import EvaMoE
from eva_b200.stack import MoEStack, make_norms

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = C.MoEConfig("small", hidden=512, inter=256, n_experts=16, topk=4, router="sigmoid", n_group=4,
                    topk_group=2, route_scale=2.5, norm_topk=True, shared_inter=384, bits=3, shared_bits=4)


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("M,with_add", [(1, False), (7, True), (300, True)])
def test_rmsnorm_residual_kernel(oracle, M, with_add):
    lib = _lib.load()
    H = 7168
    g = torch.Generator().manual_seed(M)
    resid = (torch.randn(M, H, generator=g) * 2).to(DEV)
    add = torch.randn(M, H, generator=g).to(DEV) if with_add else None
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(DEV)
    h = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
    r0 = resid.cpu().numpy() + (add.cpu().numpy() if with_add else 0)
    _lib.check(lib.eva_rmsnorm_residual(H, M, resid.data_ptr(), _lib.ptr(add), w.data_ptr(), 1, 1e-6, h.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream), "rms")
    torch.cuda.synchronize()
    np.testing.assert_allclose(resid.cpu().numpy(), r0.astype(np.float32), rtol=0, atol=0)
    ref = oracle.rmsnorm(r0.astype(np.float32), oracle.bf16_to_f32(_bits(w)), 1e-6)
    got = oracle.bf16_to_f32(_bits(h))
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 8e-3, err      # BF16 output rounding


@pytest.mark.parametrize("M,slots", [(8, 6), (24, 5), (24, 16)])
def test_resident_experts_match_whole_layer(M, slots):
    host = make_layer(SMALL, "cpu", seed=12)
    full = host.to(DEV)
    pl = ExpertPlacement.contiguous(SMALL.n_experts, 1)
    res = ExpertResidency(host, slots, DEV)
    ep = EPMoE(host, pl, max_tokens=M, residency=res)
    moe = EvaMoE(full, max_rows=M)
    g = torch.Generator(device=DEV).manual_seed(M)
    for step in range(3):
        x = torch.randn(M, SMALL.hidden, device=DEV, generator=g).to(torch.bfloat16)
        a = torch.empty(M, SMALL.hidden, device=DEV)
        b = torch.empty(M, SMALL.hidden, device=DEV)
        ep.forward(x, out_f32=a)
        moe.forward(x, out_f32=b)
        torch.cuda.synchronize()
        assert ep.status() == 0 and moe.status() == 0
        err = (a - b).abs().max().item() / b.abs().max().item()
        assert err < 1e-4, (step, err)
    assert res.stats["misses"] > 0
    if slots < SMALL.n_experts:
        assert res.stats["h2d_bytes"] >= res.stats["misses"] * res.record_bytes
    ep.close()


def test_three_layer_stack_matches_oracle(oracle):
    L, M = 3, 5
    hosts = [make_layer(SMALL, "cpu", seed=20 + i) for i in range(L)]
    ops = [EvaMoE(h.to(DEV), max_rows=M) for h in hosts]
    norms = make_norms(L, SMALL.hidden, DEV, seed=4)
    stack = MoEStack(ops, norms)
    x = torch.randn(M, SMALL.hidden, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    out = stack.forward(x.to(DEV))
    torch.cuda.synchronize()
    resid = oracle.bf16_to_f32(_bits(x)).astype(np.float64)
    for i in range(L):
        w = oracle.bf16_to_f32(_bits(norms[i]))
        hb = oracle.f32_to_bf16(oracle.rmsnorm(resid.astype(np.float32), w, 1e-6))
        y, _, _, _ = oracle.layer_forward(hb, hosts[i])
        resid = resid + y
    ref = oracle.rmsnorm(resid.astype(np.float32), oracle.bf16_to_f32(_bits(norms[-1])), 1e-6)
    got = oracle.bf16_to_f32(_bits(out))
    err = np.abs(got - ref).max() / np.abs(ref).max()
    cos = float((got.ravel() @ ref.ravel()) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err < 2e-2 and cos > 0.9999, (err, cos)


def test_layer_from_pack_runs_like_the_original(tmp_path):
    from eva_b200.pack import Pack, load_layer, write_pack
    cfg = SMALL
    src = make_layer(cfg, "cpu", seed=31)
    path = tmp_path / "experts.bin"
    write_pack(str(path), [src])
    back = load_layer(Pack.open(str(path)), 0, src, device=DEV)
    M = 6
    x = torch.randn(M, cfg.hidden, device=DEV).to(torch.bfloat16)
    a = torch.empty(M, cfg.hidden, device=DEV)
    b = torch.empty(M, cfg.hidden, device=DEV)
    EvaMoE(back, max_rows=M).forward(x, out_f32=a)
    EvaMoE(src.to(DEV), max_rows=M).forward(x, out_f32=b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
