"""The float32 CPU path that bench.py times as its CPU baseline (oracle/cpu_fast.c) agrees with the
float64 oracle it is a faster form of. CPU only."""
import numpy as np
import pytest
import torch

from eva_b200 import config as C
from eva_b200.experts import make_layer


def _close(a, b, rel):
    assert np.isfinite(a).all()
    err = np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
    cos = float((a.astype(np.float64) * b).sum() / (np.linalg.norm(a) * np.linalg.norm(b)))
    assert err <= rel and cos >= 0.999999, (err, cos)


@pytest.mark.parametrize("bits,shared_bits", [(2, 4), (3, 3), (4, 2)])
def test_fast_cpu_path_matches_oracle(oracle, bits, shared_bits):
    cfg = C.MoEConfig("t", hidden=512, inter=256, n_experts=8, topk=3, router="softmax", shared_inter=384,
                      bits=bits, shared_bits=shared_bits, swiglu_limit=7.0)
    layer = make_layer(cfg, "cpu", seed=3)
    rng = np.random.default_rng(bits)
    M = 41                                        # more rows than one 32-row pass, ragged tail
    sel = np.stack([rng.choice(cfg.n_experts, cfg.topk, replace=False) for _ in range(M)])
    sel[2] = [1, 1, 4]                            # one expert in two slots of a row
    sel[7] = [5, 5, 5]
    rw = (rng.random((M, cfg.topk)) + 0.1).astype(np.float32)
    rw[3, 1] = 0                                  # inactive slot
    rw[9, :] = 0                                  # a row with no active slot
    x = torch.randn(M, cfg.hidden, generator=torch.Generator().manual_seed(bits)).to(torch.bfloat16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    for shared in (True, False):
        ref = oracle.moe_forward(xb, sel, rw, layer, with_shared=shared)
        got = oracle.moe_forward_fast(xb, sel, rw, layer, with_shared=shared, threads=3)
        _close(got, ref, 2e-4)
        if not shared:
            assert np.all(got[9] == 0)


def test_fast_cpu_path_fp16_input_and_missing_expert(oracle):
    cfg = C.MoEConfig("t", hidden=256, inter=128, n_experts=4, topk=2, router="softmax", shared_inter=0, bits=3)
    layer = make_layer(cfg, "cpu", seed=5)
    sel = np.array([[0, 3], [2, 1]])
    rw = np.ones((2, 2), np.float32)
    x = torch.randn(2, cfg.hidden, generator=torch.Generator().manual_seed(0)).to(torch.float16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    _close(oracle.moe_forward_fast(xb, sel, rw, layer, x_is_f16=True),
           oracle.moe_forward(xb, sel, rw, layer, x_is_f16=True), 2e-4)
    layer.packed[0, 2] = 0                        # unbound expert 2 (zero trellis pointer)
    with pytest.raises(RuntimeError):
        oracle.moe_forward_fast(xb, sel, rw, layer)
