"""Generate the DeepSeek-V3 and DeepSeek-V2-Lite routing fixtures in this folder.

The reference project itself routes only with sqrtsoftplus (runtime/ds41/model.py:404-416, pinned by
route_sqrtsoftplus.npz from make_golden.py). The two other routers this library implements follow the
published DeepSeek gating, and the installed `transformers` package (5.5.0) carries that gating as
plain PyTorch:
  route_v3_sigmoid.npz    DeepseekV3MoE.route_tokens_to_experts: sigmoid scores, + e_score_correction_bias
                          for selection, group score = sum of the top-2 biased scores of each of 8
                          groups, top-4 groups kept, top-8 experts, unbiased weights renormalised
                          (sum + 1e-20), x routed_scaling_factor 2.5.
  route_v2lite_softmax.npz
                          DeepseekV2Moe.route_tokens_to_experts with topk_method "greedy": float32
                          softmax, top-6, no renormalisation, x routed_scaling_factor 1.0.
Both functions are called unbound on a namespace holding just the attributes they read, so no expert
weights are allocated. transformers returns the top-k unsorted (torch.topk sorted=False); the fixture
stores each row's experts in ascending id order with their weights alongside.

transformers masks the experts of dropped groups with 0.0 where DeepSeek's own inference code uses
-inf. The two agree whenever every kept expert has a positive biased score, which this script asserts
for the rows it writes.

Usage: python tests/golden/make_route_pins.py
"""
from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import numpy as np

OUT = Path(__file__).resolve().parent


def v3_inputs(M: int, E: int, seed: int):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((M, E)) * 1.7).astype(np.float32)
    # a few rows with one strong group and one strong expert outside the kept groups
    logits[:4, 32:64] += 3.0
    logits[4:8, 200] += 6.0
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32)
    return logits, bias


def v2lite_inputs(M: int, E: int, seed: int):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((M, E)) * 1.3).astype(np.float32)
    logits[:4, :6] += 4.0
    return logits


def transformers_v3_route(logits: np.ndarray, bias: np.ndarray):
    """indices (int64, ascending per row) and float32 weights from transformers' DeepSeek-V3 gating."""
    import torch
    from transformers.models.deepseek_v3.modeling_deepseek_v3 import DeepseekV3MoE
    M, E = logits.shape
    self = SimpleNamespace(gate=SimpleNamespace(e_score_correction_bias=torch.tensor(bias)),
                           n_routed_experts=E, n_group=8, topk_group=4, norm_topk_prob=True,
                           routed_scaling_factor=2.5, top_k=8)
    with torch.no_grad():
        idx, w = DeepseekV3MoE.route_tokens_to_experts(self, torch.tensor(logits))
        choice = torch.tensor(logits).sigmoid() + torch.tensor(bias)
        assert bool((choice.gather(1, idx) > 0).all()), "a kept expert scored <= 0: 0.0 vs -inf masking"
    return _ascending(idx.numpy(), w.numpy())


def transformers_v2lite_route(logits: np.ndarray):
    """indices (int64, ascending per row) and float32 weights from transformers' DeepSeek-V2 greedy gating."""
    import torch
    from transformers.models.deepseek_v2.modeling_deepseek_v2 import DeepseekV2Moe
    self = SimpleNamespace(topk_method="greedy", top_k=6, routed_scaling_factor=1.0)
    with torch.no_grad():
        idx, w = DeepseekV2Moe.route_tokens_to_experts(self, torch.tensor(logits)[None])
    return _ascending(idx.numpy(), w.numpy())


def _ascending(idx: np.ndarray, w: np.ndarray):
    order = np.argsort(idx, axis=-1, kind="stable")
    return (np.take_along_axis(idx, order, -1).astype(np.int64),
            np.take_along_axis(w, order, -1).astype(np.float32))


def main():
    logits, bias = v3_inputs(128, 256, seed=31)
    idx, w = transformers_v3_route(logits, bias)
    np.savez(OUT / "route_v3_sigmoid.npz", logits=logits, bias=bias, indices=idx, weights=w)

    logits = v2lite_inputs(256, 64, seed=32)
    idx, w = transformers_v2lite_route(logits)
    np.savez(OUT / "route_v2lite_softmax.npz", logits=logits, indices=idx, weights=w)
    print("wrote route_v3_sigmoid.npz, route_v2lite_softmax.npz")


if __name__ == "__main__":
    main()
