"""A decode stream through a stack of MoE layers (the 58-layer DeepSeek-V3 configuration): per layer
h = RMSNorm(x) * w_layer, x += MoE_layer(h), attention stubbed out (it adds nothing to the residual
stream), and a final RMSNorm.

Reference: the per-layer residual flow of runtime/ds41/model.py:1453-1483 and `rms`
(model.py:968-970). The residual stream stays in FP32 between layers; one kernel per layer boundary
(eva_rmsnorm_residual) adds the previous layer's output and normalises the next layer's BF16 input.
"""
from __future__ import annotations

import torch

from . import _lib

_BF16, _F32 = torch.bfloat16, torch.float32


class MoEStack:
    """layers: MoE operators with forward(h_bf16, out_f32=...) (EPMoE or EvaMoE), in order;
    norms: per-layer RMSNorm weights (BF16 [H] on the device) plus one final norm (len(layers) + 1)."""

    def __init__(self, layers, norms, eps: float = 1e-6):
        if len(norms) != len(layers) + 1:
            raise ValueError("one norm weight per layer plus the final norm")
        self.layers, self.norms, self.eps = list(layers), list(norms), float(eps)
        self.lib = _lib.load()
        self.hidden = norms[0].numel()

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x: BF16 [M, H] on the device; returns the final normalised BF16 [M, H]."""
        if x.dim() != 2 or x.shape[1] != self.hidden or x.dtype != _BF16:
            raise ValueError(f"x must be BF16 [M, {self.hidden}]")
        M, H = x.shape
        dev = x.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        resid = x.to(_F32)
        h = torch.empty(M, H, dtype=_BF16, device=dev)
        y = torch.empty(M, H, dtype=_F32, device=dev)
        add = None
        for layer, w in zip(self.layers, self.norms):
            _lib.check(self.lib.eva_rmsnorm_residual(H, M, resid.data_ptr(), _lib.ptr(add), w.data_ptr(), 1, self.eps,
                                                     h.data_ptr(), stream), "eva_rmsnorm_residual")
            layer.forward(h, out_f32=y)
            add = y
        if out is None:
            out = torch.empty(M, H, dtype=_BF16, device=dev)
        _lib.check(self.lib.eva_rmsnorm_residual(H, M, resid.data_ptr(), _lib.ptr(add), self.norms[-1].data_ptr(), 1,
                                                 self.eps, out.data_ptr(), stream), "eva_rmsnorm_residual")
        return out

    __call__ = forward


def make_norms(n_layers: int, hidden: int, device, seed: int = 0):
    """Synthetic RMSNorm weights near 1 (seeded)."""
    g = torch.Generator().manual_seed(seed)
    return [(1.0 + 0.1 * torch.randn(hidden, generator=g)).to(_BF16).to(device) for _ in range(n_layers + 1)]
