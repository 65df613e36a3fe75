"""Shape and routing configuration of one DeepSeek MoE layer.

The reference carries these as `ModelArgs` fields (runtime/ds41/args.py:6-24) plus the per-layer
EXL3 bit width from its k-map (runtime/ds41/model.py:1044-1050). The reference only ships the
"sqrtsoftplus" router (runtime/ds41/model.py:404-416); "softmax" (DeepSeek-V2-Lite) and
"sigmoid" with group-limited selection (DeepSeek-V3) follow the published DeepSeek gating.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

ROUTERS = ("softmax", "sigmoid", "sqrtsoftplus")
ROUTER_CODE = {name: i for i, name in enumerate(ROUTERS)}


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int                 # H
    inter: int                  # routed expert intermediate width I
    n_experts: int              # E routed experts
    topk: int
    router: str                 # one of ROUTERS
    n_group: int = 1            # group-limited routing (sigmoid): groups of E / n_group experts
    topk_group: int = 1         # groups kept per token
    route_scale: float = 1.0    # routed_scaling_factor / route_scale
    norm_topk: bool = False     # renormalise the selected weights to sum 1 (+1e-20)
    shared_inter: int = 0       # shared expert intermediate width (0: no shared expert)
    bits: int = 3               # EXL3 K of the routed experts
    shared_bits: int = 3        # EXL3 K of the shared expert
    swiglu_limit: float = 0.0   # 0 = no clamp

    def __post_init__(self):
        if self.router not in ROUTERS:
            raise ValueError(f"router must be one of {ROUTERS}")
        if self.hidden % 256 or self.inter % 128 or (self.shared_inter and self.shared_inter % 128):
            raise ValueError("hidden must be a multiple of 256 and inter widths multiples of 128")
        if self.bits not in (2, 3, 4) or self.shared_bits not in (2, 3, 4):
            raise ValueError("EXL3 K must be 2, 3 or 4")
        if not 1 <= self.topk <= 32 or self.topk > self.n_experts:
            raise ValueError("topk must be in 1..32 and <= n_experts")
        if self.n_experts % self.n_group or not 1 <= self.topk_group <= self.n_group:
            raise ValueError("n_group must divide n_experts and topk_group <= n_group")
        if self.n_experts > 1024:
            raise ValueError("at most 1024 routed experts")

    def with_(self, **kw) -> "MoEConfig":
        return replace(self, **kw)

    @property
    def router_code(self) -> int:
        return ROUTER_CODE[self.router]

    def expert_bytes(self, bits: int | None = None, inter: int | None = None) -> int:
        """Bytes of one expert record: 3 trellis tensors + suh/svh fp16 vectors."""
        k = self.bits if bits is None else bits
        i = self.inter if inter is None else inter
        h = self.hidden
        return 3 * h * i * k // 8 + 2 * (h + i) * 3


# DeepSeek-V2-Lite: hidden 2048, 64 routed experts top-6 softmax (no renormalisation), expert
# intermediate 1408, 2 shared experts (one MLP of width 2 * 1408).
V2_LITE = MoEConfig("v2-lite", hidden=2048, inter=1408, n_experts=64, topk=6, router="softmax",
                    route_scale=1.0, norm_topk=False, shared_inter=2816, bits=4, shared_bits=4)

# DeepSeek-V3: hidden 7168, 256 routed experts top-8 sigmoid with e_score_correction_bias,
# n_group 8 / topk_group 4, routed_scaling 2.5, normalised weights, 1 shared expert of 2048.
V3 = MoEConfig("v3", hidden=7168, inter=2048, n_experts=256, topk=8, router="sigmoid",
               n_group=8, topk_group=4, route_scale=2.5, norm_topk=True, shared_inter=2048,
               bits=3, shared_bits=3)

# eva's own checkpoint shape (runtime/ds41/args.py:12-24): sqrt(softplus) router + bias,
# normalised weights x 1.5, SwiGLU limit 10; K3 routed experts.
REF_NATIVE = MoEConfig("ref-native", hidden=5120, inter=2304, n_experts=384, topk=6,
                       router="sqrtsoftplus", route_scale=1.5, norm_topk=True, shared_inter=2304,
                       bits=3, shared_bits=3, swiglu_limit=10.0)

CONFIGS = {c.name: c for c in (V2_LITE, V3, REF_NATIVE)}
