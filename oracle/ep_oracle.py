"""CPU checker for the expert-parallel exchange — TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module; the product (eva_b200) never does and has no CPU fallback.

The reference has no expert parallelism. What it restates is the per-rank slot filter the
reference kernel anticipates (runtime/ds41/csrc/moe_coop2048/vendor/exl3_moe_coop_kernel.cuh:
208-223, slot_info: a slot counts on this rank only when its expert is local) and the empty-row
rule (:573-610: a token with no local expert gets a shared-only or zero row), written as an
explicit dispatch plan, plus the sum the layer must produce (runtime/ds41/model.py:454-499:
shared expert + routed experts). `ep_plan` is the specification eva_ep_dispatch follows;
`OracleEpOps` runs one rank's share of the layer with the oracle so that the exchange logic of
eva_b200.ep.EPMoE can be checked with gloo ranks on a CPU.
"""
from __future__ import annotations

import numpy as np
import torch

from . import oracle as O


def ep_plan(idx, w, owner, local_id, world: int, capacity: int, segment: int = 0):
    """Dispatch plan of one rank: (counts [world], pos [world, M], send_sel [cap, k], send_rw [cap, k],
    capacity_overflow). Token m goes to rank r once when one of its slots with a non-zero weight
    has an expert owned by r; rows for r are in token order, starting at r * segment (fixed) or
    after rank r-1's rows (packed)."""
    idx = np.asarray(idx)
    w = np.asarray(w, dtype=np.float32)
    owner = np.asarray(owner)
    local_id = np.asarray(local_id)
    M, k = idx.shape
    dest = np.full((M, k), -1, dtype=np.int64)
    act = w != 0
    dest[act] = owner[idx[act]]
    counts = np.zeros(world, dtype=np.int32)
    within = np.full((world, M), -1, dtype=np.int64)
    for r in range(world):
        to_r = (dest == r).any(axis=1)
        within[r, to_r] = np.arange(int(to_r.sum()))
        counts[r] = int(to_r.sum())
    offs = np.arange(world) * segment if segment else np.concatenate([[0], np.cumsum(counts)[:-1]])
    pos = np.full((world, M), -1, dtype=np.int32)
    send_sel = np.zeros((capacity, k), dtype=np.int32)
    send_rw = np.zeros((capacity, k), dtype=np.float32)
    overflow = bool((counts > segment).any()) if segment else int(counts.sum()) > capacity
    for r in range(world):
        for m in np.flatnonzero(within[r] >= 0):
            p = int(offs[r] + within[r, m])
            if (segment and within[r, m] >= segment) or (not segment and p >= capacity):
                continue
            pos[r, m] = p
            on = dest[m] == r
            send_sel[p, on] = local_id[idx[m, on]]
            send_rw[p, on] = w[m, on]
    return counts, pos, send_sel, send_rw, overflow


class OracleEpOps:
    """One rank's device work of eva_b200.ep.EPMoE, done on the CPU by the oracle."""

    def __init__(self, layer, placement):
        self.cfg, self.layer, self.placement = layer.cfg, layer, placement
        self.world = placement.world
        self.device = torch.device("cpu")

    @staticmethod
    def _bits(x):
        return x.contiguous().view(torch.int16).numpy().view(np.uint16)

    def route(self, x):
        logits = O.router_logits(O.bf16_to_f32(self._bits(x)), self.layer.router_w.numpy())
        idx, w = O.route(logits, self.layer.router_b.numpy(), self.cfg)
        return torch.as_tensor(idx.astype(np.int32)), torch.as_tensor(w.astype(np.float32))

    def dispatch(self, x, idx, w, capacity, segment):
        counts, pos, ssel, srw, _ = ep_plan(idx.numpy(), w.numpy(), self.placement.owner, self.placement.local_id,
                                            self.world, capacity, segment)
        sx = torch.zeros(capacity, self.cfg.hidden, dtype=x.dtype)
        for r in range(self.world):
            for m in np.flatnonzero(pos[r] >= 0):
                sx[pos[r, m]] = x[m]
        return (torch.as_tensor(counts), torch.as_tensor(pos), sx, torch.as_tensor(ssel), torch.as_tensor(srw))

    def experts(self, x, sel, rw, out_f32):
        if x.shape[0]:
            out_f32.copy_(torch.as_tensor(O.moe_forward(self._bits(x), sel.numpy(), rw.numpy(), self.layer,
                                                        with_shared=False)))
        return out_f32

    def shared(self, x):
        if self.layer.shared is None:
            return None
        M = x.shape[0]
        z = np.zeros((M, self.cfg.topk), dtype=np.int32)
        return torch.as_tensor(O.moe_forward(self._bits(x), z, z.astype(np.float32), self.layer, with_shared=True))

    def combine(self, back, pos, base, out_bf16, out_f32=None):
        M = pos.shape[1]
        acc = torch.zeros(M, self.cfg.hidden, dtype=torch.float32) if base is None else base.clone()
        for r in range(self.world):
            for m in np.flatnonzero(pos[r].numpy() >= 0):
                acc[m] += back[int(pos[r, m])]
        if out_f32 is not None:
            out_f32.copy_(acc)
        if out_bf16 is not None:
            out_bf16.copy_(acc.to(torch.bfloat16))

    def read_status(self) -> int:
        return 0
