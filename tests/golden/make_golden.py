"""Generate the golden fixtures in this folder by running the reference's own Python code.

Needs a checkout of the reference (Findddx/eva); pass its root as the first argument or set
EVA_REFERENCE. The fixtures it writes are small and committed; the tests never read the reference.

What is pinned, and by which reference function (paths within the reference project):
  run_tables.json   runtime/ds41/moe_coop2048.py:91-111 and moe_coop3072.py reference_table: the exact
                    int32 run table of the MoE coop kernels for seeded routes and Half route weights
                    (zeros = inactive slots), plus reference_runs from moe_coop512.py:54-73.
  route_sqrtsoftplus.npz
                    runtime/ds41/model.py:404-416 Block.route on CPU: x (Half-rounded), FP32 gate
                    weights/bias -> FP32 logits (stable_linear), weights, indices.
  swiglu.npz        runtime/ds41/kernels.py:213-217 swiglu(gate, up, limit).
  mul1.json         runtime/ds41/cpu_precision_reference.py:43-45 mul1_integer on seeded states, and
                    MUL1_SCALE.
  rms.npz           runtime/ds41/model.py:968-970 rms(x, weight, eps) for FP32 and BF16 rows with a BF16
                    weight.

Usage: python tests/golden/make_golden.py [/path/to/reference]
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

OUT = Path(__file__).resolve().parent


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EVA_REFERENCE")
    if not ref:
        sys.exit("pass the reference checkout's root as the first argument or set EVA_REFERENCE")
    ref = Path(ref)
    sys.path.insert(0, str(ref / "runtime"))
    import torch
    import ds41.cpu_precision_reference as cpr
    import ds41.kernels as kernels
    import ds41.model as model
    import ds41.moe_coop2048 as c2048
    import ds41.moe_coop3072 as c3072
    import ds41.moe_coop512 as c512

    rng = np.random.default_rng(1234)

    # ---- run tables -------------------------------------------------------------------------
    cases = []

    def routes(rows, n_experts=384, skew=False):
        out = []
        for _ in range(rows):
            if skew:   # concentrate on few experts to make long runs (> 8 slots of one expert)
                pool = rng.choice(24, size=6, replace=False)
            else:
                pool = rng.choice(n_experts, size=6, replace=False)
            out.append([int(e) for e in pool])
        return out

    def half_weights(rows, zero_frac):
        w = rng.random((rows, 6)).astype(np.float32) + 0.05
        w[rng.random((rows, 6)) < zero_frac] = 0.0
        return torch.tensor(w).to(torch.float16).float().tolist()

    for module, name, caps in ((c2048, "moe_coop2048", (256,)), (c3072, "moe_coop3072", (512,))):
        for rows, skew, zero in ((1, False, 0.0), (3, False, 0.0), (17, True, 0.0), (40, True, 0.25),
                                 (64, False, 0.1), (200, True, 0.05)):
            if rows > caps[0]:
                continue
            idx = routes(rows, skew=skew)
            w = half_weights(rows, zero)
            table = module.reference_table(idx, w, capacity=caps[0])
            runs = module.reference_runs(idx, w)
            cases.append({"module": name, "capacity": caps[0], "indices": idx, "weights": w,
                          "table": table, "runs": runs})
    for rows, skew in ((1, False), (9, True), (64, True)):
        idx = routes(rows, skew=skew)
        runs = c512.reference_runs(idx)
        cases.append({"module": "moe_coop512", "capacity": 64, "indices": idx,
                      "weights": [[1.0] * 6 for _ in idx], "table": None, "runs": runs})
    (OUT / "run_tables.json").write_text(json.dumps({"cases": cases}, separators=(",", ":")))

    # ---- Block.route (sqrt(softplus) + bias top-6, normalised x 1.5) --------------------------
    torch.manual_seed(7)
    E, H, M = 384, 128, 32
    gate_w = (torch.randn(E, H) * 0.05).float()
    gate_b = (torch.randn(E) * 0.02).float()
    x = torch.randn(M, H).to(torch.float16)
    blk = SimpleNamespace(gate_w=gate_w, gate_b=gate_b, gate_b_vl=None, layer_id=0,
                          args=SimpleNamespace(n_activated_experts=6, route_scale=1.5))
    w, idx = model.Block.route(blk, x, None)
    logits = model.stable_linear(x.float(), gate_w)
    np.savez_compressed(OUT / "route_sqrtsoftplus.npz", x_f16=x.numpy(), gate_w=gate_w.numpy(),
                        gate_b=gate_b.numpy(), logits=logits.numpy(), weights=w.numpy(),
                        indices=idx.numpy().astype(np.int64), topk=6, route_scale=1.5)

    # ---- swiglu --------------------------------------------------------------------------------
    g = torch.randn(64, 128) * 6
    u = torch.randn(64, 128) * 6
    outs = {f"out_{lim}": kernels.swiglu(g, u, float(lim)).numpy() for lim in (0, 10, 2.5)}
    np.savez_compressed(OUT / "swiglu.npz", gate=g.numpy(), up=u.numpy(), **outs)

    # ---- mul1 integer identity ----------------------------------------------------------------
    states = [0, 1, 0x1234, 0xFFFF, 0x8000, 0x7FFF] + [int(s) for s in rng.integers(0, 65536, 250)]
    (OUT / "mul1.json").write_text(json.dumps({
        "states": states, "mul1_integer": [cpr.mul1_integer(s) for s in states],
        "MUL1_SCALE": cpr.MUL1_SCALE, "MUL1_MULT": cpr.MUL1_MULT}))
    # ---- rms (the layer-stack RMSNorm) ----------------------------------------------------------
    torch.manual_seed(11)
    xr = (torch.randn(6, 512) * 3).float()
    wr = (1.0 + 0.1 * torch.randn(512)).to(torch.bfloat16)
    out_f32 = model.rms(xr, wr, 1e-6)
    out_bf16 = model.rms(xr.to(torch.bfloat16), wr, 1e-6)
    np.savez_compressed(OUT / "rms.npz", x=xr.numpy(), w_bf16=wr.view(torch.int16).numpy(), eps=1e-6,
                        out_f32=out_f32.float().numpy(), out_bf16=out_bf16.view(torch.int16).numpy())
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
