"""One rank of the multi-GPU expert-parallel check (launched by tests/test_gpu_ep.py under
torch.distributed.run): EPMoE over NCCL ranks, then rank 0 runs every rank's tokens through the
whole layer on its own GPU (EvaMoE) and writes the largest relative difference as JSON."""
import argparse
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np
import torch
import torch.distributed as dist

from eva_b200 import config as C
from eva_b200.ep import EPMoE, ExpertPlacement
from eva_b200.experts import make_layer

SMALL = C.MoEConfig("small", hidden=512, inter=256, n_experts=16, topk=4, router="sigmoid", n_group=4,
                    topk_group=2, route_scale=2.5, norm_topk=True, shared_inter=384, bits=3, shared_bits=4)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", default="fixed")
    ap.add_argument("--transport", default="peers")
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    out_dir = Path(a.out).parent
    try:
        pl = ExpertPlacement.balanced(np.arange(SMALL.n_experts, 0, -1), world)
        layer = make_layer(SMALL, dev, seed=4, experts=pl.experts_of(rank))
        M = a.tokens
        ep = EPMoE(layer, pl, max_tokens=M, mode=a.mode, transport=a.transport)
        m_r = M if a.mode == "fixed" else M - 3 * rank    # unequal token counts per rank
        g = torch.Generator(device=dev).manual_seed(10 + rank)
        x = torch.randn(m_r, SMALL.hidden, device=dev, generator=g).to(torch.bfloat16)
        y = torch.empty(m_r, SMALL.hidden, device=dev)
        for _ in range(2):                                   # twice: buffers reused across calls
            ep.forward(x, out_f32=y)
        torch.cuda.synchronize()
        st = ep.status()
        np.save(out_dir / f"x{rank}.npy", x.view(torch.int16).cpu().numpy())
        np.save(out_dir / f"y{rank}.npy", y.cpu().numpy())
        sts = [None] * world
        dist.all_gather_object(sts, st)
        dist.barrier()
        if rank == 0:
            from eva_b200.runner import EvaMoE
            full = make_layer(SMALL, dev, seed=4)
            moe = EvaMoE(full, max_rows=M)
            err = 0.0
            for r in range(world):
                xr = torch.as_tensor(np.load(out_dir / f"x{r}.npy")).view(torch.bfloat16).to(dev)
                yr = torch.as_tensor(np.load(out_dir / f"y{r}.npy")).to(dev)
                ref = torch.empty_like(yr)
                moe.forward(xr, out_f32=ref)
                torch.cuda.synchronize()
                err = max(err, ((yr - ref).abs().max() / ref.abs().max()).item())
            res = {"status": int(np.bitwise_or.reduce(np.array(sts + [moe.status()]))), "max_rel_err": err,
                   "world": world, "mode": a.mode, "transport": a.transport}
            Path(a.out).write_text(json.dumps(res))
        dist.barrier()
        ep.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
