"""One rank of the multi-GPU expert-parallel check (launched by tests/test_gpu_ep.py under
torch.distributed.run): EPMoE over NCCL ranks, then rank 0 runs every rank's tokens through the
whole layer on its own GPU (EvaMoE) and writes the largest relative difference as JSON. With
--pool the ranks' experts live behind the device expert cache (two layers sharing one pool)."""
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
    ap.add_argument("--pool", action="store_true",
                    help="two layers per rank behind one device expert pool smaller than their experts")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    out_dir = Path(a.out).parent
    try:
        if a.pool:
            return pooled(a, rank, world, dev, out_dir)
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


def pooled(a, rank, world, dev, out_dir):
    """Two layers on every rank whose experts live in pinned host memory behind one ExpertPool of
    n_local + 2 slots (so the layers evict each other's experts), each layer prefetching the other;
    three steps with new inputs per layer and step. Rank 0 checks every step of both layers against the
    whole layers on one GPU."""
    from eva_b200.residency import ExpertPool
    pl = ExpertPlacement.balanced(np.arange(SMALL.n_experts, 0, -1), world)
    mine = pl.experts_of(rank)
    hosts = [make_layer(SMALL, dev, seed=4 + li, experts=mine).host_copy(pinned=True) for li in range(2)]
    pool = ExpertPool(dev, len(mine) + 2, hosts[0].record_bytes)
    pls = [pool.add_layer(h) for h in hosts]
    pls[0].next, pls[1].next = pls[1], pls[0]
    M = a.tokens
    eps = [EPMoE(h, pl, max_tokens=M, mode=a.mode, transport="peers", residency=r) for h, r in zip(hosts, pls)]
    g = torch.Generator(device=dev).manual_seed(20 + rank)
    steps = 3
    for step in range(steps):
        for li in range(2):
            x = torch.randn(M, SMALL.hidden, device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty(M, SMALL.hidden, device=dev)
            eps[li].forward(x, out_f32=y)
            np.save(out_dir / f"px{rank}_{step}_{li}.npy", x.view(torch.int16).cpu().numpy())
            np.save(out_dir / f"py{rank}_{step}_{li}.npy", y.cpu().numpy())
    torch.cuda.synchronize()
    st = eps[0].status() | eps[1].status() | pool.status()
    copied = pool.bytes_copied()
    sts = [None] * world
    dist.all_gather_object(sts, (st, copied))
    dist.barrier()
    if rank == 0:
        from eva_b200.runner import EvaMoE
        moes = [EvaMoE(make_layer(SMALL, dev, seed=4 + li), max_rows=M) for li in range(2)]
        err = 0.0
        for r in range(world):
            for step in range(steps):
                for li in range(2):
                    xr = torch.as_tensor(np.load(out_dir / f"px{r}_{step}_{li}.npy")).view(torch.bfloat16).to(dev)
                    yr = torch.as_tensor(np.load(out_dir / f"py{r}_{step}_{li}.npy")).to(dev)
                    ref = torch.empty_like(yr)
                    moes[li].forward(xr, out_f32=ref)
                    torch.cuda.synchronize()
                    err = max(err, ((yr - ref).abs().max() / ref.abs().max()).item())
        status = int(np.bitwise_or.reduce(np.array([s for s, _ in sts] + [m.status() for m in moes])))
        res = {"status": status, "max_rel_err": err, "world": world, "mode": a.mode, "transport": "peers",
               "pool_bytes_copied": [c for _, c in sts]}
        Path(a.out).write_text(json.dumps(res))
    dist.barrier()
    for e in eps:
        e.close()


if __name__ == "__main__":
    main()
