"""Benchmark of the B200 DeepSeek MoE hot path (one JSON line on rank 0).

Workload (N = 1): one DeepSeek-V3-shape MoE layer in decode (hidden 7168, 256 routed experts top-8
sigmoid group-limited n_group 8 / topk_group 4 with e_score_correction_bias, routed_scaling 2.5,
expert intermediate 2048, 1 shared expert, EXL3 K = 3 = 4.24 GB of experts), batch of --batch
tokens (default 8) per step. A step = router -> permutation -> fused experts -> combine + shared.
Each step routes a different pre-generated batch, so the experts touched change from step to step
and the 4.24 GB of expert weights never fit the 126 MB L2 (inputs larger than L2; no flush).

value     tokens/s with inputs already in HBM, timed with CUDA events on the launching stream.
e2e       tokens/s through the public API (EvaMoE.forward) with every step's batch copied from pinned
          host memory and its result copied back inside the timed region (two buffer sets: the next
          batch's copy and this result's read-back run on a copy stream under the compute).
roofline  the fused experts launch (eva_moe_experts: permutation + experts kernel): algorithmic
          bytes = U * R + S (U distinct routed experts of the step, R bytes per expert record, S the
          shared expert record) over its event-timed duration, against MEASURED_PEAKS.json hbm_gbs.
cpu_baseline  the CPU port of the path (FP32 numpy router + oracle/cpu_fast.c: float32 experts with the
          EXL3 dequantization fused into the GEMV, all host threads; checked against the float64
          oracle by the tests) on rank 0's host cores, N = 1, over a few whole batch steps.

N > 1 (torchrun): expert parallelism. Each rank holds n_experts / N experts (placed by expected
load) and its own batch of --batch tokens (weak scaling; global batch N * batch); a step is
EPMoE.forward: route, dispatch (each token's row stored into its experts' owners' arenas over NVLink
by this library's peer-memory kernels; --ep-transport nccl: NCCL send/recv instead), shared + local
experts, combine (partial sums read back from the peers). value = all ranks' tokens / max over ranks
of the timed region; phase_ms_per_step splits the step by phase (max / min over ranks) and
placement_balance gives the routed slots and distinct experts per rank. The prefill leg runs
--prefill-tokens tokens per rank the same way with exact splits.

--impl reference: the same CPU port of the path on the host cores, one whole batch step per step,
rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "moe_layer_decode_tokens_per_s"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="eva", choices=["eva", "reference"])
    ap.add_argument("--config", default="v3")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--small", action="store_true", help="small case for ncu captures (64 experts)")
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--graph", action="store_true",
                    help="N = 1 decode: also time the same steps replayed from CUDA graphs (one per batch)")
    ap.add_argument("--prefill-only", action="store_true")
    ap.add_argument("--stack", action="store_true",
                    help="config 5: decode stream through --stack-layers MoE layers (RMSNorm + residual, "
                         "attention stubbed), expert parallel over the ranks")
    ap.add_argument("--stack-layers", type=int, default=58,
                    help="--stack: layers (0: 58, or with --residency < 1 the most the node's host memory holds)")
    ap.add_argument("--residency", type=float, default=1.0,
                    help="--stack: fraction of each rank's experts resident on the device (misses from pinned host)")
    ap.add_argument("--staging", default="device", choices=["device", "host"],
                    help="--stack --residency < 1: device-side expert cache shared by the layers (planned and "
                         "copied by the device, next layer prefetched) or the host-managed per-layer residency")
    ap.add_argument("--decode-microbench", action="store_true",
                    help="the EXL3 decode loop alone (tiles resident in shared memory): decoded weights per SM clock "
                         "of each decode design, against the rate HBM streaming needs")
    ap.add_argument("--ep-transport", default="peers", choices=["peers", "nccl"],
                    help="N > 1: rows exchanged through NVLink peer memory by this library's kernels, or NCCL")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


HBM_SPEC_GBS = 8000.0   # the north star's nominal B200 HBM3e figure; frac_of_spec is reported beside frac


def tensor_peak():
    """Dense bf16 TFLOP/s for a kernel timed inside a long step (sustained figure)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("bf16_tflops_sustained", d.get("bf16_tflops"))), "measured (sustained)"
    return 1400.0, "fallback (sustained)"


ZIPF_S = 1.1
ZIPF_BETA = 0.1


def zipf_bias(cfg, base, seed=3):
    """Router bias skewed toward a Zipf(1.1) expert load: beta * log(rank^-s), ranks permuted by seed."""
    import numpy as np
    import torch
    rng = np.random.default_rng(seed)
    rank = np.empty(cfg.n_experts)
    rank[rng.permutation(cfg.n_experts)] = np.arange(1, cfg.n_experts + 1)
    off = torch.tensor(ZIPF_BETA * np.log(rank ** -ZIPF_S), dtype=torch.float32, device=base.device)
    return (base + off).contiguous()


# decode: identical steps for at least this long right before the timed ones (clock sampling window)
DECODE_SETTLE_S = 1.0
DECODE_SETTLE_MAX = 20000

# untimed prefill steps before the timed ones (the leg can follow seconds of CPU-only work, after
# which the GPU clocks need a few steps to come back up)
PREFILL_WARMUP = 5
PREFILL_WARMUP_S = 0.3
# the timed prefill region lasts at least this long (more steps than asked when they are short), so
# that the GPU's power management has settled: tens of milliseconds after an idle or lighter phase
# run at a higher clock than the sustained one
PREFILL_TIMED_S = 1.0
PREFILL_MAX_STEPS = 400


def prefill_measure(cfg, layer, dev, steps, warmup, M):
    """Prefill step (router + tensor-core experts) on M tokens with Zipf-skewed routing."""
    import ctypes
    import numpy as np
    import torch
    from eva_b200 import _lib
    lib = _lib.load()
    shape = _lib.shape_of(cfg)
    ws = torch.empty(lib.eva_moe_workspace_bytes(ctypes.byref(shape), M), dtype=torch.uint8, device=dev)
    ws.zero_()
    bias = zipf_bias(cfg, layer.router_b)
    tables = _lib.table_array(tuple(layer.packed.unbind(0)))
    shared = _lib.shared_array(layer.shared.tolist()) if layer.shared is not None else None
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    xs = [torch.randn(M, cfg.hidden, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=dev)
    w = torch.empty(M, cfg.topk, device=dev)
    out = torch.empty(M, cfg.hidden, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def step(i, ev=None):
        x = xs[i % 2]
        _lib.check(lib.eva_moe_route(ctypes.byref(shape), x.data_ptr(), 1, M, layer.router_w.data_ptr(), bias.data_ptr(),
                                     None, idx.data_ptr(), w.data_ptr(), ws.data_ptr(), ws.numel(), stream), "route")
        if ev is not None:
            ev[0].record()
        _lib.check(lib.eva_moe_experts_prefill(ctypes.byref(shape), x.data_ptr(), 1, M, idx.data_ptr(), 0, w.data_ptr(),
                                               tables, shared, ws.data_ptr(), ws.numel(), None, out.data_ptr(), stream),
                   "experts_prefill")
        if ev is not None:
            ev[1].record()

    # at least `warmup` untimed steps and at least PREFILL_WARMUP_S seconds of them
    t_w = time.perf_counter()
    i, t_mid = 0, None
    while i < warmup or time.perf_counter() - t_w < PREFILL_WARMUP_S:
        step(i)
        i += 1
        if i >= warmup:
            torch.cuda.synchronize()
            if t_mid is None:
                t_mid = (time.perf_counter(), i)   # the steady part starts after the first `warmup` steps
    torch.cuda.synchronize()
    t_now = time.perf_counter()
    if t_mid is not None and i > t_mid[1]:
        per_step = (t_now - t_mid[0]) / (i - t_mid[1])
    else:
        per_step = (t_now - t_w) / max(i, 1)
    steps = max(steps, min(PREFILL_MAX_STEPS, math.ceil(PREFILL_TIMED_S / max(per_step, 1e-6))))
    loads = np.bincount(idx.cpu().numpy().ravel(), minlength=cfg.n_experts)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index if dev.index is not None else 0).__enter__()
    clocks.wait_first()
    c_start = clocks.mark()
    t0.record()
    for i in range(steps):
        step(i, evs[i])
    t1.record()
    torch.cuda.synchronize()
    time.sleep(0.06)   # let the sampler report the end of the region
    c_end = clocks.mark()
    clocks.__exit__(None, None, None)
    clock_summary = clocks.summary(c_start, c_end)
    ms = t0.elapsed_time(t1) / steps
    ems = statistics.mean(a.elapsed_time(b) for a, b in evs)
    flop_exp = 6.0 * cfg.hidden * (M * cfg.topk * cfg.inter + M * cfg.shared_inter)
    flop_router = 2.0 * M * cfg.hidden * cfg.n_experts
    peak, kind = tensor_peak()
    share = np.sort(loads)[::-1] / loads.sum()
    # 256-row expert tiles the CTA pairs run (each decodes its expert's weights once): routed + shared;
    # a tile of at most 128 rows runs at half height (M = 128 pair MMAs)
    counts = [int(n) for n in loads if n > 0] + ([M] if cfg.shared_inter else [])
    tiles = sum((n + 255) // 256 for n in counts)
    half = sum(1 for n in counts if 0 < n % 256 <= 128)
    mma_rows = 256 * tiles - 128 * half
    return {"metric": "moe_layer_prefill_tokens_per_s", "value": M / (ms * 1e-3), "unit": "tokens/s",
            "tokens_per_step": M, "ms_per_step": ms, "steps": steps,
            "routing": f"router bias + {ZIPF_BETA} * log(rank^-{ZIPF_S}) (Zipf-skewed); expert load top-8 share "
                       f"{share[:8].sum():.3f}, top-32 {share[:32].sum():.3f}, experts used {(loads > 0).sum()}",
            "expert_tiles": {"tiles": tiles, "half_height_tiles": half,
                             "row_fill": (M * cfg.topk + (M if cfg.shared_inter else 0)) / mma_rows,
                             "row_fill_if_all_256": (M * cfg.topk + (M if cfg.shared_inter else 0)) / (tiles * 256.0),
                             "experts_used": int((loads > 0).sum()) + (1 if cfg.shared_inter else 0)},
            "roofline": {"bound": "tensor", "achieved": (flop_exp) / (ems * 1e-3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                         "frac": (flop_exp) / (ems * 1e-3) / 1e12 / peak, "peak_kind": kind,
                         "kernel": "eva_moe_experts_prefill (permute + rotate + gate/up + down + combine)",
                         "alg_flop_per_launch": flop_exp, "launch_ms": ems},
            "step_tflops_incl_router": (flop_exp + flop_router) / (ms * 1e-3) / 1e12,
            "clocks": clock_summary}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def wait_first(self, timeout=3.0):
        t_end = time.time() + timeout
        while not self.lines and time.time() < t_end:
            time.sleep(0.02)

    def mark(self):
        """Index of the next sample: samples from here on fall in the region being measured."""
        return len(self.lines)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, start=0, end=None):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[start:end]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def host_threads() -> int:
    """The host cores this process may run on (its CPU affinity set, else the machine's count)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_sample(cfg, layer_host, x_bits, threads):
    """CPU port of one step on the rows of x_bits (bf16 bits [M, H]): FP32 router logits (numpy),
    top-k, routed experts + shared expert in float32 with fused EXL3 dequantization (seconds, tokens)."""
    import numpy as np
    from oracle import oracle as O
    t0 = time.perf_counter()
    logits = O.bf16_to_f32(x_bits) @ layer_host.router_w.numpy().T
    idx, w = O.route(logits, layer_host.router_b.numpy(), cfg)
    O.moe_forward_fast(x_bits, idx, w, layer_host, threads=threads)
    return time.perf_counter() - t0, x_bits.shape[0]


def run_reference(args):
    """--impl reference: the CPU port of the path, one whole batch step per step, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import torch
    from eva_b200.config import CONFIGS
    from eva_b200.experts import make_layer
    cfg = CONFIGS[args.config]
    threads = host_threads()
    # every expert its own seeded record (the same bytes as the GPU arm's layer), 4.24 GB for V3
    torch.set_num_threads(threads)
    layer = make_layer(cfg, "cpu", seed=0)
    M = args.batch
    g = torch.Generator().manual_seed(1)
    xs = torch.randn(args.steps + args.warmup, M, cfg.hidden, generator=g).to(torch.bfloat16)
    xb = xs.view(torch.int16).numpy().view(np.uint16)
    rows = M
    for i in range(args.warmup):
        dt, _ = cpu_sample(cfg, layer, xb[i, :rows], threads)
        if dt * args.steps > 240.0 and rows > 1:
            rows = 1      # a slow host: one token of each batch per step keeps the run within minutes
    times, tokens = [], 0
    for i in range(args.steps):
        dt, n = cpu_sample(cfg, layer, xb[args.warmup + i, :rows], threads)
        times.append(dt)
        tokens += n
    total = sum(times)
    value = tokens / total
    sample = (f"{rows} of the {M} tokens of each step's batch through this repository's float32 C port of the "
              f"path (oracle/cpu_fast.c: FP32 router, top-{cfg.topk} routed experts + shared expert, EXL3 "
              f"dequantization fused into the GEMV, {threads} threads) over {cfg.n_experts} distinct expert records, "
              f"on rank 0's host cores; the reference's own CPU expert path needs exllamav3, which is not installed")
    world = args.gpus
    # the eva arm's config for the same run (bench.py decode line), the sample described in cpu_baseline
    config = {"workload": f"DeepSeek-{cfg.name.upper()} MoE layer decode (EXL3 K{cfg.bits}), batch {M} tokens/step"
                          + (f" per GPU, expert parallel over {world} GPUs" if world > 1 else ""),
              "hidden": cfg.hidden, "experts": cfg.n_experts, "topk": cfg.topk, "inter": cfg.inter,
              "shared_inter": cfg.shared_inter, "bits": cfg.bits, "batch": M,
              "parallelism": f"ep{world}" if world > 1 else "single",
              "reference_path": "the reference's path ported to the CPU (oracle/cpu_fast.c, float32), rank 0"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


EXCHANGE = {
    "peers": "NVLink peer memory (CUDA IPC arenas): dispatch kernel stores rows into the destinations' segments, "
             "flags released per source, combine kernel reads the peers' FP32 partial rows; no host sync, no NCCL",
    "nccl": "fixed segments (no host sync): grouped NCCL send/recv of rows, ids, weights; all-to-all of FP32 "
            "partial sums back",
}


def zipf_load(cfg, seed=3):
    """Expected relative load per expert under zipf_bias (rank^-s with the same rank permutation)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    rank = np.empty(cfg.n_experts)
    rank[rng.permutation(cfg.n_experts)] = np.arange(1, cfg.n_experts + 1)
    return rank ** -ZIPF_S


def measured_load(cfg, dev, rank, M, seed=0):
    """Expected cost per expert for placement, from routing a calibration batch of the prefill shape
    (every rank routes its own, counts summed over ranks): a tensor-core tile of 256 rows decodes the
    expert's whole weight slice, so cost = tiles + rows / 4096."""
    import ctypes
    import torch
    import torch.distributed as dist
    from eva_b200 import _lib
    from eva_b200.experts import make_router
    lib = _lib.load()
    w, b = make_router(cfg, dev, seed)
    b = zipf_bias(cfg, b)
    shape = _lib.shape_of(cfg)
    ws = torch.zeros(lib.eva_moe_workspace_bytes(ctypes.byref(shape), M), dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(101 + rank)          # a calibration batch, not the timed inputs
    x = torch.randn(M, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
    idx = torch.empty(M, cfg.topk, dtype=torch.int32, device=dev)
    wt = torch.empty(M, cfg.topk, device=dev)
    _lib.check(lib.eva_moe_route(ctypes.byref(shape), x.data_ptr(), 1, M, w.data_ptr(), b.data_ptr(), None,
                                 idx.data_ptr(), wt.data_ptr(), ws.data_ptr(), ws.numel(),
                                 torch.cuda.current_stream(dev).cuda_stream), "route")
    rows = torch.bincount(idx.view(-1).long(), minlength=cfg.n_experts).to(torch.float64)
    if dist.is_initialized():
        dist.all_reduce(rows)
    rows = rows.cpu().numpy()
    del ws
    torch.cuda.empty_cache()
    return -(-rows // 256) + rows / 4096.0


def _max_over_ranks(v, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _max_min_over_ranks(vals, dev):
    """Element-wise (max, min) over ranks of a list of floats."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    hi, lo = t.clone(), -t
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    dist.all_reduce(lo, op=dist.ReduceOp.MAX)
    return hi.tolist(), (-lo).tolist()


def _phase_split(ep, inputs, n, dev, **kw):
    """Per-phase device time of n extra EP steps (after the timed ones), mean ms per step on each rank,
    as {phase: {"max_rank": ms, "min_rank": ms}}: which phase the step time goes to, and how unevenly
    (wait = until every peer's rows arrived, combine = until every peer's partials arrived + the sum)."""
    import torch
    runs = []
    for i in range(n):
        ph = []
        ep.forward(inputs[i % len(inputs)], phases=ph, **kw)
        runs.append(ph)
    torch.cuda.synchronize()
    names = [nm for nm, _ in runs[0][1:]]
    mean = [statistics.mean(r[j][1].elapsed_time(r[j + 1][1]) for r in runs) for j in range(len(names))]
    hi, lo = _max_min_over_ranks(mean, dev)
    return {nm: {"max_rank": h, "min_rank": l} for nm, h, l in zip(names, hi, lo)}


def _placement_balance(allidx, owner, world):
    """Routed (token, k) slots and distinct experts per rank per step, from the gathered routes
    [steps, world, M, k]: max / min over ranks of the per-step means."""
    import torch
    own = owner[allidx]                                     # [steps, world, M, k] owning rank
    slots = [float((own == r).sum()) / allidx.shape[0] for r in range(world)]
    distinct = [statistics.mean(int((owner[allidx[i].unique()] == r).sum()) for i in range(allidx.shape[0]))
                for r in range(world)]
    return {"slots_per_step_max_rank": max(slots), "slots_per_step_min_rank": min(slots),
            "slots_max_over_mean": max(slots) / max(1e-9, statistics.mean(slots)),
            "distinct_experts_per_step_max_rank": max(distinct), "distinct_experts_per_step_min_rank": min(distinct)}


def ep_bench(args, cfg, dev, rank, world, local):
    """N > 1: expert parallelism. Each rank holds n_experts / N experts (placed by expected load) and
    its own batch of tokens (weak scaling); the step is EPMoE.forward: route, dispatch (peer-memory
    stores, or NCCL with --ep-transport nccl), shared + local experts, combine."""
    import dataclasses
    import numpy as np
    import torch
    import torch.distributed as dist
    from eva_b200.ep import EPMoE, ExpertPlacement
    from eva_b200.experts import make_layer

    pl = ExpertPlacement.balanced(measured_load(cfg, dev, rank, args.prefill_tokens), world)
    layer = make_layer(cfg, dev, seed=0, experts=pl.experts_of(rank))
    owner = torch.as_tensor(pl.owner, dtype=torch.int64)
    M = args.batch
    steps, warmup = args.steps, max(3, args.warmup)
    nb = steps + warmup
    routed_rec = 3 * cfg.hidden * cfg.inter * cfg.bits // 8 + 6 * (cfg.hidden + cfg.inter)
    shared_rec = (3 * cfg.hidden * cfg.shared_inter * cfg.shared_bits // 8 + 6 * (cfg.hidden + cfg.shared_inter)
                  if cfg.shared_inter else 0)
    line = None
    if not args.prefill_only:
        ep = EPMoE(layer, pl, max_tokens=M, mode="fixed", transport=args.ep_transport)
        g = torch.Generator(device=dev)
        g.manual_seed(1 + rank)
        xs = torch.randn(nb, M, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(M, cfg.hidden, dtype=torch.bfloat16, device=dev)
        idx_all = torch.empty(nb, M, cfg.topk, dtype=torch.int32, device=dev)
        clocks = ClockSampler(local).__enter__()
        clocks.wait_first()
        for i in range(warmup):
            ep.forward(xs[i], out=out, idx_out=idx_all[i])
        torch.cuda.synchronize()
        dist.barrier()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        torch.cuda.synchronize()
        dist.barrier()
        c_start = clocks.mark()
        evs[0].record()
        for i in range(steps):
            ep.forward(xs[warmup + i], out=out, idx_out=idx_all[warmup + i])
            evs[i + 1].record()
        torch.cuda.synchronize()
        time.sleep(0.06)
        c_end = clocks.mark()
        dist.barrier()
        ms_total = _max_over_ranks(evs[0].elapsed_time(evs[-1]), dev)
        step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
        st = ep.status()
        # algorithmic bytes of this rank: its experts that any rank's tokens selected, + the shared expert
        gathered = [torch.empty_like(idx_all) for _ in range(world)]
        dist.all_gather(gathered, idx_all)
        allidx = torch.stack(gathered, 1).cpu().to(torch.int64)          # [nb, world, M, k]
        U = [int(((owner[allidx[warmup + i].unique()] == rank)).sum()) for i in range(steps)]
        alg = [u * routed_rec + shared_rec for u in U]
        achieved = statistics.mean(b / (ms * 1e-3) for b, ms in zip(alg, step_ms)) / 1e9
        achieved = _max_over_ranks(achieved, dev)
        # end to end: pinned host batch in, BF16 result out, inside the timed region
        xh = xs.cpu().pin_memory()
        dist.barrier()
        e2e_ms = _max_over_ranks(_e2e_pipelined(lambda xd, od: ep.forward(xd, out=od), xh, (M, cfg.hidden), dev,
                                                warmup, steps), dev)
        clocks.__exit__(None, None, None)
        clock_summary = clocks.summary(c_start, c_end)
        if not clock_summary["samples"]:
            clock_summary = dict(clocks.summary(), note="timed region shorter than the 50 ms sampling period; "
                                                        "samples from warm-up through e2e")
        st = int(_max_over_ranks(st, dev))
        phases = (_phase_split(ep, [xs[warmup + i] for i in range(steps)], min(steps, 20), dev, out=out)
                  if args.ep_transport == "peers" else None)
        balance = _placement_balance(allidx[warmup:], owner, world)
        peak, peak_kind = peaks()
        tokens = M * steps * world
        line = {
            "metric": METRIC, "value": tokens / (ms_total * 1e-3), "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_total / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 (EXL3 K3 weights decoded to fp16, fp32 accumulate), bf16 in/out",
            "data": "synthetic (seeded random EXL3 trellis codes, N(0,1) bf16 hidden states)",
            "config": {"workload": f"DeepSeek-{cfg.name.upper()} MoE layer decode (EXL3 K{cfg.bits}), batch {M} "
                                   f"tokens/step per GPU, expert parallel over {world} GPUs"
                                   + (" [small]" if args.small else ""),
                       "hidden": cfg.hidden, "experts": cfg.n_experts, "experts_per_gpu": layer.n_local,
                       "topk": cfg.topk, "inter": cfg.inter, "shared_inter": cfg.shared_inter, "bits": cfg.bits,
                       "batch": M, "global_batch": M * world, "parallelism": f"ep{world}",
                       "exchange": EXCHANGE[args.ep_transport],
                       "l2": "inputs larger than L2 (4.24 GB experts over the ranks, new routes every step)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "frac_of_spec": achieved / HBM_SPEC_GBS,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole EP step per rank (bytes: this rank's selected experts + shared, "
                                   "max over ranks)",
                         "distinct_local_experts_per_step": statistics.mean(U)},
            "cpu_baseline": None,
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "copies": E2E_COPIES,
                    "h2d_bytes_per_step": M * cfg.hidden * 2,
                    "d2h_bytes_per_step": M * cfg.hidden * 2},
            "gpu_launches": (12 if args.ep_transport == "peers" else 9) * steps,
            "clocks": clock_summary,
            "device_status": st,
            "phase_ms_per_step": phases,
            "placement_balance": balance,
            "rank_evidence": "the peer-memory exchange makes no NCCL calls on the step (NCCL only for setup "
                             "and the max-over-ranks reductions): N busy GPUs show the ranks",
        }
        ep.close()
        del ep, xs
        torch.cuda.empty_cache()

    prefill = None
    if not args.no_prefill:
        P = args.prefill_tokens
        player = dataclasses.replace(layer, router_b=zipf_bias(cfg, layer.router_b))
        ep = EPMoE(player, pl, max_tokens=P, mode="exact", transport=args.ep_transport)
        g = torch.Generator(device=dev)
        g.manual_seed(11 + rank)
        xs = [torch.randn(P, cfg.hidden, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
        out = torch.empty(P, cfg.hidden, dtype=torch.bfloat16, device=dev)
        idx = torch.empty(P, cfg.topk, dtype=torch.int32, device=dev)
        for i in range(PREFILL_WARMUP):
            ep.forward(xs[i % 2], out=out, idx_out=idx)
        torch.cuda.synchronize()
        dist.barrier()
        psteps = max(1, min(steps, 10))
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(psteps):
            ep.forward(xs[i % 2], out=out)
        t1.record()
        torch.cuda.synchronize()
        pms = _max_over_ranks(t0.elapsed_time(t1) / psteps, dev)
        pst = int(_max_over_ranks(ep.status(), dev))
        pphases = _phase_split(ep, xs, 4, dev, out=out) if args.ep_transport == "peers" else None
        ep.forward(xs[0], out=out, idx_out=idx)
        gathered = [torch.empty_like(idx) for _ in range(world)]
        dist.all_gather(gathered, idx)
        pbalance = _placement_balance(torch.stack(gathered, 0)[None].cpu().to(torch.int64), owner, world)
        flop = 6.0 * cfg.hidden * (P * world * cfg.topk * cfg.inter + P * world * cfg.shared_inter)
        peak, kind = tensor_peak()
        achieved = flop / world / (pms * 1e-3) / 1e12
        prefill = {"metric": "moe_layer_prefill_tokens_per_s", "value": P * world / (pms * 1e-3), "unit": "tokens/s",
                   "tokens_per_step": P * world, "tokens_per_gpu": P, "ms_per_step": pms, "steps": psteps,
                   "parallelism": f"ep{world}", "device_status": pst,
                   "routing": f"router bias + {ZIPF_BETA} * log(rank^-{ZIPF_S}) (Zipf-skewed); experts placed on "
                              f"ranks by the routed load of a calibration batch (tiles + rows/4096 per expert)",
                   "exchange": EXCHANGE[args.ep_transport] if args.ep_transport == "peers" else
                               "exact splits (counts all-to-all + one host sync), grouped NCCL send/recv of rows, "
                               "all-to-all of FP32 partial sums back",
                   "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                                "frac": achieved / peak, "peak_kind": kind,
                                "kernel": "whole EP prefill step per rank (routed + shared expert FLOPs / N)"},
                   "phase_ms_per_step": pphases, "placement_balance": pbalance}
        ep.close()
        del ep
        torch.cuda.empty_cache()
    if line is None:
        line = prefill
    else:
        line["prefill"] = prefill
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


E2E_COPIES = ("every step: its batch copied from pinned host memory and its result read back into pinned host "
              "memory, inside the timed region, on a copy stream overlapping the compute (two buffer sets); "
              "the region ends after the last read-back")


def _e2e_pipelined(fwd, xh, out_shape, dev, warmup, steps):
    """End-to-end ms of `steps` steps through fwd(x_device, out_device): every step copies its batch
    from pinned host memory and reads its result back into pinned host memory, with two buffer sets so
    that the next batch's copy and this result's read (on a copy stream) overlap the compute, as a
    serving loop would. The timed region ends after the last result has reached the host."""
    import torch
    stream = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    xd = [torch.empty_like(xh[0], device=dev) for _ in range(2)]
    od = [torch.empty(out_shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    oh = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_read = [torch.cuda.Event() for _ in range(2)]

    def run(first, n):
        cs.wait_stream(stream)                         # the first copy starts after the start event
        with torch.cuda.stream(cs):
            xd[0].copy_(xh[first], non_blocking=True)
            ev_in[0].record(cs)
        for i in range(n):
            b = i & 1
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_read[b])          # od[b]'s previous result has been read back
            fwd(xd[b], od[b])
            ev_done[b].record(stream)
            with torch.cuda.stream(cs):
                if i + 1 < n:
                    if i >= 1:
                        cs.wait_event(ev_done[b ^ 1])  # xd[b ^ 1] no longer read by step i - 1
                    xd[b ^ 1].copy_(xh[first + i + 1], non_blocking=True)
                    ev_in[b ^ 1].record(cs)
                cs.wait_event(ev_done[b])
                oh[b].copy_(od[b], non_blocking=True)
                ev_read[b].record(cs)
        stream.wait_stream(cs)

    run(0, warmup)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(warmup, steps)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def _graph_replay_ms(launch, stream, nb, warmup, steps):
    """ms per step of the decode step replayed from CUDA graphs: launch(i, s) queues batch i's step
    on stream s; one graph is captured per batch, then batches warmup .. warmup + steps - 1 are
    replayed back to back on `stream` between two events (the eager timed region's batches)."""
    import torch
    side = torch.cuda.Stream(stream.device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        launch(0, side)                    # once outside capture
    stream.wait_stream(side)
    torch.cuda.synchronize()
    graphs = []
    for i in range(nb):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch(i, torch.cuda.current_stream(stream.device))
        graphs.append(g)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for i in range(warmup):
            graphs[i].replay()
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(steps):
            graphs[warmup + i].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del graphs
    return ms


def _dma_h2d_gbs(dev, nbytes=256 << 20):
    """Pinned host -> device rate of one cudaMemcpyAsync (the copy engine), for context beside the
    cache's device-side copy kernel."""
    import torch
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dst.copy_(src, non_blocking=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(4):
        dst.copy_(src, non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    return 4 * nbytes / (a.elapsed_time(b) * 1e-3) / 1e9


def stack_bench(args, cfg, dev, rank, world, local):
    """Config 5: a decode stream of batch --batch per rank through --stack-layers layers, experts
    sharded over the ranks (EPMoE, peer-memory exchange). With --residency r < 1 only r of each rank's
    experts (over all layers) have device slots: by default one ExpertPool per rank shared by the
    layers (needed experts planned and copied from pinned host memory by the device, the next layer's
    predicted experts prefetched on a side stream under the current layer), with --staging host the
    host-managed per-layer ExpertResidency. The cached run is followed by the same stack fully
    resident, which gives the exposed staging time (step time difference) and so the fraction of the
    staging work that ran hidden under compute."""
    import math
    import torch
    import torch.distributed as dist
    from eva_b200.ep import EPMoE, ExpertPlacement
    from eva_b200.experts import make_layer
    from eva_b200.residency import ExpertPool, ExpertResidency
    from eva_b200.stack import MoEStack, make_norms

    L, M = args.stack_layers, args.batch
    pl = ExpertPlacement.balanced(zipf_load(cfg), world)
    mine = pl.experts_of(rank)
    cached = args.residency < 1.0
    ram_limited = False
    if cached:
        # every rank pins its experts of every layer in host memory
        rec = 3 * cfg.hidden * cfg.inter * cfg.bits // 8 + 6 * (cfg.hidden + cfg.inter)
        per_layer = len(mine) * (rec + 4096) * int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
        avail = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
        fit = int(0.7 * avail // per_layer)
        if world > 1:
            fit = int(_max_min_over_ranks([fit], dev)[1][0])
        if L <= 0:              # the largest layer count the host memory of the node holds
            L, ram_limited = min(fit, 58), fit < 58
        if L > fit or L < 1:
            raise SystemExit(f"--residency {args.residency}: {L * per_layer / 2**30:.0f} GiB of pinned host memory over "
                             f"the node's ranks, {avail / 2**30:.0f} GiB available; at most {fit} layers")
    elif L <= 0:
        L = 58
    pooled = cached and args.staging == "device"
    steps, warmup = args.steps, max(3, args.warmup)
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    xs = torch.randn(steps + warmup, M, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(M, cfg.hidden, dtype=torch.bfloat16, device=dev)
    norms = make_norms(L, cfg.hidden, dev, seed=5)

    def run(layers, timed_start=None):
        stack = MoEStack(layers, norms)
        for i in range(warmup):
            stack.forward(xs[i], out=out)
        torch.cuda.synchronize()
        if timed_start is not None:
            timed_start()
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        t0.record()
        for i in range(steps):
            stack.forward(xs[warmup + i], out=out)
        t1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
        st = 0
        for lay in layers:
            st |= lay.status()
        return t0.elapsed_time(t1), wall, st

    def made(li):
        lay = make_layer(cfg, dev, seed=1000 + li, experts=mine)
        return dataclasses_replace(lay, router_b=zipf_bias(cfg, lay.router_b))

    t_build = time.perf_counter()
    hosts, stats = [], None
    if cached:
        for li in range(L):
            lay = made(li)
            hosts.append(lay.host_copy(pinned=True))
            del lay
        if pooled:
            n_slots = max(len(mine), math.ceil(args.residency * L * len(mine)))
            pool = ExpertPool(dev, n_slots, hosts[0].record_bytes, max_layers=L, timing=True)
            pls = [pool.add_layer(h) for h in hosts]
            for li in range(L):
                pls[li].next = pls[(li + 1) % L]     # the last layer prefetches the next step's first
            layers = [EPMoE(h, pl, max_tokens=M, residency=r) for h, r in zip(hosts, pls)]
        else:
            n_slots = max(1, math.ceil(args.residency * len(mine)))
            residencies = [ExpertResidency(h, n_slots, dev) for h in hosts]
            layers = [EPMoE(h, pl, max_tokens=M, residency=r) for h, r in zip(hosts, residencies)]
    else:
        layers = [EPMoE(made(li), pl, max_tokens=M) for li in range(L)]
    t_build = time.perf_counter() - t_build

    b0 = [0]

    def timed_start():      # counters cover the timed steps only
        if pooled:
            b0[0] = pool.bytes_copied()
            pool.staging_ms()
        elif cached:
            for r in residencies:
                r.stats.update(hits=0, misses=0, h2d_bytes=0)

    ms, wall, st = run(layers, timed_start)
    resident_ms = None
    if pooled:
        h2d = pool.bytes_copied() - b0[0]
        stg = pool.staging_ms()
        st |= pool.status()
        stats = {"kind": "device expert cache (ExpertPool): one pool per GPU shared by the layers",
                 "slots_per_gpu": n_slots, "slots_per_gpu_if_resident": L * len(mine),
                 "h2d_bytes_per_step": h2d / steps,
                 "plan_ms_per_step": stg["plan"] / steps,
                 "miss_copy_ms_per_step": stg["copy"] / steps,
                 "prefetch_ms_per_step": stg["prefetch"] / steps,
                 "h2d_gbs_of_copy_launches": h2d / max(1e-9, stg["copy"] + stg["prefetch"]) / 1e6,
                 "h2d_gbs_copy_engine_256mb": _dma_h2d_gbs(dev)}
    elif cached:
        h2d = sum(r.stats["h2d_bytes"] for r in residencies)
        stats = {"kind": "host-managed per-layer residency (ExpertResidency)", "slots_per_layer": n_slots,
                 "h2d_bytes_per_step": h2d / steps, "misses": sum(r.stats["misses"] for r in residencies),
                 "hits": sum(r.stats["hits"] for r in residencies)}
    if cached:
        # the same stack with every expert resident (if the device holds it): exposed staging time
        for lay in layers:
            lay.close()
        del layers
        if pooled:
            del pls, pool
        else:
            del residencies
        torch.cuda.empty_cache()
        full_bytes = L * sum(h.storage.numel() for h in hosts[:1])
        fits = full_bytes < 0.8 * torch.cuda.mem_get_info(dev)[0]
        if world > 1:
            fits = _max_over_ranks(0 if fits else 1, dev) == 0
        if fits:
            layers = [EPMoE(h.to(dev), pl, max_tokens=M) for h in hosts]
            resident_ms, _, st_r = run(layers)
            st |= st_r
    if world > 1:
        ms = _max_over_ranks(ms, dev)
        st = int(_max_over_ranks(st, dev))
        if resident_ms is not None:
            resident_ms = _max_over_ranks(resident_ms, dev)
        if stats is not None:
            for k in [k for k in stats if k.startswith(("h2d", "plan", "miss", "prefetch"))]:
                stats[k] = _max_over_ranks(stats[k], dev)
    if stats is not None:
        stats["resident_ms_per_step"] = None if resident_ms is None else resident_ms / steps
        if resident_ms is not None:
            exposed = max(0.0, (ms - resident_ms) / steps)
            stats["exposed_staging_ms_per_step"] = exposed
            if pooled:
                total = sum(stats[k] for k in ("plan_ms_per_step", "miss_copy_ms_per_step", "prefetch_ms_per_step"))
                stats["staging_hidden_fraction"] = None if total <= 0 else max(0.0, 1.0 - exposed / total)
        stats["note"] = ("max over ranks; exposed = cached minus resident step time; hidden fraction = 1 - exposed / "
                         "device time of all staging launches (plans, miss copies, prefetches)")
    line = {"metric": "moe_stack_decode_tokens_per_s", "value": M * world * steps / (ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (EXL3 K3), bf16 in/out, fp32 residual",
            "data": "synthetic (seeded random EXL3 trellis codes; Zipf-skewed router bias)",
            "config": {"workload": f"config 5: {L} DeepSeek-{cfg.name.upper()} MoE layers, RMSNorm + residual, "
                                   f"attention stubbed, decode batch {M} tokens/step per GPU, expert parallel over "
                                   f"{world} GPUs", "layers": L, "batch": M, "global_batch": M * world,
                       "experts_per_gpu_per_layer": len(mine), "residency": args.residency,
                       "staging": args.staging if cached else None,
                       "layers_limited_by_host_ram": ram_limited,
                       "parallelism": f"ep{world}", "exchange": EXCHANGE["peers"]},
            "residency_stats": stats,
            "wall_ms_per_step": 1e3 * wall / steps, "build_s": t_build, "device_status": st}
    if rank == 0:
        print(json.dumps(line), flush=True)
    for lay in layers:
        lay.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


MICRO_VARIANTS = {
    0: "mma.sync decode of the fused decode kernel (4 words + 2 funnel shifts per lane-tile, mul1 byte sums, "
       "fp16 pairs, mma.m16n8k16)",
    1: "two-word decode -> mul1 products -> tcgen05.st into TMEM (kind::i8 operand form), no MMA",
    2: "two-word decode -> raw codebook fp16 -> tcgen05.st into TMEM (kind::f16 operand form), no MMA",
    3: "variant 1 + tcgen05.mma.kind::i8 with A in TMEM (M 128, N 16), 7-slot TMEM ring, one issuing thread",
    4: "variant 2 + tcgen05.mma.kind::f16 with A in TMEM, same ring",
    5: "variant 1 without the ALU/FMA split of the window extraction",
    6: "two-word decode (2 words + 2 funnel shifts per lane-tile) + mma.m16n8k16, pairs packed by IMAD",
    7: "variant 6 with pairs packed by PRMT",
    8: "variant 7 with 2 windows extracted as multiply + shift (FMA pipe)",
    9: "variant 6 with 2 windows extracted as multiply + shift",
    10: "variant 7 with 4 windows extracted as multiply + shift",
    11: "variant 8 with a stage's bookkeeping around each pass (B fragments from shared memory, mbarrier arrive + "
        "wait, warp barrier)",
    12: "the fused kernel's pipeline: a producer warp streams 32 trellis rows + 8 B rows per stage from a 1 GB buffer "
        "(HBM) into a 4-stage ring, 16 decoding warps as variant 8",
    13: "variant 12 with a 32 MB source (resident in L2)",
    14: "variant 12 with 5 ring stages",
    15: "variant 12 with decoders not waiting for the data (shared-memory contention only)",
    16: "variant 12 with one contiguous copy per stage instead of 32 row copies",
    17: "variant 12 with one 2-D tensor copy (TMA tensor map over the strided rows) per stage",
    18: "variant 12 with the stage copied by cp.async 16-byte copies from the producer warp",
    19: "variant 8 with the byte sum left to 8-bit MMAs: each weight's mul1 product as 4 u8 K positions, "
        "activations as two 8-bit digits (m16n8k32 u8 x s8 and u8 x u8), 4 MMAs per tile, no dp4a or packing",
}


def decode_microbench(args):
    """One JSON line: decoded weights per SM clock of each decode design (eva_decode_microbench)."""
    import ctypes
    import torch
    from eva_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    hbm, hbm_kind = peaks()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    clocks = ClockSampler(0).__enter__()
    clocks.wait_first()
    c0 = clocks.mark()
    res = {}
    for bits in (3, 2, 4):
        for v in sorted(MICRO_VARIANTS):
            out = (ctypes.c_double * 5)()
            _lib.check(lib.eva_decode_microbench(v, bits, 64, out, stream), "eva_decode_microbench")   # warm-up
            # about 50 ms per measurement
            iters = max(64, int(64 * 50.0 / max(out[4], 1e-3)))
            _lib.check(lib.eva_decode_microbench(v, bits, iters, out, stream), "eva_decode_microbench")
            res[f"K{bits}_v{v}"] = {"weights_per_sm_clock": out[0], "sm_clocks": out[1], "ms": out[4],
                                    "weights": out[2], "device_status": int(out[3])}
    time.sleep(0.06)
    c1 = clocks.mark()
    clocks.__exit__(None, None, None)
    cs = clocks.summary(c0, c1)
    f_ghz = (cs["sm_mhz"] or 1965.0) / 1000.0
    need = {b: hbm * 1e9 / (b / 8.0) / sms / (f_ghz * 1e9) for b in (2, 3, 4)}
    line = {"metric": "decode_loop_weights_per_sm_clock", "unit": "weights / SM / clock",
            "value": res["K3_v0"]["weights_per_sm_clock"],
            "config": {"workload": "EXL3 decode loop alone, trellis tiles resident in shared memory (no HBM), one "
                                   "CTA per SM, clock64 per CTA", "variants": MICRO_VARIANTS},
            "results": res,
            "hbm_rate_needs_weights_per_sm_clock": {f"K{b}": need[b] for b in need},
            "hbm_peak": {"gbs": hbm, "kind": hbm_kind, "sm_clock_ghz": f_ghz},
            "ceiling_frac_of_hbm": {k: r["weights_per_sm_clock"] / need[int(k[1])] for k, r in res.items()},
            "clocks": cs}
    print(json.dumps(line), flush=True)


def dataclasses_replace(obj, **kw):
    import dataclasses
    return dataclasses.replace(obj, **kw)


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.decode_microbench:
        return decode_microbench(args)
    import numpy as np
    import torch
    import torch.distributed as dist
    from eva_b200 import _lib
    from eva_b200.config import CONFIGS
    from eva_b200.experts import make_layer
    from eva_b200.runner import EvaMoE

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    cfg = CONFIGS[args.config]
    if args.small:
        cfg = cfg.with_(n_experts=64, n_group=8, topk_group=4)
    if args.stack:
        return stack_bench(args, cfg, dev, rank, world, local)
    if world > 1:
        return ep_bench(args, cfg, dev, rank, world, local)
    if args.prefill_only:
        layer = make_layer(cfg, dev, seed=0)
        res = prefill_measure(cfg, layer, dev, max(1, min(args.steps, 10)), PREFILL_WARMUP, args.prefill_tokens)
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    M = args.batch
    steps, warmup = args.steps, max(3, args.warmup)
    layer = make_layer(cfg, dev, seed=0)
    moe = EvaMoE(layer, max_rows=max(M, 8))
    stream = torch.cuda.current_stream(dev)
    nb = steps + warmup
    g = torch.Generator(device=dev)
    g.manual_seed(1 + rank)
    xs = torch.randn(nb, M, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(M, cfg.hidden, dtype=torch.bfloat16, device=dev)
    idx_all = torch.empty(nb, M, cfg.topk, dtype=torch.int32, device=dev)
    w_all = torch.empty(nb, M, cfg.topk, device=dev)
    # routes of every batch (for the algorithmic byte count; the timed steps route again)
    for i in range(nb):
        moe.forward(xs[i], out=out, idx_out=idx_all[i], w_out=w_all[i])
    torch.cuda.synchronize()
    if moe.status():
        raise RuntimeError(f"device status {moe.status():#x}")
    idx_host = idx_all.cpu().numpy()

    lib = _lib.load()
    import ctypes
    shape = moe.shape
    tables, shared = moe._tables, moe._shared
    ws = moe.workspace
    routed_rec = 3 * cfg.hidden * cfg.inter * cfg.bits // 8 + 6 * (cfg.hidden + cfg.inter)
    shared_rec = (3 * cfg.hidden * cfg.shared_inter * cfg.shared_bits // 8 + 6 * (cfg.hidden + cfg.shared_inter)
                  if cfg.shared_inter else 0)
    router_bytes = cfg.n_experts * cfg.hidden * 4 + cfg.n_experts * 4

    def step(i, ev=None):
        x = xs[i]
        rc = lib.eva_moe_route(ctypes.byref(shape), x.data_ptr(), 1, M, layer.router_w.data_ptr(),
                               layer.router_b.data_ptr(), None, idx_all[i].data_ptr(), w_all[i].data_ptr(),
                               ws.data_ptr(), ws.numel(), stream.cuda_stream)
        _lib.check(rc, "route")
        if ev is not None:
            ev[0].record(stream)
        rc = lib.eva_moe_experts(ctypes.byref(shape), x.data_ptr(), 1, M, idx_all[i].data_ptr(), 0,
                                 w_all[i].data_ptr(), tables, shared, ws.data_ptr(), ws.numel(), None,
                                 out.data_ptr(), stream.cuda_stream)
        _lib.check(rc, "experts")
        if ev is not None:
            ev[1].record(stream)

    clocks = ClockSampler(local).__enter__()
    clocks.wait_first()
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # settle: identical steps (cycling over the batches) for at least DECODE_SETTLE_S right before
    # the timed steps, so that the clocks sampled over settle + timed steps describe the timed
    # region (K steps of < 1 ms each are shorter than the sampler's period); timed on their own as
    # the sustained figure
    c_start = clocks.mark()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    settle_steps, w_settle = 0, time.perf_counter()
    s0.record(stream)
    while time.perf_counter() - w_settle < DECODE_SETTLE_S and settle_steps < DECODE_SETTLE_MAX:
        step(settle_steps % nb)
        settle_steps += 1
        if settle_steps % 64 == 0:
            torch.cuda.synchronize()   # keep the host from running far ahead of the device
    s1.record(stream)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    settle_ms = s0.elapsed_time(s1)
    if world > 1:
        dist.barrier()
    c_timed = clocks.mark()
    t0.record(stream)
    for i in range(steps):
        step(warmup + i, evs[i])
    t1.record(stream)
    torch.cuda.synchronize()
    time.sleep(0.06)   # let the sampler report the end of the region
    c_end = clocks.mark()
    if world > 1:
        dist.barrier()
    ms_total = t0.elapsed_time(t1)
    exp_ms = [a.elapsed_time(b) for a, b in evs]
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    st = moe.status()

    # ---- end to end through the public API with host buffers --------------------------------
    graph_ms = None
    if args.graph and world == 1:
        def launch(i, s):
            _lib.check(lib.eva_moe_route(ctypes.byref(shape), xs[i].data_ptr(), 1, M, layer.router_w.data_ptr(),
                                         layer.router_b.data_ptr(), None, idx_all[i].data_ptr(), w_all[i].data_ptr(),
                                         ws.data_ptr(), ws.numel(), s.cuda_stream), "route")
            _lib.check(lib.eva_moe_experts(ctypes.byref(shape), xs[i].data_ptr(), 1, M, idx_all[i].data_ptr(), 0,
                                           w_all[i].data_ptr(), tables, shared, ws.data_ptr(), ws.numel(), None,
                                           out.data_ptr(), s.cuda_stream), "experts")
        graph_ms = _graph_replay_ms(launch, stream, nb, warmup, steps)

    xh = xs.cpu().pin_memory()
    if world > 1:
        dist.barrier()
    e2e_ms = _e2e_pipelined(lambda xd, od: moe.forward(xd, out=od), xh, (M, cfg.hidden), dev, warmup, steps)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    clocks.__exit__(None, None, None)
    clock_summary = clocks.summary(c_start, c_end)
    clock_summary["window"] = (f"{settle_steps} identical untimed steps ({settle_ms:.0f} ms, no gap) immediately "
                               f"before the {steps} timed steps, and the timed steps; "
                               f"{clocks.summary(c_timed, c_end)['samples']} samples inside the timed steps alone")

    # ---- roofline of the fused experts launch -------------------------------------------------
    U = [len(np.unique(idx_host[warmup + i])) for i in range(steps)]
    alg_bytes = [u * routed_rec + shared_rec for u in U]
    achieved = statistics.mean(b / (ms * 1e-3) for b, ms in zip(alg_bytes, exp_ms)) / 1e9
    peak, peak_kind = peaks()
    traffic = None
    prof = ROOT / "profiles" / "experts_kernel_traffic.txt"
    if prof.exists():
        try:
            per_expert = float(prof.read_text().split("bytes_per_expert_record_equivalent:")[1].split()[0])
            traffic = per_expert * (statistics.mean(U) + (shared_rec / routed_rec if routed_rec else 0))
        except (IndexError, ValueError):
            traffic = None

    # the prefill leg before the CPU baseline: the GPU is still busy from the decode leg
    prefill = None
    if not args.no_prefill and world == 1:
        del moe
        torch.cuda.empty_cache()
        prefill = prefill_measure(cfg, layer, dev, max(1, min(steps, 10)), PREFILL_WARMUP, args.prefill_tokens)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the device layer's own records in host memory: every expert distinct, the same 4.24 GB
        host = layer.host_copy()
        xb = xs[:min(nb, 8)].cpu().view(torch.int16).numpy().view(np.uint16)
        threads = host_threads()
        cpu_sample(cfg, host, xb[0], threads)   # warm-up
        ts, n_tok = [], 0
        t_end = time.perf_counter() + 20.0
        while time.perf_counter() < t_end and len(ts) < len(xb):
            dt, n = cpu_sample(cfg, host, xb[len(ts)], threads)
            ts.append(dt)
            n_tok += n
        cpu = {"value": n_tok / sum(ts), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{len(ts)} whole batch-{M} steps of this run's inputs through this repository's float32 C "
                         f"port of the path (oracle/cpu_fast.c: FP32 router, top-{cfg.topk} routed experts + shared "
                         f"expert with the EXL3 dequantization fused into the GEMV), over the same "
                         f"{cfg.n_experts} distinct expert records as the GPU run; not the reference's own code, "
                         f"whose CPU expert path needs exllamav3 (not installed)"}

    tokens = M * steps * world
    line = {
        "metric": METRIC, "value": tokens / (ms_total * 1e-3), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms_total / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 (EXL3 K3 weights decoded to fp16, fp32 accumulate), bf16 in/out",
        "data": "synthetic (seeded random EXL3 trellis codes, N(0,1) bf16 hidden states)",
        "config": {"workload": f"DeepSeek-{cfg.name.upper()} MoE layer decode (EXL3 K{cfg.bits}), batch {M} tokens/step"
                               + (" [small]" if args.small else ""),
                   "hidden": cfg.hidden, "experts": cfg.n_experts, "topk": cfg.topk, "inter": cfg.inter,
                   "shared_inter": cfg.shared_inter, "bits": cfg.bits, "batch": M,
                   "parallelism": "replicas" if world > 1 else "single",
                   "l2": "inputs larger than L2 (4.24 GB experts, different routes every step)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "frac_of_spec": achieved / HBM_SPEC_GBS,
                     "traffic": traffic, "peak_kind": peak_kind, "kernel": "eva_moe_experts (permute + experts_kernel)",
                     "alg_bytes_per_launch": statistics.mean(alg_bytes), "launch_ms": statistics.mean(exp_ms),
                     "distinct_experts_per_step": statistics.mean(U),
                     "distinct_experts_by_batch": [int(len(np.unique(idx_host[i]))) for i in range(nb)]},
        "cpu_baseline": cpu,
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "copies": E2E_COPIES,
                    "h2d_bytes_per_step": M * cfg.hidden * 2,
                "d2h_bytes_per_step": M * cfg.hidden * 2},
        "gpu_launches": 4 * steps,
        "clocks": clock_summary,
        "sustained": {"value": M * settle_steps / (settle_ms * 1e-3), "unit": UNIT, "steps": settle_steps,
                      "ms_per_step": settle_ms / max(settle_steps, 1),
                      "note": "the settle steps before the timed region, timed as one block (>= 1 s)"},
        "device_status": st,
        **({"graph": {"value": M / (graph_ms * 1e-3), "unit": UNIT, "ms_per_step": graph_ms,
                      "note": "the timed steps' batches replayed from CUDA graphs (one captured per batch: "
                              "router, top-k, permutation, experts), device-timed; value above is eager "
                              "launches"}} if graph_ms is not None else {}),
        "prefill": prefill,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
