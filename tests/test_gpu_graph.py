"""EvaMoE.forward captured in a CUDA graph and replayed.

The reference's coop binding refuses graph capture (runtime/ds41/csrc/moe_coop2048/binding.cu:83-85);
this library's forward path issues only stream-ordered work (router, top-k, permutation, experts; the
counters each launch needs are zeroed by the permutation of the same call) and no host
synchronisation, so a serving loop can capture a whole layer step once and replay it with new inputs
copied into the captured input buffer. Each replay is compared with an eager call on the same input:
decode and prefill (tensor-core) paths of the DeepSeek-V2-Lite shape, and the DeepSeek-V3 decode
shape of the bench.
"""
import numpy as np
import pytest
import torch

from eva_b200 import config as C
from eva_b200.experts import make_layer
from eva_b200.runner import EvaMoE

DEV = "cuda"


def _close(out, ref, rel=3e-3, cos=0.99999):
    out = out.double().cpu().numpy().ravel()
    ref = ref.double().cpu().numpy().ravel()
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    c = float(out @ ref / (np.linalg.norm(out) * np.linalg.norm(ref)))
    assert err <= rel and c >= cos, f"max-rel-err {err:.3e} cosine {c:.7f}"


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,M", [(C.V2_LITE, 8), (C.V2_LITE, 256), (C.V3, 8)],
                         ids=["v2-lite-decode-8", "v2-lite-prefill-256", "v3-decode-8"])
def test_forward_replays_from_a_cuda_graph(cfg, M):
    layer = make_layer(cfg, DEV, seed=31)
    moe = EvaMoE(layer, max_rows=max(M, 64))
    gen = torch.Generator().manual_seed(5)
    x_static = torch.randn(M, cfg.hidden, generator=gen).to(torch.bfloat16).to(DEV)
    out_static = torch.empty(M, cfg.hidden, dtype=torch.bfloat16, device=DEV)
    # warm-up on a side stream before capture (library attributes and driver entry points resolved)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        moe.forward(x_static, out=out_static)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        moe.forward(x_static, out=out_static)
    for _ in range(3):
        x_new = torch.randn(M, cfg.hidden, generator=gen).to(torch.bfloat16).to(DEV)
        x_static.copy_(x_new)
        g.replay()
        got = out_static.clone()
        ref = moe.forward(x_new)                       # eager, same stream, after the replay
        torch.cuda.synchronize()
        assert moe.status() == 0
        assert torch.isfinite(got.float()).all()
        _close(got, ref)
    del g
    del moe, layer
    torch.cuda.empty_cache()
