"""The CPU oracle against the reference's own golden vectors (tests/golden/, made by make_golden.py)
and against independent restatements. CPU only."""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_mul1_integer_matches_reference(oracle):
    g = json.loads((GOLDEN / "mul1.json").read_text())
    L = oracle.lib()
    assert L.eo_mul1_integer(0x1234) == -85          # known answer computed by the reference
    for s, v in zip(g["states"], g["mul1_integer"]):
        assert L.eo_mul1_integer(s) == v
    # the codebook scale of the reference is the fp16 constant 0x1eee
    assert g["MUL1_SCALE"] == float(np.array([0x1EEE], np.uint16).view(np.float16)[0])


def test_codebook_single_fp16_rounding(oracle):
    """All 65536 states: fp16(round((1024 + bytesum) * c0 + c1)) computed independently by numpy."""
    c0 = np.float64(np.array([0x1EEE], np.uint16).view(np.float16)[0])
    c1 = np.float64(np.array([0xC931], np.uint16).view(np.float16)[0])
    st = np.arange(65536, dtype=np.uint64)
    prod = (st * 0x83DCD12D) & 0xFFFFFFFF
    bs = sum(((prod >> s) & 255) for s in (0, 8, 16, 24)).astype(np.float64)
    ref = ((1024 + bs) * c0 + c1).astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.mul1_table(), ref)
    # the codebook is the integer identity times the scale, shifted by the constant
    # (1024 * c0 + c1) + 510 * c0 = -476 / 2^18, then rounded once to fp16 (half an ulp <= 2^-10)
    ints = bs - 510
    vals = ref.view(np.float16).astype(np.float64)
    offset = 1024 * c0 + c1 + 510 * c0
    assert offset == -476 / 2**18
    assert np.max(np.abs(vals - (ints * c0 + offset))) <= 2.0**-10


@pytest.mark.parametrize("K", [2, 3, 4])
def test_tile_window_two_word_extraction(oracle, K):
    rng = np.random.default_rng(K)
    for _ in range(20):
        tile = rng.integers(0, 2**32, 8 * K, dtype=np.uint64).astype(np.uint32)
        for p in range(256):
            assert oracle.tile_state(tile, K, p) == oracle.tile_state(tile, K, p, fast=True)


def test_tile_position_map_is_a_bijection(oracle):
    seen = {oracle.tile_pos(p) for p in range(256)}
    assert len(seen) == 256 and all(0 <= k < 16 and 0 <= n < 16 for k, n in seen)
    # lane l's first two positions are the mma.m16n8k16 fragment pair (k = 2(l%4), n = l/4)
    for lane in range(32):
        assert oracle.tile_pos(8 * lane) == (2 * (lane % 4), lane // 4)
        assert oracle.tile_pos(8 * lane + 1) == (2 * (lane % 4) + 1, lane // 4)


@pytest.mark.parametrize("K", [2, 3, 4])
def test_dequant_definition(oracle, K):
    """eo_dequant equals the bit-by-bit definition: state window -> codebook -> (k, n) placement."""
    rng = np.random.default_rng(10 + K)
    tr = rng.integers(-32768, 32768, (3, 2, 16 * K), dtype=np.int64).astype(np.int16)
    w = oracle.dequant(tr, K)
    table = oracle.mul1_table()
    words = tr.view(np.uint32).reshape(3, 2, 8 * K)
    for kt in range(3):
        for nt in range(2):
            for p in range(0, 256, 7):
                k, n = oracle.tile_pos(p)
                st = oracle.tile_state(words[kt, nt], K, p)
                assert w[kt * 16 + k, nt * 16 + n] == table[st]


def test_hadamard_is_orthonormal(oracle):
    eye = np.eye(128)
    h = oracle.hadamard128(eye)
    assert np.allclose(h @ h.T, eye, atol=1e-12)
    assert np.allclose(np.abs(h), 1 / np.sqrt(128))
    # natural order: H[i][j] = (-1)^popcount(i & j) / sqrt(128)
    i, j = np.meshgrid(np.arange(128), np.arange(128), indexing="ij")
    sign = (-1.0) ** np.vectorize(lambda v: bin(v).count("1"))(i & j)
    assert np.allclose(h, sign / np.sqrt(128))


def test_linear_matches_dense_restatement(oracle):
    rng = np.random.default_rng(3)
    fin, fout, K = 256, 128, 3
    tr = rng.integers(-32768, 32768, (fin // 16, fout // 16, 16 * K), dtype=np.int64).astype(np.int16)
    w16 = oracle.dequant(tr, K)
    suh = (rng.choice([-1.0, 1.0], fin) * rng.uniform(0.75, 1.25, fin)).astype(np.float16).view(np.uint16)
    svh = (rng.choice([-0.02, 0.02], fout)).astype(np.float16).view(np.uint16)
    x = rng.standard_normal((3, fin))
    y = oracle.linear(x, suh, svh, w16, round_in=False)
    W = w16.view(np.float16).astype(np.float64)
    xr = oracle.hadamard128(x * suh.view(np.float16).astype(np.float64))
    ref = oracle.hadamard128(xr @ W) * svh.view(np.float16).astype(np.float64)
    assert np.allclose(y, ref, rtol=1e-10, atol=1e-10)


def test_run_tables_match_reference(oracle):
    data = json.loads((GOLDEN / "run_tables.json").read_text())
    n = 0
    for c in data["cases"]:
        sel = np.array(c["indices"], dtype=np.int64)
        w = np.array(c["weights"], dtype=np.float32)
        if c["table"] is not None:
            assert oracle.run_table(sel, w, c["capacity"]) == c["table"], c["module"]
            n += 1
        # runs view: expert + slots of each run
        t = oracle.run_table(sel, w, max(c["capacity"], len(sel)))
        S = max(c["capacity"], len(sel)) * sel.shape[1]
        runs = []
        for r in range(t[0]):
            a, b = t[2 + r], t[2 + r + 1]
            slots = t[2 + S + 1 + a: 2 + S + 1 + b]
            runs.append({"expert": int(sel.ravel()[slots[0]]), "slots": slots})
        assert runs == c["runs"]
    assert n >= 10


def test_sqrtsoftplus_route_matches_reference(oracle):
    from eva_b200.config import REF_NATIVE
    g = np.load(GOLDEN / "route_sqrtsoftplus.npz")
    logits = oracle.router_logits(g["x_f16"].astype(np.float32), g["gate_w"])
    assert np.allclose(logits, g["logits"], rtol=1e-5, atol=1e-5)
    idx, w = oracle.route(g["logits"], g["gate_b"], REF_NATIVE)
    assert np.array_equal(idx, g["indices"])
    assert np.allclose(w, g["weights"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("limit", [0, 10, 2.5])
def test_swiglu_matches_reference(oracle, limit):
    g = np.load(GOLDEN / "swiglu.npz")
    L = oracle.lib()
    gate, up = g["gate"].astype(np.float64), g["up"].astype(np.float64)
    out = np.vectorize(lambda a, b: L.eo_act(a, b, float(limit), 1))(gate, up)
    assert np.allclose(out, g[f"out_{limit}"], rtol=2e-6, atol=2e-6)


def test_clamp_after_differs_from_swiglu_only_above_limit(oracle):
    L = oracle.lib()
    assert L.eo_act(12.0, 3.0, 10.0, 0) == pytest.approx(30.0)               # min(silu(12), 10) * 3
    assert L.eo_act(12.0, 3.0, 10.0, 1) == pytest.approx(10 / (1 + np.exp(-10)) * 3)
    assert L.eo_act(1.5, -20.0, 10.0, 0) == pytest.approx(L.eo_act(1.5, -20.0, 10.0, 1))


def test_rmsnorm_matches_reference_rms(oracle):
    """model.py:968-970 rms on FP32 and BF16 rows (tests/golden/rms.npz)."""
    g = np.load(GOLDEN / "rms.npz")
    w = oracle.bf16_to_f32(g["w_bf16"].view(np.uint16))
    got = oracle.rmsnorm(g["x"], w, float(g["eps"]))
    np.testing.assert_allclose(got, g["out_f32"], rtol=2e-6, atol=1e-6)
    xb = oracle.f32_to_bf16(g["x"])
    got_b = oracle.f32_to_bf16(oracle.rmsnorm(oracle.bf16_to_f32(xb), w, float(g["eps"])))
    ref_b = g["out_bf16"].view(np.uint16)
    diff = np.abs(got_b.astype(np.int32) - ref_b.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.99


def _ascending(idx, w):
    order = np.argsort(idx, axis=-1, kind="stable")
    return np.take_along_axis(idx, order, -1).astype(np.int64), np.take_along_axis(w, order, -1)


@pytest.mark.parametrize("fixture,name", [("route_v3_sigmoid.npz", "v3"), ("route_v2lite_softmax.npz", "v2-lite")])
def test_published_gating_matches_transformers(oracle, fixture, name):
    """Sigmoid group-limited (DeepSeek-V3) and softmax greedy (DeepSeek-V2-Lite) routing against the
    transformers 5.5.0 gating functions (make_route_pins.py): same expert sets, weights to float32
    rounding. The oracle orders each row by selection score, transformers leaves it unsorted, so both
    are compared in ascending expert order."""
    from eva_b200.config import CONFIGS
    cfg = CONFIGS[name]
    g = np.load(GOLDEN / fixture)
    bias = g["bias"] if "bias" in g.files else np.zeros(cfg.n_experts, np.float32)
    idx, w = _ascending(*oracle.route(g["logits"], bias, cfg))
    assert np.array_equal(idx, g["indices"])
    np.testing.assert_allclose(w, g["weights"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("name", ["v3", "v2-lite"])
def test_published_gating_matches_transformers_live(oracle, name):
    """The same comparison on 4096 fresh rows, calling transformers directly when it is installed."""
    pytest.importorskip("transformers")
    sys.path.insert(0, str(GOLDEN))
    import make_route_pins as P
    from eva_b200.config import CONFIGS
    cfg = CONFIGS[name]
    if name == "v3":
        logits, bias = P.v3_inputs(4096, cfg.n_experts, seed=77)
        ref_idx, ref_w = P.transformers_v3_route(logits, bias)
    else:
        logits, bias = P.v2lite_inputs(4096, cfg.n_experts, seed=78), np.zeros(cfg.n_experts, np.float32)
        ref_idx, ref_w = P.transformers_v2lite_route(logits)
    idx, w = _ascending(*oracle.route(logits, bias, cfg))
    same = (idx == ref_idx).all(-1)
    np.testing.assert_allclose(w[same], ref_w[same], rtol=2e-6, atol=1e-7)
    # Rows whose expert sets differ must be ties: torch.topk breaks equal scores in no fixed order
    # (the oracle takes the lower expert id), and torch's CPU sigmoid is not correctly rounded (the
    # oracle's is), which moves a score by 1 ulp. The selection scores of both sets then agree.
    choice = (oracle.scores(logits, cfg.router) + (bias if cfg.router != "softmax" else 0)).astype(np.float32)
    diff = np.where(~same)[0]
    assert len(diff) <= max(2, len(idx) // 1000)
    for r in diff:
        a, b = np.sort(choice[r, idx[r]]), np.sort(choice[r, ref_idx[r]])
        np.testing.assert_allclose(a, b, rtol=3e-7, atol=0)
