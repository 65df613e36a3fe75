"""Tensor-memory layouts the TMEM-operand decode relies on, checked on the B200 (-m gpu).

* The 16x256b shape of tcgen05.st puts register i of thread t of a warp at TMEM lane
  16 half + t / 4 + 8 (i / 2 % 2) of the warp's 32 lanes, column 8 (i / 4) + 2 (t % 4) + i % 2: the
  mma.sync fragment layout, so a lane's decoded 16 x 16 tile positions land in TMEM rows n and
  columns k of the weight tile without any exchange between lanes (eva_b200/csrc/decode_tc.cuh).
* tcgen05.mma.kind::i8 (u8 x s8 -> s32) and kind::f16 with the A operand read from TMEM and B from
  128B-swizzled shared memory compute A x B^T (M 128, N 16).
* The pair MMA (tcgen05.mma.cta_group::2) places its accumulators as the prefill kernels read them,
  for full (M = 256) and half-height (M = 128) tiles.
* The decode micro-benchmark runs every variant to completion with a clean device status.
"""
import ctypes

import numpy as np
import pytest
import torch

from eva_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _selftest(what, a=None, b=None, shape=(128, 16)):
    lib = _lib.load()
    out = torch.zeros(int(np.prod(shape)), dtype=torch.int32, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.eva_tc_selftest(what, None if a is None else a.data_ptr(), None if b is None else b.data_ptr(),
                             out.data_ptr(), st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "eva_tc_selftest")
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    return out.cpu().numpy().view(np.uint32).reshape(shape)


def test_tmem_16x256b_store_layout():
    got = _selftest(0)
    want = np.zeros((128, 16), np.uint32)
    for w in range(4):
        for half in range(2):
            for t in range(32):
                for i in range(8):
                    lane = 32 * w + 16 * half + t // 4 + 8 * ((i // 2) % 2)
                    col = 8 * (i // 4) + 2 * (t % 4) + i % 2
                    want[lane, col] = (half << 12) | (t << 4) | i
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)[:8]
        pytest.fail("16x256b mapping differs at (lane, col) " + ", ".join(
            f"({l},{c}): got half {got[l, c] >> 12} t {(got[l, c] >> 4) & 255} r {got[l, c] & 15}" for l, c in bad))


def test_umma_i8_with_a_in_tmem():
    rng = np.random.default_rng(0)
    a = rng.integers(0, 256, (128, 32), dtype=np.uint8)
    b = rng.integers(-128, 128, (16, 32), dtype=np.int8)
    got = _selftest(1, torch.tensor(a.view(np.uint32).reshape(-1).view(np.int32), device=DEV),
                    torch.tensor(b.view(np.uint32).reshape(-1).view(np.int32), device=DEV)).view(np.int32)
    want = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(got.astype(np.int64), want)


def test_umma_f16_with_a_in_tmem():
    rng = np.random.default_rng(1)
    a = rng.standard_normal((128, 16)).astype(np.float16)
    b = rng.standard_normal((16, 16)).astype(np.float16)
    got = _selftest(2, torch.tensor(a.view(np.uint32).reshape(-1).view(np.int32), device=DEV),
                    torch.tensor(b.view(np.uint32).reshape(-1).view(np.int32), device=DEV)).view(np.float32)
    want = a.astype(np.float64) @ b.astype(np.float64).T
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("variant", list(range(20)))
def test_decode_microbench_runs(variant):
    lib = _lib.load()
    out = (ctypes.c_double * 5)()
    _lib.check(lib.eva_decode_microbench(variant, 3, 64, out, torch.cuda.current_stream().cuda_stream),
               "eva_decode_microbench")
    assert out[3] == 0 and out[0] > 0


@pytest.mark.parametrize("M", [256, 128])
def test_pair_mma_tmem_layout(M):
    """tcgen05.mma.cta_group::2 (kind::f16, N = 256): with M = 256, CTA r's TMEM lane l, column c holds
    D[128 r + l][c]; with M = 128 each CTA's 64 rows x 256 columns are folded into 128 lanes x 128
    columns: lane l < 64 holds row 64 r + l, columns 0..127, lane l >= 64 row 64 r + l - 64, columns
    128..255 (the prefill kernels' half-height tiles read their accumulators this way)."""
    out = _selftest(3 if M == 256 else 4, shape=(2, 128, 256))
    want = np.full((2, 128, 256), 0xffffffff, np.uint32)
    for r in range(2):
        for lane in range(128):
            if M == 256:
                i, cols, n0 = 128 * r + lane, 256, 0
            else:
                i, cols, n0 = 64 * r + lane % 64, 128, 128 * (lane // 64)
            n = np.arange(cols) + n0
            want[r, lane, :cols] = np.float32((i + 1) + 256 * (n + 1)).view(np.uint32)
    assert np.array_equal(out, want)
