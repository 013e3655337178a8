"""GPU parity of the reference's 148-byte Q4_K prepack
(kernels/q4k/abra-packed-q4.cuh:3-31) and of the MMVQ over packed weights.

The pack must give the reference's bytes: fp16 d and dmin, then for each
pair j of sub-blocks the word [sc_2j, sc_2j+1, m_2j, m_2j+1] of the 6-bit
scales and mins (get_scale_min_k4's unpacking, restated below), then the 128
nibble bytes.  The packed MMVQ reads the same integers in the same order, so
y is bit-identical to the canonical oracle."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import to_dev, tol_check

pytestmark = pytest.mark.gpu


def _pack_reference(w: np.ndarray) -> np.ndarray:
    """The 148-byte form of Q4_K superblocks, restated from the struct and
    abra_pack_q4_one (kernels/q4k/abra-packed-q4.cuh:3-27)."""
    blk = w.reshape(-1, 144)
    out = np.zeros((blk.shape[0], 148), dtype=np.uint8)
    out[:, 0:4] = blk[:, 0:4]
    s = blk[:, 4:16].astype(np.uint32)
    sc = np.zeros((blk.shape[0], 8), dtype=np.uint32)
    mn = np.zeros((blk.shape[0], 8), dtype=np.uint32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63
            mn[:, j] = s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    for j in range(4):
        out[:, 4 + 4 * j + 0] = sc[:, 2 * j]
        out[:, 4 + 4 * j + 1] = sc[:, 2 * j + 1]
        out[:, 4 + 4 * j + 2] = mn[:, 2 * j]
        out[:, 4 + 4 * j + 3] = mn[:, 2 * j + 1]
    out[:, 20:148] = blk[:, 16:144]
    return out.reshape(-1)


@pytest.mark.parametrize("N,K", [(9728, 2560), (2560, 4096), (2560, 9728), (300, 2304), (64, 256)])
def test_pack_bytes_and_packed_mmvq_bit_exact(dev, N, K):
    import torch
    import abra_b200 as A

    w = O.gen_q4k(N, K, 0, 61)
    x = O.gen_normal_f32((1, K), 62)
    xq = O.quantize_q8_1(x)
    nb = N * K // 256
    dw = to_dev(w.reshape(-1), dev)
    dp = torch.zeros(nb * 148, dtype=torch.uint8, device=dev)
    A.pack_q4k(dw, dp, nb)
    torch.cuda.synchronize()
    assert np.array_equal(dp.cpu().numpy(), _pack_reference(w)), "packed bytes differ from the reference layout"
    dy = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
    A.mmvq_packed(dp, to_dev(xq.reshape(-1), dev), dy, N, K, pdl=True)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    y = dy.cpu().numpy().reshape(1, N)
    assert np.array_equal(y, O.gemv(w, xq, K, nthreads=8)), "not bit-exact to the canonical oracle"
    tol_check(y, O.gemv_f64(w, xq, K), O.absdot_f64(w, xq, K), 1e-5)


def test_packed_mmvq_rejects_bad_shapes(dev):
    import torch
    import abra_b200 as A

    dp = torch.zeros(148 * 8, dtype=torch.uint8, device=dev)
    dx = torch.zeros(36 * 8, dtype=torch.uint8, device=dev)
    dy = torch.zeros(8, dtype=torch.float32, device=dev)
    with pytest.raises(ValueError):
        A.mmvq_packed(dp, dx, dy, 8, 200)
