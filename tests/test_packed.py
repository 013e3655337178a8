"""CPU check of the 148-byte prepack layout restated in test_packed_gpu.py
(kernels/q4k/abra-packed-q4.cuh:3-27): weights rebuilt from the packed
bytes equal the oracle's dequantization of the original Q4_K superblocks."""
from __future__ import annotations

import numpy as np

import oracle as O
from test_packed_gpu import _pack_reference


def test_packed_layout_dequantizes_like_q4k():
    w = O.gen_q4k(24, 1024, 0, 71)
    p = _pack_reference(w).reshape(-1, 148)
    d = p[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    dmin = p[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(-1)
    y = np.zeros((p.shape[0], 256), dtype=np.float32)
    for j in range(8):
        sc = p[:, 4 + 4 * (j // 2) + (j % 2)].astype(np.float32)
        mn = p[:, 4 + 4 * (j // 2) + 2 + (j % 2)].astype(np.float32)
        qs = p[:, 20 + 32 * (j // 2): 20 + 32 * (j // 2) + 32]
        q = (qs >> 4) if j % 2 else (qs & 0xF)
        y[:, 32 * j: 32 * j + 32] = (d * sc)[:, None] * q.astype(np.float32) - (dmin * mn)[:, None]
    ref = O.dequant_q4k(w).reshape(-1, 256)
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)
