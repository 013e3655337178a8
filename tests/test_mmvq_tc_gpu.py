"""Batch-32 MMVQ on the tcgen05 tensor cores, through the C ABI.

The tensor core produces the exact int32 sub-block dot products; the fp32
scaling follows the canonical order, so the outputs must equal the CPU
oracle (and therefore the dp4a kernels) bit for bit, for every k-split.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import to_dev, tol_check

pytestmark = pytest.mark.gpu

NC = 32


def _run_tc(dev, w, xq, N, K, ks):
    import torch
    import abra_b200 as A

    dw, dx = to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev)
    dy = torch.full((NC * N,), float("nan"), dtype=torch.float32, device=dev)
    ws = torch.empty(ks * NC * N, dtype=torch.float32, device=dev) if ks > 1 else None
    A.mmvq_tc(dw, dx, dy, N, K, ks=ks, d_workspace=ws)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return dy.cpu().numpy().reshape(NC, N)


@pytest.mark.parametrize("N,K", [(128, 256), (77, 2560), (300, 2304), (1000, 4096)])
@pytest.mark.parametrize("ks", [1, 2, 4, 8])
def test_tc_bit_exact_small(dev, N, K, ks):
    w = O.gen_q4k(N, K, 3, 61)
    xq = O.quantize_q8_1(O.gen_normal_f32((NC, K), 17))
    y = _run_tc(dev, w, xq, N, K, ks)
    assert np.array_equal(y, O.gemv(w, xq, K, nthreads=8)), "not bit-exact to the canonical oracle"


@pytest.mark.parametrize("N,K,ks", [(4096, 2560, 1), (2560, 4096, 4), (9728, 2560, 1),
                                    (2560, 9728, 8), (6144, 2560, 2)])
def test_tc_qwen_shapes(dev, N, K, ks):
    w = O.gen_q4k(N, K, 5, 62)
    xq = O.quantize_q8_1(O.gen_normal_f32((NC, K), 18))
    y = _run_tc(dev, w, xq, N, K, ks)
    assert np.array_equal(y, O.gemv(w, xq, K, nthreads=8))
    tol_check(y, O.gemv_f64(w, xq, K), O.absdot_f64(w, xq, K), 1e-5)
