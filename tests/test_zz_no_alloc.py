"""The allocation-free combined pipeline (abra_q4k_mmvq_combined_static).

Its Q8_1 scratch is a static device array, so the results must equal those
of abra_q4k_mmvq_combined with a caller scratch buffer, bit for bit, on two
calls in a row (the second call reuses the scratch the first one left).
This file is named to be collected last: it must pass both alone and after
every other test has run in the same process.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import to_dev

MAX_VALUES = 131072  # K * ncols that the static scratch holds


def _lib():
    from abra_b200 import _lib

    return _lib


def test_static_scratch_rejects_oversize_without_launching():
    L = _lib()
    rc = L.lib.abra_q4k_mmvq_combined_static(0, 16, 16, 16, 8, 65536, 3, None)
    assert rc == L.ABRA_E_UNSUPPORTED
    assert "static" in L.last_error() and "131072" in L.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,ncols", [(9728, 2560, 1), (2560, 9728, 8), (1183, 4096, 3),
                                       (4096, 16384, 8)])
def test_static_scratch_matches_combined(dev, N, K, ncols):
    import torch

    L = _lib()
    assert K * ncols <= MAX_VALUES
    w = O.gen_q4k(N, K, 3, 17)
    dw = to_dev(w.reshape(-1), dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):  # two calls in a row, different inputs
        x = O.gen_normal_f32((ncols, K), 100 + call)
        dx = to_dev(x.reshape(-1), dev)
        scratch = torch.empty(ncols * K // 32 * 36, dtype=torch.uint8, device=dev)
        y_ref = torch.full((ncols * N,), float("nan"), dtype=torch.float32, device=dev)
        y = torch.full((ncols * N,), float("nan"), dtype=torch.float32, device=dev)
        assert L.lib.abra_q4k_mmvq_combined(0, dw.data_ptr(), dx.data_ptr(), scratch.data_ptr(),
                                            y_ref.data_ptr(), N, K, ncols, stream) == 0, L.last_error()
        assert L.lib.abra_q4k_mmvq_combined_static(0, dw.data_ptr(), dx.data_ptr(), y.data_ptr(),
                                                   N, K, ncols, stream) == 0, L.last_error()
        torch.cuda.synchronize()
        a, b = y.cpu().numpy(), y_ref.cpu().numpy()
        assert not np.isnan(a).any()
        assert np.array_equal(a, b), f"call {call}: static-scratch result differs"
