"""GPU parity of the reference-named C shim (kernels/q4k/upstream_adapter.cuh:
12-26) on the single-GEMV workload: launch_pinned_upstream_q8_1_quantize and
launch_pinned_upstream_mmvq, called through ctypes exactly as a binding of the
reference's adapter would, against the CPU oracle.

The workload is the reference's config-0 GEMV: 9728 x 2560 Q4_K weights
(seed 0), one N(0,1) activation column quantized to Q8_1.  Bar: Q8_1 bytes
identical; y bit-identical to the canonical-order oracle and within 1e-5 of
each row's |w|.|x| scale against the f64 oracle."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O
from conftest import to_dev, tol_check

pytestmark = pytest.mark.gpu


def test_shim_quantize_and_mmvq_match_the_oracle(dev):
    import torch
    import abra_b200 as A

    lib = C.CDLL(str(A.LIB_PATH))
    lib.launch_pinned_upstream_q8_1_quantize.restype = None
    lib.launch_pinned_upstream_q8_1_quantize.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
    lib.launch_pinned_upstream_mmvq.restype = None
    lib.launch_pinned_upstream_mmvq.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                                C.c_void_p]
    N, K = 9728, 2560
    w = O.gen_q4k(N, K, 0, 0)
    x = O.gen_normal_f32((1, K), 1000)
    xq_ref = O.quantize_q8_1(x)

    dx = to_dev(x.reshape(-1), dev)
    dxq = torch.zeros(xq_ref.size, dtype=torch.uint8, device=dev)
    dw = to_dev(w.reshape(-1), dev)
    dy = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    lib.launch_pinned_upstream_q8_1_quantize(dx.data_ptr(), dxq.data_ptr(), K, stream)
    lib.launch_pinned_upstream_mmvq(dw.data_ptr(), dxq.data_ptr(), dy.data_ptr(), N, K, stream)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert np.array_equal(dxq.cpu().numpy(), xq_ref.reshape(-1)), "Q8_1 bytes differ from the oracle"
    y = dy.cpu().numpy().reshape(1, N)
    assert np.array_equal(y, O.gemv(w, xq_ref, K, nthreads=8)), "not bit-exact to the canonical oracle"
    tol_check(y, O.gemv_f64(w, xq_ref, K), O.absdot_f64(w, xq_ref, K), 1e-5)


def test_shim_rejects_a_bad_shape_without_launching(dev):
    """K not a multiple of 256: the shim records the error (as the reference
    throws std::invalid_argument, kernels/q4k/q4k_q8_mmvq.cu:266-268) and
    leaves y untouched."""
    import torch
    import abra_b200 as A

    lib = C.CDLL(str(A.LIB_PATH))
    lib.launch_pinned_upstream_mmvq.restype = None
    lib.launch_pinned_upstream_mmvq.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                                C.c_void_p]
    dw = torch.zeros(4 * 144, dtype=torch.uint8, device=dev)
    dxq = torch.zeros(36 * 8, dtype=torch.uint8, device=dev)
    dy = torch.full((4,), 7.0, dtype=torch.float32, device=dev)
    lib.launch_pinned_upstream_mmvq(dw.data_ptr(), dxq.data_ptr(), dy.data_ptr(), 4, 200, None)
    torch.cuda.synchronize()
    from abra_b200 import _lib

    assert _lib.last_error() != ""
    assert np.all(dy.cpu().numpy() == 7.0)
