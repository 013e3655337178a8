"""Failure detection on the GPU without a fault: the bounded cross-rank wait
of the tensor-parallel kernels, on a flag that nothing sets, gives up after
its time limit with an error status the host reads, and the context stays
usable (the next kernel runs and is right)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O
from conftest import to_dev

pytestmark = pytest.mark.gpu


def test_bounded_flag_wait_reports_and_the_context_survives(dev):
    import torch
    import abra_b200 as A
    from abra_b200 import _lib

    bits, ns = C.c_uint32(), C.c_uint64()
    assert _lib.lib.abra_test_flag_timeout(C.byref(bits), C.byref(ns)) == _lib.ABRA_OK
    assert bits.value & 2, bits.value           # ERR_FLAG_TIMEOUT
    assert 0.9e9 <= ns.value <= 5e9, ns.value   # the one-second bound, not a hang
    assert A.device_error() == 0                # read and cleared
    N, K = 300, 2560
    w = O.gen_q4k(N, K, 1, 90)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 91))
    dy = torch.empty(N, dtype=torch.float32, device=dev)
    A.mmvq(to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev), dy, N, K)
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), O.gemv(w, xq, K)[0])
