"""GPU parity tests of the Q6_K x Q8_1 MMVQ, through the C ABI.

Bar (as for Q4_K): the int32 16-weight sub-block dots bit-exact; fp32
outputs bit-identical to the canonical CPU oracle for every candidate, and
within 1e-5 of each row's |w|.|x| scale of the reference's f64 oracle.
Shapes: the reference test's grid (tests/runtime_kernel_test.cu:119-123:
N in {1, 33, 64}, K from 256 to 9728), ragged N, and the real Qwen3-4B
Q6_K tensors (attn_v 1024 x 2560, ffn_down 2560 x 9728, the tied
151936 x 2560 output).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import to_dev, tol_check

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _run(dev, w, xq, N, K, ncols, candidate=0, ldy=None, pdl=False):
    import torch
    import abra_b200 as A

    ldy = N if ldy is None else ldy
    dw, dx = to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev)
    dy = torch.full((ncols * ldy,), float("nan"), dtype=torch.float32, device=dev)
    A.mmvq_q6k(dw, dx, dy, N, K, ncols=ncols, ldy=ldy, candidate=candidate, pdl=pdl)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    y = dy.cpu().numpy().reshape(ncols, ldy)
    if ldy > N:
        assert np.isnan(y[:, N:]).all(), "wrote past N"
    return y[:, :N]


def _ids():
    import abra_b200 as A

    return sorted(A.q6k_candidates())


def test_generator_matches_oracle(dev):
    import torch
    import abra_b200 as A

    N, K = 300, 2560
    nb = N * K // 256
    d = torch.empty(nb * 210, dtype=torch.uint8, device=dev)
    A.gen_q6k(d, nb, seed=0, tensor_id=5)
    assert np.array_equal(d.cpu().numpy(), O.gen_q6k(N, K, 0, 5).reshape(-1))
    A.gen_q6k(d[: 11 * 210], 11, seed=0, tensor_id=5, block_offset=nb - 11)
    assert np.array_equal(d[: 11 * 210].cpu().numpy(), O.gen_q6k(N, K, 0, 5).reshape(-1)[-11 * 210:])


@pytest.mark.parametrize("N", [1, 33, 64])
@pytest.mark.parametrize("K", [256, 768, 2048, 2560, 4096, 4864, 9728])
def test_reference_grid_every_candidate(dev, N, K):
    w = O.gen_q6k(N, K, 1, 50)
    xq = O.quantize_q8_1(np.random.default_rng(K + N).uniform(-1, 1, (1, K)).astype(np.float32))
    ref = O.q6k_gemv(w, xq, K)
    for cid in _ids():
        y = _run(dev, w, xq, N, K, 1, candidate=cid)
        assert np.array_equal(y, ref), f"candidate {cid} differs from the canonical oracle"
    tol_check(y, O.q6k_gemv_f64(w, xq, K), O.q6k_absdot_f64(w, xq, K), TOL)


@pytest.mark.parametrize("ncols", [2, 3, 5, 8])
@pytest.mark.parametrize("N,K", [(77, 2560), (130, 4864), (9, 256)])
def test_batched_columns_every_candidate(dev, N, K, ncols):
    w = O.gen_q6k(N, K, 2, 51)
    xq = O.quantize_q8_1(O.gen_normal_f32((ncols, K), N + ncols))
    ref = O.q6k_gemv(w, xq, K)
    for cid in _ids():
        y = _run(dev, w, xq, N, K, ncols, candidate=cid, ldy=N + 3)
        assert np.array_equal(y, ref), f"candidate {cid} ncols {ncols}"


@pytest.mark.parametrize("ncols", [1, 2, 8])
@pytest.mark.parametrize("N,K", [(33, 768), (70, 2560)])
def test_partials_exact(dev, N, K, ncols):
    import torch
    import abra_b200 as A

    w = O.gen_q6k(N, K, 3, 52)
    xq = O.quantize_q8_1(O.gen_normal_f32((ncols, K), 3))
    dw, dx = to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev)
    dy = torch.empty(ncols * N, dtype=torch.float32, device=dev)
    dP = torch.full((ncols * N * (K // 256) * 16,), -7, dtype=torch.int32, device=dev)
    A.mmvq_q6k_partials(dw, dx, dy, dP, N, K, ncols=ncols)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert np.array_equal(dP.cpu().numpy().reshape(ncols, N, K // 256, 16), O.q6k_partials(w, xq, K))
    assert np.array_equal(dy.cpu().numpy().reshape(ncols, N), O.q6k_gemv(w, xq, K))


def test_zero_and_scaled_patterns(dev):
    N, K = 64, 4864
    w = np.zeros((N, K // 256 * 210), dtype=np.uint8)
    xq = O.quantize_q8_1(np.zeros((1, K), dtype=np.float32))
    y = _run(dev, w, xq, N, K, 1)
    assert not y.any() and not np.signbit(y).any()
    w = O.gen_q6k(N, K, 4, 53)
    b = w.reshape(-1, 210)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0] * 100
    b[:, 208:210] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    xq = O.quantize_q8_1(np.random.default_rng(5).uniform(-1, 1, (1, K)).astype(np.float32))
    y = _run(dev, w, xq, N, K, 1)
    assert np.array_equal(y, O.q6k_gemv(w, xq, K))


@pytest.mark.parametrize("N,K", [(1024, 2560), (2560, 9728), (151936, 2560)])
def test_qwen3_q6k_tensors(dev, N, K):
    """The real model's Q6_K shapes: tuned dispatch and two fixed feeds."""
    import torch
    import abra_b200 as A

    nb = N * K // 256
    dw = torch.empty(nb * 210, dtype=torch.uint8, device=dev)
    A.gen_q6k(dw, nb, seed=6, tensor_id=54)
    w = O.gen_q6k(N, K, 6, 54)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 6))
    dx = to_dev(xq.reshape(-1), dev)
    ref = O.q6k_gemv(w, xq, K, nthreads=O.max_threads())
    for cid in (0, 1022, 3042):
        dy = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
        A.mmvq_q6k(dw, dx, dy, N, K, candidate=cid)
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert np.array_equal(dy.cpu().numpy(), ref[0]), f"candidate {cid}"
    if N <= 4096:
        tol_check(ref, O.q6k_gemv_f64(w, xq, K), O.q6k_absdot_f64(w, xq, K), TOL)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kshard_recombines_bit_exact(dev, world):
    """Row-parallel Q6_K ffn_down: each rank's slice range of every row,
    recombined in the fixed tree, equals the unsharded output."""
    import torch
    import abra_b200 as A

    N, K = 2560, 9728
    nsb = K // 256
    w = O.gen_q6k(N, K, 7, 55)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 7))
    per = 8 // world
    parts = []
    for r in range(world):
        lo, hi = A.slice_start(nsb, r * per), A.slice_start(nsb, (r + 1) * per)
        ws = np.ascontiguousarray(w[:, lo * 210: hi * 210])
        xs = np.ascontiguousarray(xq[:, lo * 8 * 36: hi * 8 * 36])
        dy = torch.empty(N, dtype=torch.float32, device=dev)
        for cid in (0, 1042, 3082):
            A.mmvq_q6k_kshard(to_dev(ws.reshape(-1), dev), to_dev(xs.reshape(-1), dev), dy, N,
                              (hi - lo) * 256, K, r * per, per, candidate=cid)
            torch.cuda.synchronize()
            part = dy.cpu().numpy().reshape(1, N)
            if cid == 0:
                parts.append(part)
            else:
                assert np.array_equal(part, parts[-1]), f"candidate {cid} rank {r}"
    assert A.device_error() == 0
    assert np.array_equal(O.delta_tree(parts), O.q6k_gemv(w, xq, K, nthreads=O.max_threads()))


def test_pdl_launch_same_bits(dev):
    N, K = 2560, 9728
    w = O.gen_q6k(N, K, 8, 56)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 8))
    ref = O.q6k_gemv(w, xq, K, nthreads=O.max_threads())
    assert np.array_equal(_run(dev, w, xq, N, K, 1, pdl=True), ref)
