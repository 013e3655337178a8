"""GPU parity tests of the Q4_K x Q8_1 path, through the C ABI.

Bar: per-sub-block int32 dot products bit-exact;
fp32 outputs within 1e-5 of each row's |w|.|x| scale against the f64 oracle.
The kernels follow the oracle's canonical fp32 order, so they are also
checked bit-for-bit against the canonical fp32 oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import to_dev, tol_check

pytestmark = pytest.mark.gpu

TOL = 1e-5  # of sum_k |w_k| |x_k|, per row (the path's stated tolerance)


def _case(N, K, ncols, seed=0, tid=0):
    w = O.gen_q4k(N, K, seed, tid)
    x = O.gen_normal_f32((ncols, K), seed + 1000)
    return w, x, O.quantize_q8_1(x)


def _run(dev, w, xq, N, K, ncols, candidate=0, pdl=False):
    import torch
    import abra_b200 as A

    dw, dx = to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev)
    dy = torch.full((ncols * N,), float("nan"), dtype=torch.float32, device=dev)
    A.mmvq(dw, dx, dy, N, K, ncols=ncols, candidate=candidate, pdl=pdl)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return dy.cpu().numpy().reshape(ncols, N)


def test_generator_matches_oracle(dev):
    import torch
    import abra_b200 as A

    N, K = 300, 2560
    nb = N * K // 256
    d = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
    A.gen_q4k(d, nb, seed=0, tensor_id=5)
    assert np.array_equal(d.cpu().numpy(), O.gen_q4k(N, K, 0, 5).reshape(-1))
    A.gen_q4k(d[: 10 * 144], 10, seed=0, tensor_id=5, block_offset=nb - 10)
    assert np.array_equal(d[: 10 * 144].cpu().numpy(), O.gen_q4k(N, K, 0, 5).reshape(-1)[-10 * 144:])
    u = torch.empty(4099, dtype=torch.float32, device=dev)
    A.gen_uniform_f32(u, 4099, 0, 77, 0.4, 0.8)
    assert np.array_equal(u.cpu().numpy(), O.gen_uniform_f32(4099, 0, 77, 0.4, 0.8))


@pytest.mark.parametrize("fam", ["normal", "zero", "wide", "tiny", "outliers"])
@pytest.mark.parametrize("ncols", [1, 3])
def test_quantizer_bytes_bit_exact(dev, fam, ncols):
    import torch
    import abra_b200 as A

    K = 9728
    rng = np.random.default_rng(5)
    x = {"normal": rng.standard_normal((ncols, K)), "zero": np.zeros((ncols, K)),
         "wide": rng.uniform(-100, 100, (ncols, K)), "tiny": rng.standard_normal((ncols, K)) * 1e-7,
         "outliers": np.where(np.arange(K) % 64 == 0, 10.0, rng.uniform(-0.1, 0.1, (ncols, K)))}[fam]
    x = x.astype(np.float32)
    dq = torch.zeros(ncols * K // 32 * 36, dtype=torch.uint8, device=dev)
    A.launch_quantize_f32_to_q8_1(to_dev(x.reshape(-1), dev), dq, K, ncols=ncols)
    torch.cuda.synchronize()
    assert np.array_equal(dq.cpu().numpy(), O.quantize_q8_1(x).reshape(-1))


@pytest.mark.parametrize("K", [128, 2560, 4096, 9728])
def test_rmsnorm_quantize_bit_exact(dev, K):
    import torch
    import abra_b200 as A

    ncols = 2
    x = O.gen_normal_f32((ncols, K), 3) * 7.0
    g = O.gen_uniform_f32(K, 0, 91, 0.4, 0.8)
    dq = torch.zeros(ncols * K // 32 * 36, dtype=torch.uint8, device=dev)
    dxn = torch.zeros(ncols * K, dtype=torch.float32, device=dev)
    A.rmsnorm_quantize_q8_1(to_dev(x.reshape(-1), dev), to_dev(g, dev), 1e-6, dq, K, ncols=ncols,
                            d_xn_out=dxn)
    torch.cuda.synchronize()
    q_ref, xn_ref = O.rmsnorm_quantize_q8_1(x, g, 1e-6)
    assert np.array_equal(dxn.cpu().numpy().view(np.uint32), xn_ref.reshape(-1).view(np.uint32))
    assert np.array_equal(dq.cpu().numpy(), q_ref.reshape(-1))


@pytest.mark.parametrize("N,K,ncols,ks", [
    (64, 256, 1, 1), (33, 2560, 1, 2), (129, 2048, 2, 4), (64, 9728, 4, 1),
    (17, 4096, 8, 2), (300, 2560, 1, 4)])
def test_partials_bit_exact(dev, N, K, ncols, ks):
    import torch
    import abra_b200 as A

    w, _, xq = _case(N, K, ncols, seed=N + K)
    nsb = K // 256
    dP = torch.zeros(ncols * N * nsb * 8, dtype=torch.int32, device=dev)
    dM = torch.zeros(ncols * nsb * 8, dtype=torch.int32, device=dev)
    dy = torch.zeros(ncols * N, dtype=torch.float32, device=dev)
    A.mmvq_partials(to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev), dy, dP, dM, N, K,
                    ncols=ncols, ks=ks)
    torch.cuda.synchronize()
    P, M = O.partials(w, xq, K)
    assert np.array_equal(dP.cpu().numpy().reshape(P.shape), P)
    assert np.array_equal(dM.cpu().numpy().reshape(M.shape), M)
    assert np.array_equal(dy.cpu().numpy().reshape(ncols, N), O.gemv(w, xq, K))


QWEN = [(4096, 2560), (1024, 2560), (2560, 4096), (9728, 2560), (2560, 9728), (6144, 2560)]


@pytest.mark.parametrize("N,K", QWEN)
@pytest.mark.parametrize("ncols", [1, 8])
def test_qwen_shapes_tuned(dev, N, K, ncols):
    w, _, xq = _case(N, K, ncols, seed=N ^ K)
    y = _run(dev, w, xq, N, K, ncols)
    assert np.array_equal(y, O.gemv(w, xq, K, nthreads=8)), "not bit-exact to the canonical oracle"
    tol_check(y, O.gemv_f64(w, xq, K), O.absdot_f64(w, xq, K), TOL)


@pytest.mark.parametrize("N,K,ncols", [(9728, 2560, 1), (2560, 9728, 8), (1183, 4096, 3)])
def test_combined_pipeline(dev, N, K, ncols):
    """fp32 input -> Q8_1 scratch -> MMVQ in one call (tuned and named
    candidates): the scratch holds the oracle's Q8_1 bytes and y is
    bit-exact to the canonical oracle."""
    import torch
    import abra_b200 as A

    w, x, xq = _case(N, K, ncols, seed=11)
    ref = O.gemv(w, xq, K, nthreads=8)
    dw, dx = to_dev(w.reshape(-1), dev), to_dev(x.reshape(-1), dev)
    for cid in (0, 3022, 1041):
        scratch = torch.zeros(ncols * K // 32 * 36, dtype=torch.uint8, device=dev)
        dy = torch.full((ncols * N,), float("nan"), dtype=torch.float32, device=dev)
        if cid == 0:
            A.launch_q4k_autotuned_combined_pipeline(dw, dx, scratch, dy, N, K, ncols=ncols)
        else:
            A.launch_q4k_candidate_combined_pipeline(cid, dw, dx, scratch, dy, N, K, ncols=ncols)
        torch.cuda.synchronize()
        assert np.array_equal(scratch.cpu().numpy(), xq.reshape(-1))
        assert np.array_equal(dy.cpu().numpy().reshape(ncols, N), ref), f"candidate {cid}"


@pytest.mark.parametrize("N,K", [(1000, 4096), (77, 9728), (2049, 2560)])
def test_every_candidate_bit_identical(dev, N, K):
    import abra_b200 as A

    for ncols in (1, 2):
        w, _, xq = _case(N, K, ncols, seed=7)
        ref = O.gemv(w, xq, K, nthreads=8)
        for cid in A.get_all_candidate_ids():
            y = _run(dev, w, xq, N, K, ncols, candidate=cid, pdl=bool(cid % 2))
            assert np.array_equal(y, ref), f"candidate {cid} ncols={ncols} differs"


@pytest.mark.parametrize("nmat", [1, 2])
def test_ring_reuse_every_candidate_pdl_chain(dev, nmat):
    """N large enough that every CTA cycles its shared-memory ring several
    times; three back-to-back launches with programmatic dependent launch into
    three outputs; every candidate bit-exact and no bounded wait gives up."""
    import torch
    import abra_b200 as A

    N, K, ncols = 148 * 8 * 40, 2560, 1
    ws = [O.gen_q4k(N, K, 2, 51 + m) for m in range(nmat)]
    xq = O.quantize_q8_1(O.gen_normal_f32((ncols, K), 9) * (0.05 if nmat == 2 else 1.0))
    ref = O.gemv(ws[0], xq, K, 8) if nmat == 1 else O.gemv_swiglu(ws[0], ws[1], xq, K, 8)
    dws = [to_dev(w.reshape(-1), dev) for w in ws]
    dx = to_dev(xq.reshape(-1), dev)
    for cid in A.get_all_candidate_ids():
        ys = [torch.full((N,), float("nan"), dtype=torch.float32, device=dev) for _ in range(3)]
        for y in ys:
            if nmat == 1:
                A.mmvq(dws[0], dx, y, N, K, candidate=cid, pdl=True)
            else:
                A.mmvq_swiglu(dws[0], dws[1], dx, y, N, K, candidate=cid, pdl=True)
        torch.cuda.synchronize()
        assert A.device_error() == 0, f"candidate {cid}: a bounded wait gave up"
        for y in ys:
            assert np.array_equal(y.cpu().numpy(), ref[0]), f"candidate {cid} nmat={nmat}"


def _run_swiglu(dev, wg, wu, xq, N, K, ncols, candidate=0):
    import torch
    import abra_b200 as A

    dy = torch.full((ncols * N,), float("nan"), dtype=torch.float32, device=dev)
    A.mmvq_swiglu(to_dev(wg.reshape(-1), dev), to_dev(wu.reshape(-1), dev),
                  to_dev(xq.reshape(-1), dev), dy, N, K, ncols=ncols, candidate=candidate)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    return dy.cpu().numpy().reshape(ncols, N)


@pytest.mark.parametrize("N,K,ncols", [(9728, 2560, 1), (9728, 2560, 8), (333, 4096, 3), (8, 256, 1)])
def test_swiglu_fused_bit_exact(dev, N, K, ncols):
    wg = O.gen_q4k(N, K, 0, 21)
    wu = O.gen_q4k(N, K, 0, 22)
    x = O.gen_normal_f32((ncols, K), 5) * 0.05  # keep silu away from saturation
    xq = O.quantize_q8_1(x)
    y = _run_swiglu(dev, wg, wu, xq, N, K, ncols)
    ref = O.gemv_swiglu(wg, wu, xq, K, nthreads=8)
    assert np.array_equal(y, ref)


def test_swiglu_every_candidate(dev):
    import abra_b200 as A

    N, K, ncols = 700, 2560, 2
    wg, wu = O.gen_q4k(N, K, 1, 31), O.gen_q4k(N, K, 1, 32)
    xq = O.quantize_q8_1(O.gen_normal_f32((ncols, K), 6) * 0.05)
    ref = O.gemv_swiglu(wg, wu, xq, K, nthreads=8)
    for cid in A.get_all_candidate_ids():
        assert np.array_equal(_run_swiglu(dev, wg, wu, xq, N, K, ncols, cid), ref), cid


@pytest.mark.parametrize("N,K,nmat", [(6144, 2560, 1), (9728, 2560, 2), (300, 4096, 1),
                                      (77, 256, 2)])
def test_fused_rmsnorm_mmvq_bit_exact(dev, N, K, nmat):
    """abra_q4k_mmvq_rmsnorm (RMSNorm and Q8_1 in every CTA's prologue, then
    the MMVQ; nmat 2: the gate/up SwiGLU) equals the oracle's
    rmsnorm_quantize_q8_1 followed by its GEMV, and the exported Q8_1 copy
    equals the oracle's bytes."""
    import torch
    import abra_b200 as A
    from abra_b200 import AbraError, _lib

    x = O.gen_normal_f32((1, K), 17) * 3.0
    g = O.gen_uniform_f32(K, 0, 93, 0.4, 0.8)
    q_ref, _ = O.rmsnorm_quantize_q8_1(x, g, 1e-6)
    w = O.gen_q4k(N, K, 2, 61)
    wu = O.gen_q4k(N, K, 2, 62) if nmat == 2 else None
    if nmat == 2:
        ref = O.gemv_swiglu(w, wu, q_ref, K, nthreads=8)
    else:
        ref = O.gemv(w, q_ref, K, nthreads=8)
    dx, dg = to_dev(x.reshape(-1), dev), to_dev(g, dev)
    dw = to_dev(w.reshape(-1), dev)
    dwu = to_dev(wu.reshape(-1), dev) if nmat == 2 else None
    dq = torch.zeros(K // 32 * 36, dtype=torch.uint8, device=dev)
    cands = [0] + A.get_all_candidate_ids() if N < 1000 else [0, 1011, 1021, 2011, 3012, 3082]
    ran = 0
    for cid in cands:
        dy = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
        dq.zero_()
        try:
            A.mmvq_rmsnorm(dw, dx, dg, 1e-6, dy, N, K, d_w_up=dwu, d_x_q8_out=dq, candidate=cid)
        except AbraError as e:  # no fused plan for this candidate and shape
            assert e.code == _lib.ABRA_E_UNSUPPORTED, str(e)
            continue
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert np.array_equal(dy.cpu().numpy(), ref[0]), f"candidate {cid}"
        assert np.array_equal(dq.cpu().numpy(), q_ref.reshape(-1)), f"candidate {cid}: Q8_1 copy"
        ran += 1
    assert ran >= 2


def test_expf_matches_oracle(dev):
    """silu's exp: the device copy returns the oracle's bits on a dense sweep."""
    import torch
    import abra_b200 as A

    N, K = 4096, 256
    wg = O.gen_q4k(N, K, 3, 41)
    wu = O.gen_q4k(N, K, 3, 42)
    rng = np.random.default_rng(8)
    for scale in (1e-3, 0.02, 0.2):
        xq = O.quantize_q8_1(rng.standard_normal((1, K)).astype(np.float32) * scale)
        assert np.array_equal(_run_swiglu(dev, wg, wu, xq, N, K, 1),
                              O.gemv_swiglu(wg, wu, xq, K))


@pytest.mark.parametrize("ncols", [1, 2, 3, 4, 5, 6, 7, 8])
def test_all_batch_widths(dev, ncols):
    N, K = 257, 2560
    w, _, xq = _case(N, K, ncols, seed=ncols)
    assert np.array_equal(_run(dev, w, xq, N, K, ncols), O.gemv(w, xq, K))


@pytest.mark.parametrize("N", [1, 2, 3, 7, 8, 9, 31, 33, 127, 129, 1183])
@pytest.mark.parametrize("K", [256, 512, 2304, 8192])
def test_n_k_edges(dev, N, K):
    w, _, xq = _case(N, K, 1, seed=N * 7 + K)
    y = _run(dev, w, xq, N, K, 1)
    assert np.array_equal(y, O.gemv(w, xq, K))


def test_pdl_launch_and_ldy(dev):
    import torch
    import abra_b200 as A

    N, K, ncols, ldy = 500, 2560, 2, 640
    w, _, xq = _case(N, K, ncols, seed=3)
    dw, dx = to_dev(w.reshape(-1), dev), to_dev(xq.reshape(-1), dev)
    dy = torch.full((ncols * ldy,), -7.0, dtype=torch.float32, device=dev)
    for _ in range(3):
        A.mmvq(dw, dx, dy, N, K, ncols=ncols, ldy=ldy, pdl=True)
    torch.cuda.synchronize()
    y = dy.cpu().numpy().reshape(ncols, ldy)
    assert np.array_equal(y[:, :N], O.gemv(w, xq, K))
    assert (y[:, N:] == -7.0).all(), "wrote outside the rows"


def test_output_projection_full_size(dev):
    """Tied 151936 x 2560 output at full size: size-independent properties
    (bit-exact on a row sample, finite everywhere, linearity in x)."""
    import torch
    import abra_b200 as A

    N, K = 151936, 2560
    nb = N * K // 256
    dw = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
    A.gen_q4k(dw, nb, seed=0, tensor_id=1)
    x = O.gen_normal_f32((1, K), 9)
    xq = O.quantize_q8_1(x)
    dy = torch.empty(N, dtype=torch.float32, device=dev)
    A.mmvq(dw, to_dev(xq.reshape(-1), dev), dy, N, K)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    assert np.isfinite(y).all()
    rows = np.r_[0:64, N // 2: N // 2 + 64, N - 64: N]
    wr = np.concatenate([O.gen_q4k(64, K, 0, 1, r0) for r0 in (0, N // 2, N - 64)])
    assert np.array_equal(y[rows], O.gemv(wr, xq, K)[0])
    # x and 2x (exact doubling of d8 in fp16) -> y doubles exactly
    xq2 = xq.copy().reshape(-1, 36)
    d = xq2[:, 0:2].copy().view(np.float16) * np.float16(2)
    xq2[:, 0:2] = d.view(np.uint8)
    dy2 = torch.empty(N, dtype=torch.float32, device=dev)
    A.mmvq(dw, to_dev(xq2.reshape(-1), dev), dy2, N, K)
    torch.cuda.synchronize()
    assert np.array_equal(dy2.cpu().numpy(), 2 * y)


# --------------------------------------------- reference kernels on B200 ---
def test_reference_family_agrees(dev):
    """The reference's own 16 candidates (oracle/_ref) on the same inputs: its
    quantizer's bytes equal ours and its outputs are within tolerance of ours."""
    import torch
    import abra_b200 as A

    ref = O.RefFamily()
    N, K = 1024, 2560
    w, x, xq = _case(N, K, 1, seed=42)
    dw = to_dev(w.reshape(-1), dev)
    dxf = to_dev(x.reshape(-1), dev)
    dq_ref = torch.zeros(K // 32 * 36, dtype=torch.uint8, device=dev)
    ref.quantize(dxf.data_ptr(), dq_ref.data_ptr(), K)
    dq = torch.zeros_like(dq_ref)
    A.launch_quantize_f32_to_q8_1(dxf, dq, K)
    torch.cuda.synchronize()
    assert torch.equal(dq, dq_ref)
    y_ours = _run(dev, w, xq, N, K, 1)[0]
    y64 = O.gemv_f64(w, xq, K)[0]
    scale = O.absdot_f64(w, xq, K)[0]
    for cid in ref.candidate_ids():
        dy = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
        ref.launch_candidate(cid, dw.data_ptr(), dq_ref.data_ptr(), dy.data_ptr(), N, K)
        torch.cuda.synchronize()
        yr = dy.cpu().numpy()
        tol_check(yr[None], y64[None], scale[None], TOL)
        assert (np.abs(yr - y_ours) / scale).max() <= 2 * TOL
