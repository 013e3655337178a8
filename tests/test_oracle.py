"""CPU tests of the oracle: formats, generator, quantizer, exact partials,
canonical fp32 order, and the golden vectors recorded from the reference's own
kernels (tests/golden/, made by tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN, tol_check

SHAPES_QWEN = [(4096, 2560), (1024, 2560), (2560, 4096), (9728, 2560), (2560, 9728)]


def np_scale_min(sc12: np.ndarray):
    """Independent numpy restatement of get_scale_min_k4 (tests/q4k_q8_test.cu:44-52)."""
    q = sc12.astype(np.int32)
    sc = np.zeros(q.shape[:-1] + (8,), np.int32)
    m = np.zeros_like(sc)
    for j in range(8):
        if j < 4:
            sc[..., j] = q[..., j] & 63
            m[..., j] = q[..., j + 4] & 63
        else:
            sc[..., j] = (q[..., j + 4] & 0xF) | ((q[..., j - 4] >> 6) << 4)
            m[..., j] = (q[..., j + 4] >> 4) | ((q[..., j] >> 6) << 4)
    return sc, m


def np_quantize_q8_1(x: np.ndarray) -> np.ndarray:
    """numpy restatement of the reference quantizer (kernels/q4k/q4k_q8_mmvq.cu:223-255)."""
    xb = x.reshape(-1, 32).astype(np.float32)
    amax = np.max(np.abs(xb), axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d > 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = (xb * idv[:, None]).astype(np.float32)
    q = np.where(v >= 0, np.floor(v + np.float32(0.5)), -np.floor(-v + np.float32(0.5))).astype(np.int8)
    s = (d * q.astype(np.int32).sum(1).astype(np.float32)).astype(np.float32)
    out = np.zeros((xb.shape[0], 36), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = s.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 4:] = q.view(np.uint8)
    return out.reshape(-1)


def test_fp16_conversion_matches_numpy():
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                           for s in (1e-8, 3e-6, 1e-4, 1.0, 3e4, 7e4)])
    vals = np.concatenate([vals, np.float32([0, -0.0, 65504, 65520, 2.9802322e-08, 5.9604645e-08])])
    mine = np.array([O.f32_to_f16_bits(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)


def test_generator_layout_and_distributions():
    w = O.gen_q4k(512, 2560, seed=0, tensor_id=0)
    assert w.shape == (512, 10 * 144)
    blk = w.reshape(-1, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    dm = blk[:, 2:4].copy().view(np.float16).astype(np.float32).ravel()
    for a in (d, dm):
        assert a.min() >= 0.001 - 1e-6 and a.max() <= 0.02 + 1e-5
        assert abs(a.mean() - 0.0105) < 0.0005
    sc, m = np_scale_min(blk[:, 4:16])
    for a in (sc, m):
        assert a.min() == 0 and a.max() == 63 and abs(a.mean() - 31.5) < 0.5
    nib = np.concatenate([blk[:, 16:] & 15, blk[:, 16:] >> 4])
    assert nib.min() == 0 and nib.max() == 15 and abs(nib.mean() - 7.5) < 0.05
    # counter-based: any row range regenerates identical bytes
    part = O.gen_q4k(7, 2560, seed=0, tensor_id=0, row_offset=100)
    assert np.array_equal(part, w[100:107])
    assert not np.array_equal(O.gen_q4k(4, 2560, 0, 1), w[:4])


def test_dequant_matches_gguf_decoder():
    gq = pytest.importorskip("gguf.quants")
    w = O.gen_q4k(64, 2560, seed=5, tensor_id=3)
    mine = O.dequant_q4k(w)
    theirs = gq.Q4_K.dequantize_blocks(w.reshape(-1, 144)).reshape(-1).astype(np.float32)
    assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))


@pytest.mark.parametrize("dist", ["normal", "zero", "const", "alt", "wide", "outliers", "tiny"])
def test_quantizer_matches_numpy_restatement(dist):
    rng = np.random.default_rng(11)
    K = 2560
    x = {
        "normal": rng.standard_normal(K),
        "zero": np.zeros(K),
        "const": np.full(K, 0.125),
        "alt": np.where(np.arange(K) % 2 == 0, 0.5, -0.5),
        "wide": rng.uniform(-100, 100, K),
        "outliers": np.where(np.arange(K) % 64 == 0, 10.0, rng.uniform(-0.1, 0.1, K)),
        "tiny": rng.standard_normal(K) * 1e-6,
    }[dist].astype(np.float32)
    assert np.array_equal(O.quantize_q8_1(x).reshape(-1), np_quantize_q8_1(x))


def test_partials_exact_against_numpy():
    K, N = 2048, 33
    w = O.gen_q4k(N, K, seed=2, tensor_id=9)
    xq = O.quantize_q8_1(O.gen_normal_f32((3, K), 2))
    P, M = O.partials(w, xq, K)
    blk = w.reshape(N, K // 256, 144)
    qs = blk[:, :, 16:].reshape(N, K // 256, 4, 32).astype(np.int64)
    q4 = np.stack([qs & 15, qs >> 4], axis=3).reshape(N, K // 256, 8, 32)
    q8 = xq.reshape(3, K // 256, 8, 36)[..., 4:].view(np.int8).astype(np.int64)
    Pn = np.einsum("rbsl,cbsl->crbs", q4, q8)
    assert np.array_equal(P, Pn)
    assert np.array_equal(M, q8.sum(-1))


@pytest.mark.parametrize("N,K", SHAPES_QWEN[:2] + [(33, 256), (5, 9728)])
def test_canonical_fp32_within_tolerance(N, K):
    w = O.gen_q4k(N, K, seed=0, tensor_id=1)
    xq = O.quantize_q8_1(O.gen_normal_f32((2, K), 0))
    y = O.gemv(w, xq, K)
    tol_check(y, O.gemv_f64(w, xq, K), O.absdot_f64(w, xq, K), rel=1e-6)


def test_canonical_threads_do_not_change_bits():
    w = O.gen_q4k(300, 2560, seed=0, tensor_id=4)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, 2560), 4))
    assert np.array_equal(O.gemv(w, xq, 2560, 1), O.gemv(w, xq, 2560, 4))


@pytest.mark.parametrize("nsb", [1, 2, 7, 8, 10, 16, 38, 39])
def test_slices_and_tree(nsb):
    s = O.slice_starts(nsb)
    sizes = np.diff(s)
    assert s[0] == 0 and s[-1] == nsb and sizes.max() - sizes.min() <= 1
    assert list(sizes) == sorted(sizes, reverse=True)
    K = nsb * 256
    w = O.gen_q4k(9, K, seed=1, tensor_id=2)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 1))
    v = O.gemv_slices(w, xq, K)[0]
    f = np.float32
    tree = ((f(v[:, 0] + v[:, 1]) + f(v[:, 2] + v[:, 3])) + (f(v[:, 4] + v[:, 5]) + f(v[:, 6] + v[:, 7])))
    assert np.array_equal(tree.astype(np.float32), O.gemv(w, xq, K)[0])


def test_rmsnorm_quantize_reference_formula():
    K = 2560
    x = O.gen_normal_f32((2, K), 7)
    g = O.gen_uniform_f32(K, 0, 77, 0.4, 0.8)
    q, xn = O.rmsnorm_quantize_q8_1(x, g, 1e-6)
    r = 1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1) + 1e-6)
    np.testing.assert_allclose(xn, x * r[:, None] * g, rtol=2e-6, atol=1e-7)
    assert np.array_equal(q, O.quantize_q8_1(xn))


# ----------------------------------------------- golden (reference kernels) ---
def _golden_files():
    return sorted(GOLDEN.glob("ref_*.npz"))


def test_golden_fixtures_present():
    files = _golden_files()
    assert files, "tests/golden/ref_*.npz missing: run tests/golden/make_golden.py on a GPU"


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_matches_reference_kernels(path):
    """Pins the oracle against outputs of the reference's own CUDA kernels.

    Q8_1 bytes from the reference quantizer must equal the oracle's bit for
    bit; every reference MMVQ candidate's fp32 output must agree with the
    oracle's f64 value within 1e-5 of the row's |w|.|x| scale (the reference
    accumulates in fp32 in its own order)."""
    g = np.load(path)
    N, K, seed, tid = (int(g[k]) for k in ("N", "K", "seed", "tensor_id"))
    w = O.gen_q4k(N, K, seed, tid)
    assert np.array_equal(w.reshape(-1)[: g["w_head"].size], g["w_head"])
    x = g["x"]
    xq = O.quantize_q8_1(x)
    assert np.array_equal(xq.reshape(-1), g["xq_ref"].reshape(-1)), "Q8_1 bytes differ from the reference quantizer"
    y64 = O.gemv_f64(w, xq, K)
    scale = O.absdot_f64(w, xq, K)
    for key in g.files:
        if key.startswith("y_ref_"):
            tol_check(g[key].reshape(1, -1), y64, scale, rel=1e-5)
    # and the canonical fp32 oracle sits at least as close to f64
    tol_check(O.gemv(w, xq, K), y64, scale, rel=1e-6)


def test_vectorised_integer_dots_give_the_same_bits():
    """The oracle GEMV's integer sub-block dots run on the host's widest
    integer dot (AVX-512 VNNI / AVX2) or the scalar loop: identical outputs."""
    K = 2560
    w = O.gen_q4k(200, K, 2, 71)
    xq = O.quantize_q8_1(O.gen_normal_f32((3, K), 72))
    best = O.lib.orc_simd_level()
    try:
        outs = []
        for lvl in range(best + 1):
            O.lib.orc_set_simd_level(lvl)
            outs.append((O.gemv(w, xq, K, nthreads=4), O.gemv_slices(w, xq, K)))
    finally:
        O.lib.orc_set_simd_level(-1)
    for y, v in outs[1:]:
        assert np.array_equal(y, outs[0][0]) and np.array_equal(v, outs[0][1])
    assert np.array_equal(O.tree8(outs[-1][1]), outs[-1][0])


def test_cpu_baseline_q8k_path():
    """The restated llama.cpp CPU path that bench.py times (not a parity
    target): Q8_K blocks hold the block sums of 16 and map each block's
    largest-magnitude value to -127; the Q4_K x Q8_K dot equals the f64 dot
    of the dequantized operands to fp32 accuracy and stays within the
    activation quantization of the fp32 product."""
    N, K, ncols = 300, 2560, 3
    w = O.gen_q4k(N, K, 4, 9)
    x = O.gen_normal_f32((ncols, K), 12)
    x[1, :256] = 0.0  # an all-zero block
    yk = O.quantize_q8_K(x)
    b = yk.reshape(ncols, K // 256, O.Q8K_BYTES)
    d = b[:, :, :4].copy().view(np.float32)[:, :, 0]
    q = b[:, :, 4:260].view(np.int8).astype(np.int64)
    bs = b[:, :, 260:].copy().view(np.int16)
    assert np.array_equal(bs, q.reshape(ncols, K // 256, 16, 16).sum(-1))
    assert d[1, 0] == 0 and not q[1, 0].any()
    xb = x.reshape(ncols, K // 256, 256)
    idx = np.abs(xb).argmax(-1)
    live = d != 0
    assert np.all(np.take_along_axis(q, idx[..., None], -1)[..., 0][live] == -127)
    y = O.gemv_q8k(w, yk, K, nthreads=4)
    wd = O.dequant_q4k(w).reshape(N, K).astype(np.float64)
    xd = (q * d[:, :, None]).reshape(ncols, K)
    scale = np.abs(xd) @ np.abs(wd).T
    assert np.max(np.abs(y - xd @ wd.T) / scale) < 1e-6
    assert np.max(np.abs(y - x.astype(np.float64) @ wd.T) / (np.abs(x) @ np.abs(wd).T)) < 5e-3


def test_q8k_block_size_matches_gguf():
    """The gguf package (llama.cpp's Python tooling) gives block_q8_K as 256
    values in 292 bytes: fp32 d, 256 int8 and 16 int16 sums."""
    gguf = pytest.importorskip("gguf")
    assert gguf.GGML_QUANT_SIZES[gguf.GGMLQuantizationType.Q8_K] == (256, O.Q8K_BYTES)
    assert O.quantize_q8_K(np.ones((1, 512), dtype=np.float32)).shape == (1, 2 * O.Q8K_BYTES)
