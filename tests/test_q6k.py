"""CPU tests of the Q6_K oracle (no GPU).

Pins the canonical fp32 Q6_K GEMV three ways: against a loop-for-loop
restatement of the reference's f64 oracle (tests/runtime_kernel_test.cu:82-106)
on the reference test's shapes and input patterns (:119-123), against an
independent numpy decode of ggml's block_q6_K, and through its exact int32
sub-block dots.  Also checks the K-slice tree and the K-shard subtree
property that tensor parallelism relies on, and the C-ABI argument checks.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

TOL = 1e-5  # of sum_k |w_k| |x_k| per row


def _pattern(N, K, pattern, seed=0):
    """The reference test's three input patterns: 0 all-zero weights and
    input, 1 U(-1, 1) input, 2 weights scaled x100."""
    w = O.gen_q6k(N, K, seed, 40 + pattern)
    rng = np.random.default_rng(seed + 7)
    if pattern == 0:
        w = np.zeros_like(w)
        x = np.zeros((1, K), dtype=np.float32)
    else:
        x = rng.uniform(-1, 1, (1, K)).astype(np.float32)
    if pattern == 2:
        blocks = w.reshape(-1, 210)
        d = blocks[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
        d16 = np.array([O.lib.orc_f32_to_f16(float(v) * 100.0) for v in d], dtype=np.uint16)
        blocks[:, 208:210] = d16.view(np.uint8).reshape(-1, 2)
    return w, O.quantize_q8_1(x)


def _codes(w: np.ndarray) -> np.ndarray:
    """6-bit codes (nblocks, 256), decoded with numpy from the block layout."""
    b = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1, 210).astype(np.int32)
    q = np.empty((b.shape[0], 256), dtype=np.int32)
    for e in range(256):
        half, r = divmod(e, 128)
        group, lane = divmod(r, 32)
        qlb = b[:, half * 64 + lane + (group % 2) * 32]
        low = (qlb & 15) if group < 2 else (qlb >> 4)
        q[:, e] = low | (((b[:, 128 + half * 32 + lane] >> (2 * group)) & 3) << 4)
    return q


def test_generator_layout():
    w = O.gen_q6k(64, 2560, 3, 9)
    assert w.shape == (64, 10 * 210)
    b = w.reshape(-1, 210)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
    assert (d >= 0.0001 * 0.999).all() and (d <= 0.002 * 1.001).all()
    sc = b[:, 192:208].view(np.int8)
    assert sc.min() < -100 and sc.max() > 100  # full int8 range
    q = _codes(w)
    assert q.min() == 0 and q.max() == 63
    # row offsets continue the same stream
    assert np.array_equal(O.gen_q6k(10, 2560, 3, 9, row_offset=54), w[54:])


def test_dequant_c_matches_numpy_decoder():
    w = O.gen_q6k(33, 768, 1, 2)
    assert np.array_equal(O.dequant_q6k(w), O.dequant_q6k_numpy(w))


@pytest.mark.parametrize("pattern", [0, 1, 2])
@pytest.mark.parametrize("N", [1, 33, 64])
@pytest.mark.parametrize("K", [256, 768, 2048, 2560, 4096, 4864, 9728])
def test_canonical_matches_reference_f64_oracle(N, K, pattern):
    w, xq = _pattern(N, K, pattern)
    y = O.q6k_gemv(w, xq, K)
    y64 = O.q6k_gemv_f64(w, xq, K)
    scale = O.q6k_absdot_f64(w, xq, K)
    assert np.isfinite(y).all()
    if pattern == 0:
        assert not y.any() and not y64.any()
        return
    err = np.abs(y.astype(np.float64) - y64) / np.maximum(scale, 1e-30)
    assert err.max() <= TOL, err.max()


def test_f64_oracle_is_the_dequantized_dot():
    K = 2560
    w = O.gen_q6k(17, K, 5, 3)
    xq = O.quantize_q8_1(O.gen_normal_f32((2, K), 4))
    wd = O.dequant_q6k_numpy(w).astype(np.float64).reshape(17, K)
    xb = xq.reshape(2, K // 32, 36)
    d8 = xb[:, :, 0:2].copy().view(np.float16).astype(np.float64)[:, :, 0]
    q8 = xb[:, :, 4:].copy().view(np.int8).astype(np.float64)
    xd = (d8[:, :, None] * q8).reshape(2, K)
    ref = xd @ wd.T
    y64 = O.q6k_gemv_f64(w, xq, K)
    assert np.allclose(y64, ref, rtol=1e-12, atol=1e-9)


def test_partials_exact_against_numpy():
    N, K = 9, 768
    w = O.gen_q6k(N, K, 2, 6)
    xq = O.quantize_q8_1(O.gen_normal_f32((2, K), 5))
    P = O.q6k_partials(w, xq, K)
    q = _codes(w).reshape(N, K // 256, 256) - 32
    q8 = xq.reshape(2, K // 32, 36)[:, :, 4:].copy().view(np.int8).astype(np.int64).reshape(2, K // 256, 256)
    ref = np.einsum("rbe,cbe->crbe", q.astype(np.int64), q8).reshape(2, N, K // 256, 16, 16).sum(-1)
    assert np.array_equal(P, ref)


@pytest.mark.parametrize("nsb", [1, 3, 8, 10, 19, 38])
def test_slices_and_tree(nsb):
    K = nsb * 256
    w = O.gen_q6k(7, K, 1, 8)
    xq = O.quantize_q8_1(O.gen_normal_f32((3, K), 9))
    v = O.q6k_gemv_slices(w, xq, K)
    assert np.array_equal(O.tree8(v), O.q6k_gemv(w, xq, K))
    assert np.array_equal(O.q6k_gemv(w, xq, K, nthreads=4), O.q6k_gemv(w, xq, K))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kshard_partials_recombine_bit_exact(world):
    """Row-parallel shards of a Q6_K ffn_down (K = 9728) recombine exactly."""
    N, K = 40, 9728
    w = O.gen_q6k(N, K, 4, 21)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 8))
    slices = O.q6k_gemv_slices(w, xq, K)
    full = O.q6k_gemv(w, xq, K)
    per = 8 // world
    parts = [O.kshard_partial(slices, r * per, per) for r in range(world)]
    assert np.array_equal(O.delta_tree(parts), full)


def test_q6k_entry_points_reject_bad_arguments_without_gpu():
    import abra_b200 as A
    from abra_b200 import _lib

    lib = _lib.lib
    assert lib.abra_q6k_mmvq(0, 16, 16, 8, 256, 1, None) == _lib.ABRA_E_INVALID  # null
    assert lib.abra_q6k_mmvq(16, 16, 16, 8, 300, 1, None) == _lib.ABRA_E_INVALID  # K
    assert lib.abra_q6k_mmvq(16, 16, 16, 8, 256, 9, None) == _lib.ABRA_E_UNSUPPORTED  # ncols
    assert lib.abra_q6k_mmvq(18, 16, 16, 8, 256, 1, None) == _lib.ABRA_E_INVALID  # align
    assert lib.abra_q6k_mmvq_ex(16, 16, 16, 8, 256, 1, 4, 0, 0, None) == _lib.ABRA_E_INVALID  # ldy
    assert lib.abra_q6k_mmvq_ex(16, 16, 16, 8, 256, 1, 8, 4242, 0, None) == _lib.ABRA_E_INVALID
    assert "candidate" in _lib.last_error()
    # a K-shard whose width is not that of its canonical slices
    assert lib.abra_q6k_mmvq_kshard(16, 16, 16, 8, 512, 1, 9728, 0, 2, 0, 0, None) == _lib.ABRA_E_INVALID
    assert lib.abra_q6k_mmvq_kshard(16, 16, 16, 8, 256, 1, 9728, 0, 3, 0, 0, None) == _lib.ABRA_E_INVALID
    assert lib.abra_q6k_mmvq_partials(16, 16, 16, None, 8, 256, 1, None) == _lib.ABRA_E_INVALID
    assert lib.abra_gen_q6k(17, 4, 0, 0, 0, None) == _lib.ABRA_E_INVALID
    with pytest.raises(ValueError):
        A.mmvq_q6k(16, 16, 16, 8, 300)


def test_q6k_candidates_and_tuning():
    import abra_b200 as A

    c = A.q6k_candidates()
    assert len(c) >= 10
    for cid, s in c.items():
        assert s.ks in (1, 2, 4, 8) and s.mode in (0, 1, 2) and (s.mode != 1 or s.ks == 1)
    assert A.q6k_tune_get(151936, 2560) in c
    A.q6k_tune_set(777, 2560, 1, 1042)
    assert A.q6k_tune_get(777, 2560, 1) == 1042
    with pytest.raises(ValueError):
        A.q6k_tune_set(777, 2560, 1, 999999)


# Layers with Q6_K attn_v and ffn_down in Qwen3-4B-Q4_K_M, from the
# reference's GGUF census (bench/results/m3/qwen3-q4k-tensor-map.json).
CENSUS_Q6K_LAYERS = [0, 1, 2, 3, 6, 9, 12, 15, 18, 21, 24, 27, 30, 31, 32, 33, 34, 35]


def test_q4_k_m_type_map_matches_the_census():
    from abra_b200.model import q6k_layers

    assert q6k_layers(36) == CENSUS_Q6K_LAYERS
    assert [l for l in range(36) if O.lib.orc_q6k_layer(l, 36)] == CENSUS_Q6K_LAYERS
    for n in (2, 5, 9, 16):
        assert q6k_layers(n) == [l for l in range(n) if O.lib.orc_q6k_layer(l, n)]


def test_q4_k_m_model_is_single_gpu_batch_1_without_gpu():
    """Refused on the host, before any CUDA call."""
    import ctypes as C

    from abra_b200 import _lib
    from abra_b200.model import Q4_K_M, default_config

    cfg = default_config(flags=Q4_K_M)
    h = C.c_void_p()
    assert _lib.lib.abra_model_create_tp(C.byref(cfg), 0, 2, C.byref(h)) == _lib.ABRA_E_UNSUPPORTED
    assert _lib.lib.abra_model_create_batched(C.byref(cfg), 32, C.byref(h)) == _lib.ABRA_E_UNSUPPORTED
    assert b"Q4_K_M" in _lib.lib.abra_model_last_error()


def test_oracle_q4_k_m_model_differs_from_q4k_model():
    """A 2-layer oracle model under the type map (layer 1 Q6_K for n = 2,
    Q6_K tied table) gives other logits than the all-Q4_K model of the same
    seed."""
    cfg = dict(n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=1024, vocab=300, max_ctx=8, seed=1)
    a, b = O.OrcModel(**cfg), O.OrcModel(mix=1, **cfg)
    _, la = a.step(5, 0, logits=True)
    _, lb = b.step(5, 0, logits=True)
    assert np.isfinite(lb).all() and not np.array_equal(la, lb)
    a.close()
    b.close()


def test_tuning_file_q6k_entries(tmp_path):
    """q6k_entries of a tuning file feed the Q6_K table; the shipped file
    holds the measured winners of the real model's three Q6_K shapes."""
    import json

    import abra_b200 as A
    from abra_b200.q4k import TUNING_FILE, load_tuning_table

    p = tmp_path / "t.json"
    p.write_text(json.dumps({"entries": [], "q6k_entries": [{"N": 640, "K": 768, "ncols": 2, "candidate": 3082}]}))
    assert load_tuning_table(p) == 1
    assert A.q6k_tune_get(640, 768, 2) == 3082
    shipped = json.loads(TUNING_FILE.read_text())["q6k_entries"]
    assert {(e["N"], e["K"]) for e in shipped} == {(1024, 2560), (2560, 9728), (151936, 2560)}
    for e in shipped:
        assert A.q6k_tune_get(e["N"], e["K"], 1) == e["candidate"] == int(min(e["all_us"], key=e["all_us"].get))
