"""CPU tests of the C-ABI boundary: the library loads, exports every symbol
include/abra_b200.h declares, and rejects bad arguments before touching the
GPU (the reference throws std::invalid_argument in the same cases,
kernels/q4k/q4k_q8_mmvq.cu:266-268, kernels/q4k/q4k_family.cu:200-202)."""
from __future__ import annotations

import ctypes as C
import re

import pytest

from conftest import ROOT


def header_symbols() -> list[str]:
    text = (ROOT / "include" / "abra_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)) - {"if", "defined"})


def test_library_loads_and_exports_header_symbols():
    import abra_b200
    from abra_b200 import _lib

    lib = C.CDLL(str(abra_b200.LIB_PATH))
    syms = header_symbols()
    assert "abra_q4k_mmvq" in syms and "launch_pinned_upstream_mmvq" in syms
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, f"symbols declared but not exported: {missing}"
    assert set(syms) <= set(_lib.SIGNATURES), "ctypes signatures must cover the header"
    assert abra_b200.__version__.startswith("abra_b200")


def test_candidates_and_tuning_table():
    import abra_b200 as A

    ids = A.get_all_candidate_ids()
    assert len(ids) >= 8 and len(set(ids)) == len(ids)
    for cid in ids:
        s = A.get_candidate_spec(cid)
        assert s.ks in (1, 2, 4, 8) and s.ncw % s.ks == 0 and s.threads_per_block % 32 == 0
        assert s.mode in (0, 1, 2, 3) and (s.mode != 1 or s.ks == 1)
    with pytest.raises(ValueError):
        A.get_candidate_spec(12345)
    A.register_autotuned_table_entry(777, 2560, 100, ids[0])
    assert A.get_autotuned_candidate_for_shape(777, 2560, 100) == ids[0]
    with pytest.raises(ValueError):
        A.register_autotuned_table_entry(777, 2560, 100, 999999)
    assert A.get_autotuned_candidate_for_shape(999, 4096) in ids


@pytest.mark.parametrize("K", [255, 100, 2560 + 32])
def test_rejects_k_not_multiple_of_256(K):
    import abra_b200 as A

    with pytest.raises(ValueError, match="multiple of QK_K"):
        A.launch_q4k_autotuned(16, 16, 16, 8, K)
    rc = A._lib.lib.abra_q4k_mmvq(16, 16, 16, 8, K, 1, None)
    assert rc == A._lib.ABRA_E_INVALID and "QK_K" in A._lib.last_error()


def test_rejects_bad_arguments_without_gpu():
    import abra_b200 as A
    from abra_b200 import _lib

    lib = _lib.lib
    assert lib.abra_q4k_mmvq(0, 16, 16, 8, 256, 1, None) == _lib.ABRA_E_INVALID  # null
    assert lib.abra_q4k_mmvq(16, 16, 16, 0, 256, 1, None) == _lib.ABRA_E_INVALID  # N=0
    assert lib.abra_q4k_mmvq(16, 16, 16, 8, 256, 9, None) == _lib.ABRA_E_UNSUPPORTED  # ncols
    assert lib.abra_q4k_mmvq(17, 16, 16, 8, 256, 1, None) == _lib.ABRA_E_INVALID  # align
    assert "16-byte" in _lib.last_error()
    assert lib.abra_q4k_mmvq_ex(16, 16, 16, 8, 256, 1, 4, 0, 0, None) == _lib.ABRA_E_INVALID  # ldy
    assert lib.abra_quantize_q8_1(16, 16, 33, 1, None) == _lib.ABRA_E_INVALID
    assert lib.abra_q4k_mmvq_combined(0, 16, None, 16, 16, 8, 256, 1, None) == _lib.ABRA_E_INVALID
    assert lib.abra_q4k_mmvq_combined(0, 16, 16, 16, 16, 8, 300, 1, None) == _lib.ABRA_E_INVALID
    # an unknown candidate is refused before the quantize launch: with no GPU
    # here a launch would fail as ABRA_E_CUDA, so E_INVALID shows nothing ran
    assert lib.abra_q4k_mmvq_combined(4242, 16, 16, 16, 16, 8, 256, 1, None) == _lib.ABRA_E_INVALID
    assert "candidate" in _lib.last_error()
    assert lib.abra_rmsnorm_quantize_q8_1(16, 16, 1e-6, 16, None, 32768, 1, None) == _lib.ABRA_E_INVALID
    assert lib.abra_rmsnorm_quantize_q8_1(16, 18, 1e-6, 16, None, 2560, 1, None) == _lib.ABRA_E_INVALID
    assert "4-byte" in _lib.last_error()
    assert lib.abra_rmsnorm_quantize_q8_1(16, 16, 1e-6, 16, 34, 2560, 1, None) == _lib.ABRA_E_INVALID
    assert lib.abra_gen_uniform_f32(18, 8, 0, 0, 0, 1.0, 0.0, None) == _lib.ABRA_E_INVALID
    assert "4-byte" in _lib.last_error()
    # fused RMSNorm MMVQ (w, w_up, x, norm_w, eps, y, x_q8_out, N, K, candidate, flags,
    # stream): every call below fails its argument checks before any launch
    rms = lib.abra_q4k_mmvq_rmsnorm
    assert rms(None, None, 16, 16, 1e-6, 16, None, 64, 2560, 0, 0, None) == _lib.ABRA_E_INVALID
    assert rms(16, None, 16, 16, 1e-6, 16, None, 64, 2000, 0, 0, None) == _lib.ABRA_E_INVALID
    assert rms(16, None, 16, 16, 1e-6, 16, None, 64, 32768, 0, 0, None) == _lib.ABRA_E_UNSUPPORTED
    assert rms(16, 24, 16, 16, 1e-6, 16, None, 64, 2560, 0, 0, None) == _lib.ABRA_E_INVALID
    assert rms(16, None, 16, 20, 1e-6, 16, None, 64, 2560, 0, 0, None) == _lib.ABRA_E_INVALID
    assert rms(16, None, 18, 16, 1e-6, 16, None, 64, 2560, 0, 0, None) == _lib.ABRA_E_INVALID
    assert rms(16, None, 16, 16, 1e-6, 16, 34, 64, 2560, 0, 0, None) == _lib.ABRA_E_INVALID
    assert rms(16, None, 16, 16, 1e-6, 16, None, 64, 2560, 4242, 0, None) == _lib.ABRA_E_INVALID
    with pytest.raises(ValueError):
        A.launch_quantize_f32_to_q8_1(16, 16, 33)
    with pytest.raises(ValueError):
        A.launch_q4k_candidate(999999, 16, 16, 16, 8, 256)


def test_tensor_core_mmvq_rejects_bad_arguments_without_gpu():
    import abra_b200 as A
    from abra_b200 import _lib

    lib = _lib.lib
    assert lib.abra_q4k_mmvq_tc(16, 16, 16, 128, 256, 8, 128, 1, None, 0, None) == _lib.ABRA_E_UNSUPPORTED
    assert lib.abra_q4k_mmvq_tc(16, 16, 16, 128, 256, 32, 128, 2, None, 0, None) == _lib.ABRA_E_INVALID
    assert "workspace" in _lib.last_error()
    assert lib.abra_q4k_mmvq_tc(16, 16, 16, 128, 256, 32, 128, 3, None, 0, None) == _lib.ABRA_E_INVALID
    with pytest.raises(ValueError):
        A.mmvq_tc(16, 16, 16, 128, 300)


def test_new_model_entry_points_refuse_a_null_model():
    from abra_b200 import _lib

    lib = _lib.lib
    assert lib.abra_model_prefill(None, 32) == _lib.ABRA_E_INVALID
    assert lib.abra_model_prefill(None, 33) == _lib.ABRA_E_INVALID
    assert lib.abra_model_verify(None, None, 0, None, None) == _lib.ABRA_E_INVALID
    assert lib.abra_model_load_tensor(None, -1, 1, 12, None, 0) == _lib.ABRA_E_INVALID
    assert lib.abra_lookup_draft(None, -1, 2, 4, None) == _lib.ABRA_E_INVALID
    assert lib.abra_lookup_draft(None, 0, 2, 4, None) == _lib.ABRA_E_INVALID  # limit > 0, no out


def test_tuner_tie_break():
    """Within 0.5 % of the fastest the lowest candidate id wins (the band of
    the reference's table synthesis, tools/run-m4-autotune.py:196-206)."""
    from abra_b200.tune import pick_winner

    assert pick_winner({3012: 10.0, 1011: 10.03, 2011: 9.99}) == 1011  # 10.03 <= 9.99 * 1.005
    assert pick_winner({3012: 10.0, 1011: 10.2, 2011: 9.99}) == 2011
    assert pick_winner({1042: 5.0}) == 1042
    with pytest.raises(ValueError):
        pick_winner({})
