"""The adapter ABI's two host functions (kernels/q4k/upstream_adapter.cuh:28-38)
exported by libabra_b200.so: quantize_row_q4_K_upstream_cpu and
dequantize_row_q4_K_upstream_cpu.  CPU only.

The reference forwards them to llama.cpp's quantize_row_q4_K_ref and
dequantize_row_q4_K (not in this image).  Dequantization is the format's
definition and is checked bit for bit against the gguf package's Q4_K
decoder (llama.cpp's own Python tooling).  The quantizer restates the
published Q4_K algorithm; gguf has no Q4_K quantizer and llama.cpp is absent,
so its codes are checked by properties: round-trip error bounds per input
family, exact zeros, determinism, and the argument check."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from abra_b200 import _lib

gguf_quants = pytest.importorskip("gguf.quants")


def quantize(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.zeros(x.size // 256 * 144, dtype=np.uint8)
    _lib.lib.quantize_row_q4_K_upstream_cpu(x.ctypes.data, q.ctypes.data, x.size)
    return q


def dequantize(q: np.ndarray, k: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    y = np.zeros(k, dtype=np.float32)
    _lib.lib.dequantize_row_q4_K_upstream_cpu(q.ctypes.data, y.ctypes.data, k)
    return y


@pytest.mark.parametrize("centered", [0, 1])
def test_dequantize_matches_gguf_bit_for_bit(centered):
    w = O.gen_q4k(64, 2560, seed=3, tensor_id=5, centered=centered).reshape(-1)
    y = dequantize(w, 64 * 2560)
    want = gguf_quants.Q4_K.dequantize_blocks(w.reshape(-1, 144)).reshape(-1).astype(np.float32)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


FAMILIES = {
    # name: (generator, bound on the relative RMS error of the round trip)
    "normal": (lambda r, n: r.standard_normal(n), 0.08),
    "uniform": (lambda r, n: r.uniform(-1.0, 1.0, n), 0.065),
    "positive": (lambda r, n: r.uniform(0.0, 3.0, n), 0.04),
    "outliers": (lambda r, n: r.standard_normal(n) * np.where(r.random(n) < 0.01, 20.0, 1.0), 0.12),
    "wide": (lambda r, n: r.standard_normal(n) * 1e3, 0.08),
}


@pytest.mark.parametrize("family", sorted(FAMILIES))
def test_round_trip_error(family):
    gen, bound = FAMILIES[family]
    x = gen(np.random.default_rng(7), 256 * 96).astype(np.float32)
    q = quantize(x)
    y = dequantize(q, x.size)
    rel = np.sqrt(np.mean((x - y) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < bound, rel
    blocks = q.reshape(-1, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32)
    assert np.all(np.isfinite(d)) and np.all(d >= 0) and np.all(np.isfinite(dmin)) and np.all(dmin >= 0)
    # every superblock reconstructs within its own quantization steps
    step = (d * 63.0 + dmin * 63.0).reshape(-1, 1)
    err = np.abs(x - y).reshape(-1, 256)
    assert np.all(err <= step + 1e-6)


def test_zero_row_is_exactly_zero_and_deterministic():
    x = np.zeros(512, dtype=np.float32)
    q = quantize(x)
    assert not q.any()
    assert not dequantize(q, 512).any()
    r = np.random.default_rng(1).standard_normal(2560).astype(np.float32)
    assert np.array_equal(quantize(r), quantize(r))


def test_k_not_a_multiple_of_256_writes_nothing():
    x = np.ones(300, dtype=np.float32)
    q = np.full(2 * 144, 0xAB, dtype=np.uint8)
    _lib.lib.quantize_row_q4_K_upstream_cpu(x.ctypes.data, q.ctypes.data, 300)
    assert np.all(q == 0xAB)
    assert "256" in _lib.last_error()
    y = np.full(300, 7.0, dtype=np.float32)
    _lib.lib.dequantize_row_q4_K_upstream_cpu(q.ctypes.data, y.ctypes.data, 300)
    assert np.all(y == 7.0)
