"""Q6_K x Q8_1 MMVQ: the Q6_K leg of the reference's MMVQ dispatch.

The reference dispatches ``abra_dispatch_mmvq<GGML_TYPE_Q6_K>``
(kernels/q4k/abra-mmvq.cuh:209-221), whose inner product is ggml's
vec_dot_q6_K_q8_1 (abra-mmvq.cuh:138-141); its test checks it against an
f64 oracle (tests/runtime_kernel_test.cu:82-106) on N in {1, 33, 64} and K
from 256 to 9728.  Here the same product runs in libabra_b200.so with exact
int32 16-weight dots and a fixed fp32 order (abra_q6k_mmvq in
include/abra_b200.h).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib
from ._lib import call
from .q4k import QK_K, _check_k, ptr, stream_handle

Q6K_BYTES = 210


def q6k_nbytes(N: int, K: int) -> int:
    """Bytes of an N x K Q6_K matrix (K a multiple of 256)."""
    return N * (K // QK_K) * Q6K_BYTES


@dataclass(frozen=True)
class Q6KCandidateSpec:
    id: int
    mode: int  # 0 per-row bulk copies, 1 whole-unit copy, 2 direct loads
    ks: int
    ctas_per_sm: int
    stage_kb: int


def q6k_candidates() -> dict[int, Q6KCandidateSpec]:
    out = {}
    for i in range(_lib.lib.abra_q6k_candidate_count()):
        v = [C.c_int32() for _ in range(5)]
        call("abra_q6k_candidate_info", i, *[C.byref(x) for x in v])
        spec = Q6KCandidateSpec(*[x.value for x in v])
        out[spec.id] = spec
    return out


def mmvq_q6k(d_w, d_x, d_y, N: int, K: int, ncols: int = 1, ldy: int | None = None,
             candidate: int = 0, pdl: bool = False, stream=None) -> None:
    """y[c*ldy + r] = sum_k W[r,k] x[c,k] for Q6_K rows W and Q8_1 columns x."""
    _check_k(K)
    call("abra_q6k_mmvq_ex", ptr(d_w), ptr(d_x), ptr(d_y), N, K, ncols,
         N if ldy is None else ldy, candidate, _lib.ABRA_MMVQ_PDL if pdl else 0,
         stream_handle(stream))


def mmvq_q6k_kshard(d_w, d_x, d_y, N: int, K: int, K_full: int, sl_base: int, sl_cnt: int,
                    ncols: int = 1, candidate: int = 0, pdl: bool = False, stream=None) -> None:
    """Row-parallel Q6_K MMVQ over canonical K-slices [sl_base, sl_base + sl_cnt)."""
    _check_k(K)
    call("abra_q6k_mmvq_kshard", ptr(d_w), ptr(d_x), ptr(d_y), N, K, ncols, K_full, sl_base,
         sl_cnt, candidate, _lib.ABRA_MMVQ_PDL if pdl else 0, stream_handle(stream))


def mmvq_q6k_partials(d_w, d_x, d_y, d_P, N: int, K: int, ncols: int = 1, stream=None) -> None:
    """Same product, also storing the exact int32 16-weight dots P[c][r][b][16]."""
    _check_k(K)
    call("abra_q6k_mmvq_partials", ptr(d_w), ptr(d_x), ptr(d_y), ptr(d_P), N, K, ncols,
         stream_handle(stream))


def gen_q6k(d_dst, nblocks: int, seed: int, tensor_id: int, block_offset: int = 0,
            stream=None) -> None:
    """Seeded synthetic Q6_K blocks (the oracle's gen_q6k stream, on the device)."""
    call("abra_gen_q6k", ptr(d_dst), nblocks, seed, tensor_id, block_offset,
         stream_handle(stream))


def q6k_tune_set(N: int, K: int, ncols: int, candidate: int) -> None:
    call("abra_q6k_tune_set", N, K, ncols, candidate)


def q6k_tune_get(N: int, K: int, ncols: int = 1) -> int:
    return _lib.lib.abra_q6k_tune_get(N, K, ncols)
