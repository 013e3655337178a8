"""Host-side mirror of the reference's Q4_K x Q8_1 operator interface.

Names, argument meaning and error behaviour follow the reference's C++ API
(talystalys/abra):

    launch_q4k_candidate            kernels/q4k/q4k_family.cuh:63-71
    launch_q4k_candidate_combined_pipeline   q4k_family.cuh:73-82
    launch_q4k_autotuned            kernels/q4k/q4k_family.cuh:89-97
    launch_q4k_autotuned_combined_pipeline   q4k_family.cuh:99-108
    launch_quantize_f32_to_q8_1     kernels/q4k/q4k_q8_mmvq.cuh:91-96
    get_all_candidate_ids / get_candidate_spec / get_candidate_name
                                    kernels/q4k/q4k_family.cuh:59-61
    register_autotuned_table_entry / get_autotuned_candidate_for_shape
                                    kernels/q4k/q4k_family.cuh:86-87

Where the reference throws std::invalid_argument (K % 256 != 0, unknown
candidate), these raise ValueError.  Buffers are torch CUDA tensors (or raw
device addresses as ints); every call is asynchronous on ``stream`` (default:
torch's current stream).  The candidates are the sm_100a family of
libabra_b200, not the reference's Pascal warp mappings; the tuned dispatch
reads ``tuning/sm100.json``.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass
from pathlib import Path

from . import _lib
from ._lib import call, lib

QK_K = 256
QK8_1 = 32
Q4K_BYTES = 144
Q81_BYTES = 36
ARCH_SM100 = 100
CANDIDATE_AUTOTUNED_DISPATCH = 0
TUNING_FILE = Path(__file__).resolve().parent / "tuning" / "sm100.json"


def ptr(t) -> int:
    """Device address of a torch tensor (or an int address)."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return t.data_ptr()


def stream_handle(stream=None) -> int:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def q4k_nbytes(N: int, K: int) -> int:
    return N * (K // QK_K) * Q4K_BYTES


def q8_1_nbytes(K: int, ncols: int = 1) -> int:
    return ncols * (K // QK8_1) * Q81_BYTES


# ----------------------------------------------------------- candidates ---
MODE_NAMES = {0: "TMAROWS", 1: "TMAWHOLE", 2: "DIRECT", 3: "LANE"}


@dataclass(frozen=True)
class Q4KCandidateSpec:
    id: int
    name: str
    mode: int        # 0 TMA per-row bulk copies, 1 TMA whole unit, 2 direct loads
    ks: int          # k-parts per row group (warps sharing 8 rows)
    ncw: int         # consumer warps per CTA
    ctas_per_sm: int
    stage_kb: int    # shared-memory budget of the weight ring

    @property
    def threads_per_block(self) -> int:
        return (self.ncw + (0 if self.mode == 2 else 1)) * 32


def _enumerate() -> dict[int, Q4KCandidateSpec]:
    out = {}
    for i in range(lib.abra_candidate_count()):
        vals = [C.c_int32() for _ in range(6)]
        call("abra_candidate_info", i, *[C.byref(v) for v in vals])
        cid, mode, ks, ncw, cps, skb = (v.value for v in vals)
        half = "_H" if (cid // 100) % 10 == 1 else ""  # ring sized for half an SM
        out[cid] = Q4KCandidateSpec(cid, f"Q4K_SM100_{MODE_NAMES[mode]}_KS{ks}_C{cps}{half}", mode, ks,
                                    ncw, cps, skb)
    return out


_CANDIDATES = _enumerate()


def get_all_candidate_ids() -> list[int]:
    return sorted(_CANDIDATES)


PLAN_FIELDS = ("grid", "threads", "nstage", "pitch", "stage_bytes", "smem", "row_groups",
               "stage_offset")


def plan_info(N: int, K: int, ncols: int = 1, candidate: int = 0, nmat: int = 1,
              fused_rmsnorm: bool = False, q6k: bool = False, K_full: int = 0, sl_base: int = 0,
              sl_cnt: int = 8, sm_count: int = 148) -> dict | None:
    """The launch plan the dispatch makes for one MMVQ call
    (abra_mmvq_plan_info), computed on the host: no GPU is needed when
    sm_count > 0.  None when the candidate has no plan for the shape."""
    import numpy as np

    out = np.zeros(8, dtype=np.int64)
    rc = lib.abra_mmvq_plan_info(14 if q6k else 12, candidate, N, K, ncols, nmat,
                                 1 if fused_rmsnorm else 0, K_full, sl_base, sl_cnt, sm_count,
                                 out.ctypes.data)
    if rc == _lib.ABRA_E_UNSUPPORTED:
        return None
    _lib.check(rc, "abra_mmvq_plan_info")
    return dict(zip(PLAN_FIELDS, (int(v) for v in out)))


def get_candidate_spec(cid: int) -> Q4KCandidateSpec:
    if cid not in _CANDIDATES:
        raise ValueError(f"Unknown Q4KCandidateID {cid}")
    return _CANDIDATES[cid]


def get_candidate_name(cid: int) -> str:
    if cid == CANDIDATE_AUTOTUNED_DISPATCH:
        return "Q4K_AUTOTUNED_DISPATCH"
    return get_candidate_spec(cid).name


# ------------------------------------------------------------ tuning ------
def register_autotuned_table_entry(N: int, K: int, arch: int, winning_candidate: int,
                                   ncols: int = 1, nmat: int = 1) -> None:
    if arch != ARCH_SM100:
        raise ValueError(f"only arch {ARCH_SM100} is tuned here (got {arch})")
    call("abra_tune_set", N, K, ncols, nmat, winning_candidate)


def get_autotuned_candidate_for_shape(N: int, K: int, arch: int = ARCH_SM100,
                                      ncols: int = 1, nmat: int = 1) -> int:
    return int(lib.abra_tune_get(N, K, ncols, nmat))


def load_tuning_table(path: Path | str = TUNING_FILE) -> int:
    """Register every entry of a tuning JSON file; returns the entry count."""
    p = Path(path)
    if not p.exists():
        return 0
    data = json.loads(p.read_text())
    n = 0
    for e in data.get("entries", []):
        call("abra_tune_set", int(e["N"]), int(e["K"]), int(e.get("ncols", 1)),
             int(e.get("nmat", 1)), int(e["candidate"]))
        n += 1
    for e in data.get("q6k_entries", []):  # the Q6_K MMVQ's table
        call("abra_q6k_tune_set", int(e["N"]), int(e["K"]), int(e.get("ncols", 1)),
             int(e["candidate"]))
        n += 1
    return n


# -------------------------------------------------------------- kernels ---
def _check_k(K: int) -> None:
    if K % QK_K != 0:
        raise ValueError(f"K must be a multiple of QK_K=256 (K={K})")


def launch_q4k_candidate(candidate: int, d_w, d_x, d_y, N: int, K: int, stream=None,
                         ncols: int = 1) -> None:
    _check_k(K)
    if candidate == CANDIDATE_AUTOTUNED_DISPATCH:
        return launch_q4k_autotuned(d_w, d_x, d_y, N, K, ARCH_SM100, stream, ncols=ncols)
    get_candidate_spec(candidate)
    call("abra_q4k_mmvq_candidate", candidate, ptr(d_w), ptr(d_x), ptr(d_y), N, K, ncols,
         stream_handle(stream))


def launch_q4k_autotuned(d_w, d_x, d_y, N: int, K: int, arch: int = ARCH_SM100, stream=None,
                         ncols: int = 1) -> None:
    _check_k(K)
    call("abra_q4k_mmvq", ptr(d_w), ptr(d_x), ptr(d_y), N, K, ncols, stream_handle(stream))


def mmvq(d_w, d_x, d_y, N: int, K: int, ncols: int = 1, ldy: int | None = None,
         candidate: int = 0, pdl: bool = False, stream=None) -> None:
    """y[c*ldy + r] = sum_k W[r,k] x[c,k] (full form of the C ABI)."""
    _check_k(K)
    call("abra_q4k_mmvq_ex", ptr(d_w), ptr(d_x), ptr(d_y), N, K, ncols,
         N if ldy is None else ldy, candidate, _lib.ABRA_MMVQ_PDL if pdl else 0,
         stream_handle(stream))


def pack_q4k(d_w, d_packed, nblocks: int, stream=None) -> None:
    """The reference's 148-byte prepack of nblocks Q4_K superblocks
    (abra_q4k_pack; kernels/q4k/abra-packed-q4.cuh:10-27)."""
    call("abra_q4k_pack", ptr(d_w), ptr(d_packed), nblocks, stream_handle(stream))


def mmvq_packed(d_wp, d_x, d_y, N: int, K: int, pdl: bool = False, stream=None) -> None:
    """y = W x at batch 1 over packed weights (abra_q4k_mmvq_packed)."""
    _check_k(K)
    call("abra_q4k_mmvq_packed", ptr(d_wp), ptr(d_x), ptr(d_y), N, K,
         _lib.ABRA_MMVQ_PDL if pdl else 0, stream_handle(stream))


def mmvq_swiglu(d_w_gate, d_w_up, d_x, d_y, N: int, K: int, ncols: int = 1,
                ldy: int | None = None, candidate: int = 0, pdl: bool = False,
                stream=None) -> None:
    """y = (W_up x) * silu(W_gate x), one pass over the shared activation."""
    _check_k(K)
    call("abra_q4k_mmvq_swiglu", ptr(d_w_gate), ptr(d_w_up), ptr(d_x), ptr(d_y), N, K, ncols,
         N if ldy is None else ldy, candidate, _lib.ABRA_MMVQ_PDL if pdl else 0,
         stream_handle(stream))


def mmvq_rmsnorm(d_w, d_x, d_norm_w, eps: float, d_y, N: int, K: int, d_w_up=None,
                 d_x_q8_out=None, candidate: int = 0, pdl: bool = False, stream=None) -> None:
    """y = W Q8_1(RMSNorm(x) * norm_w) at batch 1 with the normalization and
    the quantization in each CTA's prologue (abra_q4k_mmvq_rmsnorm); with
    d_w_up the fused gate/up SwiGLU.  Bit-identical to rmsnorm_quantize_q8_1
    followed by mmvq / mmvq_swiglu."""
    _check_k(K)
    call("abra_q4k_mmvq_rmsnorm", ptr(d_w), ptr(d_w_up), ptr(d_x), ptr(d_norm_w), eps, ptr(d_y),
         ptr(d_x_q8_out), N, K, candidate, _lib.ABRA_MMVQ_PDL if pdl else 0, stream_handle(stream))


def mmvq_kshard(d_w, d_x, d_y, N: int, K: int, K_full: int, sl_base: int, sl_cnt: int,
                ncols: int = 1, candidate: int = 0, pdl: bool = False, stream=None) -> None:
    """Row-parallel MMVQ over canonical K-slices [sl_base, sl_base + sl_cnt)
    of K_full (see abra_q4k_mmvq_kshard): y gets this shard's partial sums."""
    _check_k(K)
    call("abra_q4k_mmvq_kshard", ptr(d_w), ptr(d_x), ptr(d_y), N, K, ncols, K_full, sl_base,
         sl_cnt, candidate, _lib.ABRA_MMVQ_PDL if pdl else 0, stream_handle(stream))


def mmvq_tc(d_w, d_x, d_y, N: int, K: int, ks: int = 1, d_workspace=None, ldy: int | None = None,
            pdl: bool = False, stream=None) -> None:
    """Batch-32 MMVQ on the tcgen05 tensor cores (32 Q8_1 columns): bit-identical
    to :func:`mmvq`; ks > 1 splits K over CTAs and needs ks*32*N floats of
    workspace."""
    _check_k(K)
    call("abra_q4k_mmvq_tc", ptr(d_w), ptr(d_x), ptr(d_y), N, K, 32, N if ldy is None else ldy, ks,
         ptr(d_workspace), _lib.ABRA_MMVQ_PDL if pdl else 0, stream_handle(stream))


def slice_start(nsb: int, i: int) -> int:
    """First superblock of canonical K-slice i of a row of nsb superblocks."""
    return i * (nsb // 8) + min(i, nsb % 8)


def mmvq_partials(d_w, d_x, d_y, d_P, d_M, N: int, K: int, ncols: int = 1, ks: int = 1,
                  stream=None) -> None:
    _check_k(K)
    call("abra_q4k_mmvq_partials", ptr(d_w), ptr(d_x), ptr(d_y), ptr(d_P), ptr(d_M), N, K,
         ncols, ks, stream_handle(stream))


def launch_quantize_f32_to_q8_1(d_x_f32, d_x_q8, K: int, stream=None, ncols: int = 1) -> None:
    if K % QK8_1 != 0:
        raise ValueError(f"K must be a multiple of QK8_1=32 (K={K})")
    call("abra_quantize_q8_1", ptr(d_x_f32), ptr(d_x_q8), K, ncols, stream_handle(stream))


launch_custom_reference_q8_1_quantizer = launch_quantize_f32_to_q8_1


def rmsnorm_quantize_q8_1(d_x, d_w, eps: float, d_x_q8, K: int, ncols: int = 1,
                          d_xn_out=None, stream=None) -> None:
    call("abra_rmsnorm_quantize_q8_1", ptr(d_x), ptr(d_w), eps, ptr(d_x_q8), ptr(d_xn_out), K,
         ncols, stream_handle(stream))


def launch_q4k_candidate_combined_pipeline(candidate: int, d_w, d_x_f32, d_x_q8_scratch, d_y,
                                           N: int, K: int, stream=None, ncols: int = 1) -> None:
    _check_k(K)
    if candidate != CANDIDATE_AUTOTUNED_DISPATCH:
        get_candidate_spec(candidate)
    cid = 0 if candidate == CANDIDATE_AUTOTUNED_DISPATCH else candidate
    call("abra_q4k_mmvq_combined", cid, ptr(d_w), ptr(d_x_f32), ptr(d_x_q8_scratch),
         ptr(d_y), N, K, ncols, stream_handle(stream))


def launch_q4k_autotuned_combined_pipeline(d_w, d_x_f32, d_x_q8_scratch, d_y, N: int, K: int,
                                           arch: int = ARCH_SM100, stream=None,
                                           ncols: int = 1) -> None:
    _check_k(K)
    call("abra_q4k_mmvq_combined", 0, ptr(d_w), ptr(d_x_f32), ptr(d_x_q8_scratch), ptr(d_y), N,
         K, ncols, stream_handle(stream))


# ------------------------------------------------------------ generator ---
def gen_q4k(d_dst, nblocks: int, seed: int, tensor_id: int, block_offset: int = 0,
            stream=None) -> None:
    call("abra_gen_q4k", ptr(d_dst), nblocks, seed, tensor_id, block_offset,
         stream_handle(stream))


def gen_uniform_f32(d_dst, n: int, seed: int, tensor_id: int, scale: float, offset: float,
                    offset_index: int = 0, stream=None) -> None:
    call("abra_gen_uniform_f32", ptr(d_dst), n, seed, tensor_id, offset_index, scale, offset,
         stream_handle(stream))


def device_error(clear: bool = True) -> int:
    v = C.c_uint32(0)
    call("abra_device_error", C.byref(v), 1 if clear else 0)
    return v.value


load_tuning_table()
