"""CPU oracle of the Q4_K x Q8_1 decode path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package, and only as the reference result (or the timed CPU restatement); the product
library never imports it.

``liborc.so`` (q4k_oracle.c) restates the reference's arithmetic in C:
block layouts kernels/q4k/q4k_q8_mmvq.cuh:42-57, scale unpack
tests/q4k_q8_test.cu:44-52, the f64 oracle tests/q4k_q8_test.cu:54-107,
vec_dot_q4_K_q8_1 kernels/q4k/q4k_vecdot.cuh:23-87 and the Q8_1 quantizer
kernels/q4k/q4k_q8_mmvq.cu:223-255 (paths inside talystalys/abra);
q6k_oracle.c the Q6_K leg of the dispatch (kernels/q4k/abra-mmvq.cuh:138-141)
with the reference's f64 Q6_K oracle tests/runtime_kernel_test.cu:82-106.

``_ref/libq4k_ref.so`` is the reference's own kernel family compiled from its
sources (see Makefile); ``ref`` binds it when present.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORC_PATH = HERE / "liborc.so"
REF_PATH = HERE / "_ref" / "libq4k_ref.so"

QK_K, QK8_1, Q4K_BYTES, Q81_BYTES, Q6K_BYTES = 256, 32, 144, 36, 210

_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64, _i32, _u64, _f32 = C.c_int64, C.c_int32, C.c_uint64, C.c_float


def build(ref: bool = True) -> None:
    """Build liborc.so (and _ref/ when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all" if ref else "orc"], check=True)


def _load() -> C.CDLL:
    if not ORC_PATH.exists():
        build(ref=False)
    lib = C.CDLL(str(ORC_PATH))
    sig = {
        "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_gen_q4k": (None, [_u8p, _i64, _u64, _u64, _i64]),
        "orc_gen_q4k_ex": (None, [_u8p, _i64, _u64, _u64, _i64, _i32]),
        "orc_gen_norm_f32": (None, [_f32p, _i64, _u64, _u64]),
        "orc_gen_uniform_f32": (None, [_f32p, _i64, _u64, _u64, _i64, _f32, _f32]),
        "orc_quantize_q8_1": (None, [_f32p, _u8p, _i64, _i32]),
        "orc_rmsnorm_quantize_q8_1": (None, [_f32p, _f32p, _f32, _u8p, C.c_void_p, _i64, _i32]),
        "orc_rms_scale": (C.c_float, [_f32p, _f32, _i64]),
        "orc_q4k_partials": (None, [_u8p, _u8p, _i32p, _i32p, _i64, _i64, _i32]),
        "orc_q4k_gemv": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i32, _i32]),
        "orc_q4k_gemv_slices": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i32]),
        "orc_q4k_gemv_f64": (None, [_u8p, _u8p, _f64p, _i64, _i64, _i32]),
        "orc_q4k_absdot_f64": (None, [_u8p, _u8p, _f64p, _i64, _i64, _i32]),
        "orc_dequant_q4k": (None, [_u8p, _f32p, _i64]),
        "orc_slice_starts": (None, [_i32, _i32p]),
        "orc_max_threads": (C.c_int32, []),
        "orc_simd_level": (C.c_int32, []),
        "orc_set_simd_level": (None, [C.c_int32]),
        "orc_expf": (C.c_float, [C.c_float]),
        "orc_silu": (C.c_float, [C.c_float]),
        "orc_swiglu": (None, [_f32p, _f32p, _f32p, _i64]),
        "orc_gen_q6k": (None, [_u8p, _i64, _u64, _u64, _i64]),
        "orc_q6k_partials": (None, [_u8p, _u8p, _i32p, _i64, _i64, _i32]),
        "orc_q6k_gemv": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i32, _i32]),
        "orc_q6k_gemv_slices": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i32]),
        "orc_q6k_gemv_f64": (None, [_u8p, _u8p, _f64p, _i64, _i64, _i32]),
        "orc_q6k_absdot_f64": (None, [_u8p, _u8p, _f64p, _i64, _i64, _i32]),
        "orc_dequant_q6k": (None, [_u8p, _f32p, _i64]),
        "orc_quantize_q8_K": (None, [_f32p, _u8p, _i64, _i32]),
        "orc_q4k_q8k_gemv": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i32, _i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


lib = _load()


# ------------------------------------------------------------ generators ---
def gen_q4k(N: int, K: int, seed: int, tensor_id: int, row_offset: int = 0,
            centered: bool = False) -> np.ndarray:
    """Q4_K rows [row_offset, row_offset+N) of a K-wide tensor, as uint8 (N, K/256*144)."""
    nsb = K // QK_K
    out = np.empty(N * nsb * Q4K_BYTES, dtype=np.uint8)
    lib.orc_gen_q4k_ex(out, N * nsb, seed, tensor_id, row_offset * nsb, 1 if centered else 0)
    return out.reshape(N, nsb * Q4K_BYTES)


def gen_norm_f32(n: int, seed: int, tensor_id: int) -> np.ndarray:
    """+-U(0.8, 1.2) with a random sign: the synthetic model's norm weights."""
    out = np.empty(n, dtype=np.float32)
    lib.orc_gen_norm_f32(out, n, seed, tensor_id)
    return out


def gen_uniform_f32(n: int, seed: int, tensor_id: int, scale: float, offset: float,
                    offset_index: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib.orc_gen_uniform_f32(out, n, seed, tensor_id, offset_index, scale, offset)
    return out


def gen_normal_f32(shape, seed: int) -> np.ndarray:
    """x ~ N(0, 1), host-side only (numpy PCG64)."""
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


# -------------------------------------------------------------- Q8_1 ------
def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    """x: (ncols, K) or (K,) fp32 -> uint8 (ncols, K/32*36)."""
    x2 = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    ncols, K = x2.shape
    out = np.empty(ncols * (K // QK8_1) * Q81_BYTES, dtype=np.uint8)
    lib.orc_quantize_q8_1(x2, out, K, ncols)
    return out.reshape(ncols, -1)


def rmsnorm_quantize_q8_1(x: np.ndarray, w: np.ndarray, eps: float):
    x2 = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    ncols, K = x2.shape
    q = np.empty(ncols * (K // QK8_1) * Q81_BYTES, dtype=np.uint8)
    xn = np.empty((ncols, K), dtype=np.float32)
    lib.orc_rmsnorm_quantize_q8_1(x2, np.ascontiguousarray(w, dtype=np.float32), eps, q,
                                  xn.ctypes.data, K, ncols)
    return q.reshape(ncols, -1), xn


# -------------------------------------------------------------- MMVQ ------
def _shape(w: np.ndarray, xq: np.ndarray, K: int):
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    xq2 = np.ascontiguousarray(np.atleast_2d(xq), dtype=np.uint8)
    ncols = xq2.shape[0]
    N = w.size // ((K // QK_K) * Q4K_BYTES)
    return w, xq2.reshape(-1), N, ncols


def partials(w, xq, K: int):
    """Exact int32 P (ncols, N, K/256, 8) and M (ncols, K/256, 8)."""
    w, xq, N, ncols = _shape(w, xq, K)
    nsb = K // QK_K
    P = np.empty(ncols * N * nsb * 8, dtype=np.int32)
    M = np.empty(ncols * nsb * 8, dtype=np.int32)
    lib.orc_q4k_partials(w, xq, P, M, N, K, ncols)
    return P.reshape(ncols, N, nsb, 8), M.reshape(ncols, nsb, 8)


def gemv(w, xq, K: int, nthreads: int = 1) -> np.ndarray:
    """Canonical fp32 GEMV (bit-exact target of the CUDA kernels), (ncols, N)."""
    w, xq, N, ncols = _shape(w, xq, K)
    y = np.empty(ncols * N, dtype=np.float32)
    lib.orc_q4k_gemv(w, xq, y, N, K, ncols, nthreads)
    return y.reshape(ncols, N)


Q8K_BYTES = 292  # block_q8_K: fp32 d, 256 int8, 16 int16 sums


def quantize_q8_K(x: np.ndarray) -> np.ndarray:
    """llama.cpp's CPU activation format, restated: x (ncols, K) fp32 ->
    uint8 (ncols, K/256*292)."""
    x2 = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    ncols, K = x2.shape
    out = np.empty(ncols * (K // QK_K) * Q8K_BYTES, dtype=np.uint8)
    lib.orc_quantize_q8_K(x2, out, K, ncols)
    return out.reshape(ncols, -1)


def gemv_q8k(w, yk, K: int, nthreads: int = 1) -> np.ndarray:
    """llama.cpp's CPU Q4_K x Q8_K dot, restated (the timed CPU baseline, not
    a parity target), (ncols, N)."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    yk2 = np.ascontiguousarray(np.atleast_2d(yk), dtype=np.uint8)
    ncols, N = yk2.shape[0], w.size // ((K // QK_K) * Q4K_BYTES)
    y = np.empty(ncols * N, dtype=np.float32)
    lib.orc_q4k_q8k_gemv(w, yk2.reshape(-1), y, N, K, ncols, nthreads)
    return y.reshape(ncols, N)


def gemv_slices(w, xq, K: int) -> np.ndarray:
    w, xq, N, ncols = _shape(w, xq, K)
    v = np.empty(ncols * N * 8, dtype=np.float32)
    lib.orc_q4k_gemv_slices(w, xq, v, N, K, ncols)
    return v.reshape(ncols, N, 8)


def gemv_f64(w, xq, K: int) -> np.ndarray:
    w, xq, N, ncols = _shape(w, xq, K)
    y = np.empty(ncols * N, dtype=np.float64)
    lib.orc_q4k_gemv_f64(w, xq, y, N, K, ncols)
    return y.reshape(ncols, N)


def absdot_f64(w, xq, K: int) -> np.ndarray:
    w, xq, N, ncols = _shape(w, xq, K)
    s = np.empty(ncols * N, dtype=np.float64)
    lib.orc_q4k_absdot_f64(w, xq, s, N, K, ncols)
    return s.reshape(ncols, N)


def dequant_q4k(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    nb = w.size // Q4K_BYTES
    out = np.empty(nb * QK_K, dtype=np.float32)
    lib.orc_dequant_q4k(w, out, nb)
    return out


def slice_starts(nsb: int) -> np.ndarray:
    s = np.empty(9, dtype=np.int32)
    lib.orc_slice_starts(nsb, s)
    return s


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """up * silu(gate), elementwise, in the kernels' operation order."""
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32)
    y = np.empty_like(g)
    lib.orc_swiglu(g.reshape(-1), u.reshape(-1), y.reshape(-1), g.size)
    return y


def gemv_swiglu(w_gate, w_up, xq, K: int, nthreads: int = 1) -> np.ndarray:
    return swiglu(gemv(w_gate, xq, K, nthreads), gemv(w_up, xq, K, nthreads))


# -------------------------------------------------------------- Q6_K ------
def gen_q6k(N: int, K: int, seed: int, tensor_id: int, row_offset: int = 0) -> np.ndarray:
    """Q6_K rows [row_offset, row_offset+N) of a K-wide tensor, uint8 (N, K/256*210)."""
    nsb = K // QK_K
    out = np.empty(N * nsb * Q6K_BYTES, dtype=np.uint8)
    lib.orc_gen_q6k(out, N * nsb, seed, tensor_id, row_offset * nsb)
    return out.reshape(N, nsb * Q6K_BYTES)


def _shape6(w: np.ndarray, xq: np.ndarray, K: int):
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    xq2 = np.ascontiguousarray(np.atleast_2d(xq), dtype=np.uint8)
    ncols = xq2.shape[0]
    N = w.size // ((K // QK_K) * Q6K_BYTES)
    return w, xq2.reshape(-1), N, ncols


def q6k_partials(w, xq, K: int) -> np.ndarray:
    """Exact int32 sub-block dots (ncols, N, K/256, 16)."""
    w, xq, N, ncols = _shape6(w, xq, K)
    P = np.empty(ncols * N * (K // QK_K) * 16, dtype=np.int32)
    lib.orc_q6k_partials(w, xq, P, N, K, ncols)
    return P.reshape(ncols, N, K // QK_K, 16)


def q6k_gemv(w, xq, K: int, nthreads: int = 1) -> np.ndarray:
    """Canonical fp32 Q6_K GEMV, (ncols, N)."""
    w, xq, N, ncols = _shape6(w, xq, K)
    y = np.empty(ncols * N, dtype=np.float32)
    lib.orc_q6k_gemv(w, xq, y, N, K, ncols, nthreads)
    return y.reshape(ncols, N)


def q6k_gemv_slices(w, xq, K: int) -> np.ndarray:
    w, xq, N, ncols = _shape6(w, xq, K)
    v = np.empty(ncols * N * 8, dtype=np.float32)
    lib.orc_q6k_gemv_slices(w, xq, v, N, K, ncols)
    return v.reshape(ncols, N, 8)


def q6k_gemv_f64(w, xq, K: int) -> np.ndarray:
    """The reference's f64 Q6_K oracle (tests/runtime_kernel_test.cu:82-106)."""
    w, xq, N, ncols = _shape6(w, xq, K)
    y = np.empty(ncols * N, dtype=np.float64)
    lib.orc_q6k_gemv_f64(w, xq, y, N, K, ncols)
    return y.reshape(ncols, N)


def q6k_absdot_f64(w, xq, K: int) -> np.ndarray:
    w, xq, N, ncols = _shape6(w, xq, K)
    s = np.empty(ncols * N, dtype=np.float64)
    lib.orc_q6k_absdot_f64(w, xq, s, N, K, ncols)
    return s.reshape(ncols, N)


def dequant_q6k(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    nb = w.size // Q6K_BYTES
    out = np.empty(nb * QK_K, dtype=np.float32)
    lib.orc_dequant_q6k(w, out, nb)
    return out


def dequant_q6k_numpy(w: np.ndarray) -> np.ndarray:
    """Independent vectorised decode of block_q6_K (ggml layout: ql[128],
    qh[64], int8 scales[16], fp16 d), used to cross-check the C decoder."""
    b = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1, Q6K_BYTES)
    ql, qh = b[:, :128].astype(np.int32), b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
    q = np.empty((b.shape[0], 256), dtype=np.int32)
    for half in range(2):
        for group in range(4):
            qlb = ql[:, half * 64 + (group % 2) * 32: half * 64 + (group % 2) * 32 + 32]
            low = (qlb & 15) if group < 2 else (qlb >> 4)
            hi = (qh[:, half * 32: half * 32 + 32] >> (2 * group)) & 3
            q[:, half * 128 + group * 32: half * 128 + group * 32 + 32] = low | (hi << 4)
    scale = (d[:, None] * np.repeat(sc, 16, axis=1)).astype(np.float32)
    return (scale * (q - 32).astype(np.float32)).reshape(-1)


def expf(x: float) -> float:
    return float(lib.orc_expf(x))


def f32_to_f16_bits(f: float) -> int:
    return int(lib.orc_f32_to_f16(f))


def max_threads() -> int:
    return int(lib.orc_max_threads())


# --------------------------------------------- reference kernel family ----
class RefFamily:
    """The reference's own MMVQ family (oracle/_ref/libq4k_ref.so), GPU only."""

    def __init__(self, path: Path = REF_PATH):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        L = C.CDLL(str(path))
        vp = C.c_void_p
        L.ref_launch_candidate.argtypes = [C.c_int, vp, vp, vp, C.c_int, C.c_int, vp]
        L.ref_launch_variant.argtypes = [C.c_int, vp, vp, vp, C.c_int, C.c_int, vp]
        L.ref_quantize_q8_1.argtypes = [vp, vp, C.c_int, vp]
        L.ref_candidate_ids.argtypes = [C.POINTER(C.c_int), C.c_int]
        L.ref_autotuned_candidate.argtypes = [C.c_int, C.c_int, C.c_int]
        self.lib = L

    def candidate_ids(self) -> list[int]:
        buf = (C.c_int * 64)()
        n = self.lib.ref_candidate_ids(buf, 64)
        return list(buf[:n])

    def launch_candidate(self, cid: int, w: int, x: int, y: int, N: int, K: int,
                         stream: int = 0) -> None:
        if self.lib.ref_launch_candidate(cid, w, x, y, N, K, stream) != 0:
            raise ValueError(f"reference launch_q4k_candidate({cid}) threw")

    def quantize(self, x: int, y: int, K: int, stream: int = 0) -> None:
        if self.lib.ref_quantize_q8_1(x, y, K, stream) != 0:
            raise ValueError("reference quantizer threw")

    def autotuned_candidate(self, N: int, K: int, arch: int = 61) -> int:
        return int(self.lib.ref_autotuned_candidate(N, K, arch))


# ------------------------------------------------------------ decode model --
class OrcModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("max_ctx", C.c_int32), ("rope_theta", C.c_float),
                ("eps", C.c_float), ("seed", C.c_uint64), ("centered", C.c_int32),
                ("mix", C.c_int32)]


def _bind_model():
    vp = C.c_void_p
    sig = {
        "orc_model_default_config": (None, [C.POINTER(OrcModelConfig)]),
        "orc_tensor_id": (C.c_uint64, [C.c_int32, C.c_int32]),
        "orc_q6k_layer": (C.c_int32, [C.c_int32, C.c_int32]),
        "orc_rope_table": (None, [_f32p, C.c_int32, C.c_int32, C.c_float]),
        "orc_model_create": (vp, [C.POINTER(OrcModelConfig)]),
        "orc_model_destroy": (None, [vp]),
        "orc_model_step": (C.c_int32, [vp, C.c_int32, C.c_int32, vp, C.c_int32]),
        "orc_model_step_cpu": (C.c_int32, [vp, C.c_int32, C.c_int32, C.c_int32]),
        "orc_model_generate": (None, [vp, vp, C.c_int32, C.c_int32, vp, C.c_int32]),
        "orc_model_hidden": (C.POINTER(C.c_float), [vp]),
        "orc_add_rmsnorm_quantize": (None, [_f32p, vp, _f32p, C.c_float, _u8p, _i64]),
        "orc_qk_norm_rope": (None, [_f32p, _f32p, _f32p, C.c_float, _f32p, C.c_int, C.c_int,
                                    C.c_int, _f32p, vp, vp]),
        "orc_attention_head": (None, [_f32p, vp, vp, C.c_int, C.c_int, C.c_float, _f32p]),
        "orc_argmax": (C.c_int32, [_f32p, _i64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args


_bind_model()


def model_config(**kw) -> OrcModelConfig:
    c = OrcModelConfig()
    lib.orc_model_default_config(C.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def tensor_id(layer: int, which: int) -> int:
    return int(lib.orc_tensor_id(layer, which))


def rope_table(ctx: int, head_dim: int, theta: float) -> np.ndarray:
    out = np.empty(ctx * head_dim, dtype=np.float32)
    lib.orc_rope_table(out, ctx, head_dim, theta)
    return out.reshape(ctx, head_dim // 2, 2)


class OrcModel:
    """CPU evaluation of the seeded Qwen3-4B-shaped model, bit-identical in
    order of operations to abra_b200's decode runtime."""

    def __init__(self, **cfg):
        self.cfg = model_config(**cfg)
        self.ptr = lib.orc_model_create(C.byref(self.cfg))
        self.threads = max_threads()
        self._destroy = lib.orc_model_destroy  # still bound when module globals are gone

    def close(self):
        if self.ptr:
            self._destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()

    def step(self, token: int, pos: int, logits: bool = False):
        out = np.empty(self.cfg.vocab, dtype=np.float32) if logits else None
        tok = lib.orc_model_step(self.ptr, token, pos, out.ctypes.data if logits else None,
                                 self.threads)
        return (tok, out) if logits else tok

    def step_cpu(self, token: int, pos: int) -> int:
        """One decode step on llama.cpp's CPU path (Q8_K activations): the
        timed CPU baseline, not the canonical order."""
        return lib.orc_model_step_cpu(self.ptr, token, pos, self.threads)

    def hidden(self) -> np.ndarray:
        p = lib.orc_model_hidden(self.ptr)
        return np.ctypeslib.as_array(p, shape=(self.cfg.hidden,)).copy()

    def generate(self, prompt, n_gen: int) -> np.ndarray:
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_gen, dtype=np.int32)
        lib.orc_model_generate(self.ptr, pr.ctypes.data, pr.size, n_gen, out.ctypes.data,
                               self.threads)
        return out


def attention_head(q: np.ndarray, K16: np.ndarray, V16: np.ndarray, L: int, scale: float):
    hd = q.size
    out = np.empty(hd, dtype=np.float32)
    lib.orc_attention_head(np.ascontiguousarray(q, dtype=np.float32),
                           np.ascontiguousarray(K16).ctypes.data,
                           np.ascontiguousarray(V16).ctypes.data, L, hd, scale, out)
    return out


def qk_norm_rope(qkv, q_norm, k_norm, eps, cs_row, n_heads, n_kv, hd):
    q = np.empty(n_heads * hd, dtype=np.float32)
    k = np.empty(n_kv * hd, dtype=np.uint16)
    v = np.empty(n_kv * hd, dtype=np.uint16)
    lib.orc_qk_norm_rope(np.ascontiguousarray(qkv, dtype=np.float32),
                         np.ascontiguousarray(q_norm, dtype=np.float32),
                         np.ascontiguousarray(k_norm, dtype=np.float32), eps,
                         np.ascontiguousarray(cs_row, dtype=np.float32).reshape(-1),
                         n_heads, n_kv, hd, q, k.ctypes.data, v.ctypes.data)
    return q, k, v


def argmax(x: np.ndarray) -> int:
    return int(lib.orc_argmax(np.ascontiguousarray(x, dtype=np.float32), x.size))


# --------------------------------------------------- K-shard arithmetic ---
def tree8(v: np.ndarray) -> np.ndarray:
    """The canonical fp32 tree over the last axis (8 slice sums):
    ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7))."""
    v = np.asarray(v, dtype=np.float32)
    a = (v[..., 0] + v[..., 1]) + (v[..., 2] + v[..., 3])
    b = (v[..., 4] + v[..., 5]) + (v[..., 6] + v[..., 7])
    return (a + b).astype(np.float32)


def kshard_partial(slices: np.ndarray, sl_base: int, sl_cnt: int) -> np.ndarray:
    """A K-shard's partial sum as the kernel forms it: its global slices
    [sl_base, sl_base + sl_cnt) at local slices 0, s, 2s, .. (s = 8 / sl_cnt),
    the other local slices +0.0, then the canonical tree."""
    local = np.zeros(slices.shape, dtype=np.float32)
    local[..., ::8 // sl_cnt] = slices[..., sl_base:sl_base + sl_cnt]
    return tree8(local)


def delta_tree(parts) -> np.ndarray:
    """Fixed tree over G partials: 1: p0; 2: p0+p1; 4: (p0+p1)+(p2+p3);
    8: ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7))."""
    p = [np.asarray(x, dtype=np.float32) for x in parts]
    while len(p) > 1:
        p = [(p[i] + p[i + 1]).astype(np.float32) for i in range(0, len(p), 2)]
    return p[0]
