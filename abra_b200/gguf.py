"""GGUF v3 files for the decode runtime: read, write, and load into a model.

The reference reads Qwen3-4B-Q4_K_M through llama.cpp. Its own GGUF tooling is
a header parser that lists each tensor's name, ggml type, dimensions and offset
(tools/extract-qwen3-tensor-map.py:15-141), whose output is the census
bench/results/m3/qwen3-q4k-tensor-map.json. This module implements the
published GGUF v3 layout in its own code:

* header: magic "GGUF", version, tensor count, metadata count;
* metadata: key (u64 length + bytes), value type, value (arrays: element
  type, u64 count, elements);
* tensor infos: name, n_dims, dims (ne[0] = innermost), ggml type, offset;
* data: the tensor data, from the next multiple of ``general.alignment``
  (default 32), each offset a multiple of it.

It maps the Qwen3 tensor names onto the model's slots
(``abra_model_load_tensor``).
"""
from __future__ import annotations

import ctypes as C
import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import _lib

MAGIC = b"GGUF"
VERSION = 3
DEFAULT_ALIGNMENT = 32

# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}
_NUMPY = {U8: np.uint8, I8: np.int8, U16: np.uint16, I16: np.int16, U32: np.uint32,
          I32: np.int32, F32: np.float32, BOOL: np.bool_, U64: np.uint64, I64: np.int64,
          F64: np.float64}

# ggml tensor types: (elements per block, bytes per block)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 8, 12, 13, 14
GGML_BLOCKS = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144),
               GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}
GGML_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K",
              GGML_Q5_K: "Q5_K", GGML_Q6_K: "Q6_K"}


class GGUFError(ValueError):
    """Malformed or unsupported GGUF content."""


@dataclass(frozen=True)
class Typed:
    """A metadata value with an explicit GGUF value type (e.g. Typed(U32, 64))."""

    vtype: int
    value: object


def tensor_nbytes(dims, ggml_type: int) -> int:
    if ggml_type not in GGML_BLOCKS:
        raise GGUFError(f"unsupported ggml type {ggml_type}")
    per, size = GGML_BLOCKS[ggml_type]
    n = int(np.prod(dims, dtype=np.int64)) if len(dims) else 1
    if dims and dims[0] % per:
        raise GGUFError(f"row length {dims[0]} is not a multiple of the {per}-element block")
    return n // per * size


@dataclass
class TensorInfo:
    name: str
    dims: tuple  # ne[0] (innermost, the reduction length K of a weight) first
    ggml_type: int
    offset: int  # relative to the data section
    nbytes: int


@dataclass
class GGUFFile:
    """A GGUF file, memory-mapped; tensor data are views into the map."""

    path: Path
    version: int
    metadata: dict
    tensors: dict = field(default_factory=dict)  # name -> TensorInfo, file order
    alignment: int = DEFAULT_ALIGNMENT
    data_offset: int = 0
    _mm: mmap.mmap | None = None

    def data(self, name: str) -> np.ndarray:
        """The raw bytes of a tensor (a read-only view into the map)."""
        t = self.tensors[name]
        start = self.data_offset + t.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.nbytes, offset=start)

    def close(self) -> None:
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:  # a tensor view is still alive: the map closes with it
                pass
            self._mm = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class _Cursor:
    def __init__(self, buf, pos: int = 0):
        self.buf, self.pos = buf, pos

    def take(self, fmt: str):
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.take("<Q")
        if n > len(self.buf) - self.pos:
            raise GGUFError("string runs past the end of the file")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == STRING:
            return self.string()
        if vtype == ARRAY:
            etype, count = self.take("<I"), self.take("<Q")
            if etype in _NUMPY:
                size = np.dtype(_NUMPY[etype]).itemsize
                if count * size > len(self.buf) - self.pos:
                    raise GGUFError("array runs past the end of the file")
                a = np.frombuffer(self.buf, dtype=_NUMPY[etype], count=count, offset=self.pos).copy()
                self.pos += count * size
                return a
            return [self.value(etype) for _ in range(count)]
        raise GGUFError(f"unknown metadata value type {vtype}")


def read_gguf(path) -> GGUFFile:
    """Parse the header, metadata and tensor infos; map the file."""
    path = Path(path)
    if path.stat().st_size < 24:
        raise GGUFError(f"{path}: not a GGUF file")
    f = open(path, "rb")
    try:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    finally:
        f.close()
    try:
        cur = _Cursor(mm)
        if len(mm) < 24 or mm[:4] != MAGIC:
            raise GGUFError(f"{path}: not a GGUF file")
        cur.take("<4s")  # the magic
        version = cur.take("<I")
        if version != VERSION:
            raise GGUFError(f"{path}: GGUF version {version}, expected {VERSION}")
        n_tensors, n_kv = cur.take("<Q"), cur.take("<Q")
        meta = {}
        for _ in range(n_kv):
            key = cur.string()
            meta[key] = cur.value(cur.take("<I"))
        align = int(meta.get("general.alignment", DEFAULT_ALIGNMENT))
        if align <= 0 or align & (align - 1):
            raise GGUFError(f"general.alignment {align} is not a power of two")
        g = GGUFFile(path, version, meta, alignment=align, _mm=mm)
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.take("<I")
            dims = tuple(cur.take("<Q") for _ in range(nd))
            gt, off = cur.take("<I"), cur.take("<Q")
            if off % align:
                raise GGUFError(f"tensor {name}: offset {off} not aligned to {align}")
            nbytes = tensor_nbytes(dims, gt) if gt in GGML_BLOCKS else -1
            g.tensors[name] = TensorInfo(name, dims, gt, off, nbytes)
        g.data_offset = -(-cur.pos // align) * align
        for t in g.tensors.values():
            if t.nbytes >= 0 and g.data_offset + t.offset + t.nbytes > len(mm):
                raise GGUFError(f"tensor {t.name} runs past the end of the file")
        return g
    except Exception:
        mm.close()
        raise


def _put_value(out: bytearray, v, vtype: int | None = None) -> int:
    """Append a metadata value; returns its type.  Python ints become INT64
    (or UINT64 when too large), floats FLOAT32, str STRING, bool BOOL,
    numpy arrays their element type, lists of str an array of STRING."""
    if vtype is None:
        if isinstance(v, bool):
            vtype = BOOL
        elif isinstance(v, (int, np.integer)):
            vtype = I64 if -(1 << 63) <= int(v) < (1 << 63) else U64
        elif isinstance(v, (float, np.floating)):
            vtype = F32
        elif isinstance(v, str):
            vtype = STRING
        elif isinstance(v, (np.ndarray, list, tuple)):
            vtype = ARRAY
        else:
            raise GGUFError(f"cannot store {type(v).__name__} in GGUF metadata")
    if vtype in _SCALAR:
        out += struct.pack(_SCALAR[vtype], v)
    elif vtype == STRING:
        b = v.encode("utf-8")
        out += struct.pack("<Q", len(b)) + b
    elif vtype == ARRAY:
        if isinstance(v, np.ndarray):
            et = {np.dtype(t): k for k, t in _NUMPY.items()}[v.dtype]
            out += struct.pack("<IQ", et, v.size) + np.ascontiguousarray(v).tobytes()
        else:
            items = list(v)
            et = STRING if all(isinstance(x, str) for x in items) else I64
            out += struct.pack("<IQ", et, len(items))
            for x in items:
                _put_value(out, x, et)
    else:
        raise GGUFError(f"unknown metadata value type {vtype}")
    return vtype


def write_gguf(path, metadata: dict, tensors, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Write a GGUF v3 file.  metadata: key -> value (or Typed(vtype, value)
    to force a type); tensors: (name, dims, ggml_type, uint8 data)."""
    meta = dict(metadata)
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = Typed(U32, alignment)
    head = bytearray(MAGIC + struct.pack("<IQQ", VERSION, len(tensors), len(meta)))
    for k, v in meta.items():
        kb = k.encode("utf-8")
        head += struct.pack("<Q", len(kb)) + kb
        slot = len(head)
        head += b"\0\0\0\0"  # the value type, known once the value is written
        vt = _put_value(head, v.value, v.vtype) if isinstance(v, Typed) else _put_value(head, v)
        struct.pack_into("<I", head, slot, vt)
    offs, off = [], 0
    for name, dims, gt, data in tensors:
        if np.asarray(data).nbytes != tensor_nbytes(dims, gt):
            raise GGUFError(f"tensor {name}: {np.asarray(data).nbytes} bytes for dims {dims}")
        nb = name.encode("utf-8")
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", gt, off)
        offs.append(off)
        off = -(-(off + tensor_nbytes(dims, gt)) // alignment) * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (-len(head) % alignment))
        base = f.tell()
        for (name, dims, gt, data), o in zip(tensors, offs):
            f.seek(base + o)
            f.write(np.ascontiguousarray(data).view(np.uint8).tobytes())
        f.seek(base + off)
        f.truncate()


# ----------------------------------------------------------------- Qwen3 ---
# GGUF names of the Qwen3 tensors (llama.cpp's naming, as in the census) and
# the model's load slots (ABRA_TENSOR_* in include/abra_b200.h).
GLOBAL_SLOTS = {"token_embd.weight": (-1, 1), "output_norm.weight": (-1, 2)}
LAYER_SLOTS = {"attn_norm": 0, "attn_q": 1, "attn_q_norm": 2, "attn_k_norm": 3,
               "attn_output": 4, "ffn_norm": 5, "ffn_gate": 6, "ffn_up": 7, "ffn_down": 8,
               "attn_k": 9, "attn_v": 10}


def slot_of(name: str):
    """(layer, slot) of a Qwen3 tensor name, or None."""
    if name in GLOBAL_SLOTS:
        return GLOBAL_SLOTS[name]
    parts = name.split(".")
    if len(parts) == 4 and parts[0] == "blk" and parts[3] == "weight" and parts[2] in LAYER_SLOTS:
        try:
            return int(parts[1]), LAYER_SLOTS[parts[2]]
        except ValueError:
            return None
    return None


def model_config(g: GGUFFile) -> dict:
    """abra_model_config fields from the GGUF metadata (architecture qwen3)."""
    arch = g.metadata.get("general.architecture")
    if arch != "qwen3":
        raise GGUFError(f"architecture {arch!r} is not qwen3")
    m = g.metadata

    def need(key):
        if f"{arch}.{key}" not in m:
            raise GGUFError(f"missing metadata {arch}.{key}")
        return m[f"{arch}.{key}"]

    if "output.weight" in g.tensors:
        raise GGUFError("untied output.weight: the runtime decodes a tied embedding/output")
    emb = g.tensors.get("token_embd.weight")
    if emb is None:
        raise GGUFError("missing token_embd.weight")
    hidden, heads = int(need("embedding_length")), int(need("attention.head_count"))
    cfg = {"n_layers": int(need("block_count")), "hidden": hidden, "n_heads": heads,
           "n_kv_heads": int(need("attention.head_count_kv")),
           "head_dim": int(m.get(f"{arch}.attention.key_length", hidden // heads)),
           "ffn": int(need("feed_forward_length")), "vocab": int(emb.dims[1]),
           "rope_theta": float(need("rope.freq_base")),
           "eps": float(need("attention.layer_norm_rms_epsilon"))}
    if emb.dims[0] != hidden:
        raise GGUFError(f"token_embd.weight is {emb.dims}, hidden is {hidden}")
    return cfg


def type_flags(g: GGUFFile, n_layers: int) -> int:
    """ABRA_MODEL_Q4_K_M when the file follows the Q4_K_M type map, 0 when
    every linear weight is Q4_K; otherwise GGUFError (no other mix is built)."""
    from .model import Q4_K_M, q6k_layers

    q6 = set(q6k_layers(n_layers))
    want = {0: {}, Q4_K_M: {}}
    for name, t in g.tensors.items():
        s = slot_of(name)
        if s is None or t.ggml_type == GGML_F32:
            continue
        layer, slot = s
        mix6 = (layer == -1) or (slot in (8, 10) and layer in q6)
        want[0][name] = GGML_Q4_K
        want[Q4_K_M][name] = GGML_Q6_K if mix6 else GGML_Q4_K
    for flags in (0, Q4_K_M):
        if all(g.tensors[n].ggml_type == t for n, t in want[flags].items()):
            return flags
    found = {}
    for n, t in g.tensors.items():
        found.setdefault(GGML_NAMES.get(t.ggml_type, str(t.ggml_type)), 0)
        found[GGML_NAMES.get(t.ggml_type, str(t.ggml_type))] += 1
    raise GGUFError(f"tensor types {found} follow neither all-Q4_K nor the Q4_K_M map")


def load_into(model, g: GGUFFile) -> int:
    """Copy every Qwen3 tensor of the file into a created DecodeModel;
    returns the number of tensors loaded (all slots must be present)."""
    cfg = model.cfg
    expected = {(-1, 1), (-1, 2)} | {(l, s) for l in range(cfg.n_layers) for s in LAYER_SLOTS.values()}
    seen = set()
    for name, t in g.tensors.items():
        s = slot_of(name)
        if s is None:
            continue
        if s not in expected:
            raise GGUFError(f"tensor {name} has no slot in a {cfg.n_layers}-layer model")
        data = g.data(name)
        rc = _lib.lib.abra_model_load_tensor(model.handle, s[0], s[1], t.ggml_type,
                                             data.ctypes.data_as(C.c_void_p), data.nbytes)
        if rc != _lib.ABRA_OK:
            msg = _lib.lib.abra_model_last_error()
            raise GGUFError(f"{name}: {msg.decode() if msg else rc}")
        seen.add(s)
    missing = expected - seen
    if missing:
        raise GGUFError(f"{len(missing)} tensors missing, e.g. (layer, slot) {sorted(missing)[:4]}")
    return len(seen)
