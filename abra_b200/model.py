"""Qwen3-4B-shaped Q4_K decode on B200: one GPU, or tensor parallel over 2/4/8.

Thin host wrapper of the native runtime in libabra_b200 (abra_model_* in
include/abra_b200.h): weights are generated on the device from a seed, the
decode step is one CUDA graph replayed per token, and prompt feeding and
greedy generation never leave the device.  The reference runs the same
architecture through llama.cpp (tools/qwen3-4b.py, tests/runtime_logits.cpp).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("max_ctx", C.c_int32), ("rope_theta", C.c_float),
                ("eps", C.c_float), ("seed", C.c_uint64), ("centered", C.c_int32),
                ("flags", C.c_int32)]


class TpShard(C.Structure):
    """What one rank of a tensor-parallel group holds (abra_tp_shard)."""
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("q_head_lo", C.c_int32),
                ("q_heads", C.c_int32), ("kv_head_lo", C.c_int32), ("kv_heads", C.c_int32),
                ("ffn_lo", C.c_int32), ("ffn_hi", C.c_int32), ("sl_base", C.c_int32),
                ("sl_cnt", C.c_int32), ("vocab_lo", C.c_int64), ("vocab_hi", C.c_int64)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


EAGER = 1   # ABRA_MODEL_EAGER
NO_PDL = 2  # ABRA_MODEL_NO_PDL
NO_PREFETCH = 4  # ABRA_MODEL_NO_PREFETCH
Q4_K_M = 8  # ABRA_MODEL_Q4_K_M: the real Qwen3-4B-Q4_K_M type map (Q6_K attn_v/ffn_down/output)
KERNEL_CHAIN = 16  # ABRA_MODEL_KERNEL_CHAIN: per-operation kernels instead of the persistent step


def persist_plan(sms: int = 148, **config) -> dict:
    """Host-only check of the persistent decode kernel's plan for a model
    shape (abra_persist_plan): every weight copy of every CTA checked against
    its ring slot and its tensor.  Raises AbraError when the shape does not
    fit the kernel."""
    c = default_config(**config)
    out = np.zeros(9, dtype=np.int64)
    _check(_lib.lib.abra_persist_plan(C.byref(c), sms, out.ctypes.data), "abra_persist_plan")
    keys = ("smem", "ring_bytes", "units_max", "copies", "rows_qkv", "rows_o", "rows_gate_up",
            "rows_down", "rows_output")
    return dict(zip(keys, (int(v) for v in out)))


def lookup_draft(history, key: int, limit: int) -> np.ndarray:
    """Prompt-lookup draft of the native loop (abra_lookup_draft): the
    tokens after the most recent earlier occurrence of the last ``key``."""
    h = np.ascontiguousarray(history, dtype=np.int32)
    out = np.empty(max(limit, 1), dtype=np.int32)
    n = _lib.lib.abra_lookup_draft(h.ctypes.data if h.size else None, h.size, key, limit,
                                   out.ctypes.data)
    if n < 0:
        raise ValueError("abra_lookup_draft: bad arguments")
    return out[:n]


def q6k_layers(n_layers: int) -> list[int]:
    """Layers whose attn_v and ffn_down are Q6_K under the Q4_K_M type map
    (llama.cpp's use_more_bits: l < n/8, l >= 7n/8 or (l - n/8) % 3 == 2)."""
    a, b = n_layers // 8, 7 * n_layers // 8
    return [l for l in range(n_layers) if l < a or l >= b or (l - a) % 3 == 2]


IPC_HANDLE_BYTES = 64


def exchange_handles(mine: bytes, world: int, group=None) -> bytes:
    """All ranks' fixed-size handles, concatenated in rank order (one
    all_gather over the torch.distributed group)."""
    import torch.distributed as dist

    if len(mine) != IPC_HANDLE_BYTES:
        raise ValueError(f"handle must be {IPC_HANDLE_BYTES} bytes")
    handles = [None] * world
    dist.all_gather_object(handles, mine, group=group)
    if any(not isinstance(h, bytes) or len(h) != IPC_HANDLE_BYTES for h in handles):
        raise RuntimeError("a rank sent a malformed arena handle")
    return b"".join(handles)


def shard_info(rank: int, world: int, **config) -> TpShard:
    """The split rank `rank` of `world` would hold (no GPU needed)."""
    c = default_config(**config)
    s = TpShard()
    _check(_lib.lib.abra_tp_shard_info(C.byref(c), rank, world, C.byref(s)), "abra_tp_shard_info")
    return s


def default_config(**overrides) -> ModelConfig:
    c = ModelConfig()
    _lib.lib.abra_model_default_config(C.byref(c))
    for k, v in overrides.items():
        setattr(c, k, v)
    return c


def _check(rc: int, what: str) -> None:
    if rc != _lib.ABRA_OK:
        msg = _lib.lib.abra_model_last_error()
        raise _lib.AbraError(rc, what, msg.decode() if msg else "")


class BatchedDecodeModel:
    """32 sequences decoded in lockstep at one shared position, every GEMV on
    the tcgen05 tensor cores (abra_model_create_batched); per sequence the
    logits and tokens equal the batch-1 model's bit for bit.  With world > 1
    this process holds rank ``rank`` of the tensor-parallel split
    (abra_model_create_batched_tp; handles exchanged as for DecodeModel), and
    ``logits()`` returns this rank's vocab rows."""

    def __init__(self, batch: int = 32, rank: int = 0, world: int = 1, group=None, **config):
        self.handle = None
        self.batch = batch
        self.cfg = default_config(**config)
        self.shard = shard_info(rank, world, **config)
        self._destroy = _lib.lib.abra_model_destroy  # still bound at interpreter exit
        h = C.c_void_p()
        if world > 1:
            _check(_lib.lib.abra_model_create_batched_tp(C.byref(self.cfg), batch, rank, world, C.byref(h)),
                   "abra_model_create_batched_tp")
        else:
            _check(_lib.lib.abra_model_create_batched(C.byref(self.cfg), batch, C.byref(h)),
                   "abra_model_create_batched")
        self.handle = h
        if world > 1:
            DecodeModel._connect(self, group)

    def close(self) -> None:
        if self.handle:
            self._destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def reset(self, prompts) -> None:
        """prompts: (batch, n_prompt) token ids."""
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        if p.ndim != 2 or p.shape[0] != self.batch:
            raise ValueError(f"prompts must be ({self.batch}, n_prompt)")
        _check(_lib.lib.abra_model_reset_batched(self.handle, p.ctypes.data, p.shape[1]),
               "abra_model_reset_batched")

    def step(self, n: int = 1) -> None:
        _check(_lib.lib.abra_model_step(self.handle, n), "abra_model_step")

    def sync(self) -> None:
        _check(_lib.lib.abra_model_sync(self.handle), "abra_model_sync")

    def tokens(self, n: int) -> np.ndarray:
        out = np.empty((self.batch, n), dtype=np.int32)
        _check(_lib.lib.abra_model_read_batched(self.handle, out.ctypes.data, n, None),
               "abra_model_read_batched")
        return out

    def logits(self) -> np.ndarray:
        out = np.empty((self.batch, int(self.shard.vocab_hi - self.shard.vocab_lo)), dtype=np.float32)
        _check(_lib.lib.abra_model_read_batched(self.handle, None, 0, out.ctypes.data),
               "abra_model_read_batched")
        return out

    @property
    def stream(self) -> int:
        st, wb, kb = C.c_void_p(), C.c_uint64(), C.c_uint64()
        _check(_lib.lib.abra_model_info(self.handle, C.byref(st), C.byref(wb), C.byref(kb)),
               "abra_model_info")
        return st.value or 0


class DecodeModel:
    """A seeded Qwen3-4B-shaped model resident on the current CUDA device.

    With ``world > 1`` this process holds rank ``rank`` of a tensor-parallel
    group (one process per GPU): the ranks exchange their arenas' IPC handles
    through ``torch.distributed`` (``group``, default the world group) and
    from then on talk only over NVLink, inside the decode graph.  Every rank
    must make the same calls in the same order.
    """

    @classmethod
    def from_gguf(cls, path, rank: int = 0, world: int = 1, group=None, max_ctx: int = 4096,
                  flags: int = 0) -> "DecodeModel":
        """A model whose shape, type map and weights come from a Qwen3 GGUF
        file (abra_b200.gguf): created seeded, then every tensor copied in."""
        from . import gguf

        with gguf.read_gguf(path) as g:
            cfg = gguf.model_config(g)
            tflags = gguf.type_flags(g, cfg["n_layers"])
            m = cls(rank=rank, world=world, group=group, max_ctx=max_ctx,
                    flags=flags | tflags, **cfg)
            try:
                gguf.load_into(m, g)
            except Exception:
                m.close()
                raise
        return m

    def __init__(self, rank: int = 0, world: int = 1, group=None, **config):
        self.handle = None
        self.cfg = default_config(**config)
        self.shard = shard_info(rank, world, **config)
        self._destroy = _lib.lib.abra_model_destroy  # still bound at interpreter exit
        h = C.c_void_p()
        _check(_lib.lib.abra_model_create_tp(C.byref(self.cfg), rank, world, C.byref(h)),
               "abra_model_create_tp")
        self.handle = h
        if world > 1:
            self._connect(group)

    def _connect(self, group) -> None:
        mine = C.create_string_buffer(IPC_HANDLE_BYTES)
        _check(_lib.lib.abra_model_tp_handle(self.handle, mine, IPC_HANDLE_BYTES),
               "abra_model_tp_handle")
        allh = exchange_handles(bytes(mine.raw), self.shard.world, group)
        buf = C.create_string_buffer(allh, len(allh))
        _check(_lib.lib.abra_model_tp_connect(self.handle, buf, IPC_HANDLE_BYTES),
               "abra_model_tp_connect")
        import torch.distributed as dist

        dist.barrier(group=group)  # every rank mapped its peers and recorded its step

    @property
    def persistent(self) -> bool:
        """True when each decode step is one launch of the persistent decode
        kernel (abra_model_path), False for the per-operation kernel chain."""
        v = C.c_int32()
        _check(_lib.lib.abra_model_path(self.handle, C.byref(v)), "abra_model_path")
        return bool(v.value)

    def close(self) -> None:
        if self.handle:
            self._destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- state ------------------------------------------------------------
    def reset(self, prompt) -> None:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        _check(_lib.lib.abra_model_reset(self.handle, p.ctypes.data, p.size), "abra_model_reset")

    def step(self, n: int = 1) -> None:
        """Queue n decode steps on the model's stream (asynchronous)."""
        _check(_lib.lib.abra_model_step(self.handle, n), "abra_model_step")

    def prefill(self, n: int) -> None:
        """Process the next n prompt tokens (a multiple of 32) as tensor-core
        GEMV columns, chunks of up to 256 (asynchronous): the KV cache ends
        up as after n decode steps; the last prompt token is left to step()."""
        _check(_lib.lib.abra_model_prefill(self.handle, n), "abra_model_prefill")

    def feed_prompt(self, prompt) -> None:
        """reset(prompt), then prefill every whole 32-token tile of the
        first len(prompt) - 1 tokens (models the prefill supports) and step
        through the rest; afterwards the model has picked the first generated
        token."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        self.reset(p)
        # the tensor-core prefill covers one-GPU all-Q4_K models; the rest step
        can = self.shard.world == 1 and not (self.cfg.flags & Q4_K_M)
        n = (p.size - 1) // 32 * 32 if can else 0
        if n:
            self.prefill(n)
        self.step(p.size - n)

    def verify(self, draft) -> tuple[int, np.ndarray]:
        """Prompt-lookup verification of up to 31 draft tokens after the
        current token (abra_model_verify): (kept, the greedy picks)."""
        d = np.ascontiguousarray(draft, dtype=np.int32)
        picks = np.empty(d.size + 1, dtype=np.int32)
        kept = C.c_int32()
        _check(_lib.lib.abra_model_verify(self.handle, d.ctypes.data if d.size else None, d.size,
                                          picks.ctypes.data, C.byref(kept)), "abra_model_verify")
        return kept.value, picks

    def generate_lookup(self, prompt, n_gen: int, key: int = 2, draft_max: int = 16):
        """Greedy generation with prompt-lookup speculation (the reference's
        lookup_decode loop): the same tokens as generate(), plus the stats
        {proposed, accepted, blocks}."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_gen, dtype=np.int32)
        st = np.zeros(3, dtype=np.int32)
        _check(_lib.lib.abra_model_generate_lookup(self.handle, p.ctypes.data, p.size, n_gen, key,
                                                   draft_max, out.ctypes.data, st.ctypes.data),
               "abra_model_generate_lookup")
        return out, {"proposed": int(st[0]), "accepted": int(st[1]), "blocks": int(st[2])}

    def invalidate(self) -> None:
        """Drop the recorded step; the next step records it again (picks up
        tuning-table changes)."""
        _check(_lib.lib.abra_model_invalidate(self.handle), "abra_model_invalidate")

    def sync(self) -> None:
        _check(_lib.lib.abra_model_sync(self.handle), "abra_model_sync")

    def tokens(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.int32)
        _check(_lib.lib.abra_model_read(self.handle, out.ctypes.data, n, None, None), "abra_model_read")
        return out

    def logits(self) -> np.ndarray:
        """The last step's logits of this rank's vocab rows [vocab_lo, vocab_hi)."""
        out = np.empty(self.shard.vocab_hi - self.shard.vocab_lo, dtype=np.float32)
        _check(_lib.lib.abra_model_read(self.handle, None, 0, out.ctypes.data, None), "abra_model_read")
        return out

    def position(self) -> int:
        p = C.c_int32()
        _check(_lib.lib.abra_model_read(self.handle, None, 0, None, C.byref(p)), "abra_model_read")
        return p.value

    def generate(self, prompt, n_gen: int) -> np.ndarray:
        """Greedy: feed the prompt, return the n_gen picked token ids."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_gen, dtype=np.int32)
        _check(_lib.lib.abra_model_generate(self.handle, p.ctypes.data, p.size, n_gen,
                                            out.ctypes.data), "abra_model_generate")
        return out

    def decode_streaming(self, n: int) -> np.ndarray:
        """Serving loop: one token at a time with a host round trip each."""
        out = np.empty(n, dtype=np.int32)
        _check(_lib.lib.abra_model_decode_streaming(self.handle, n, out.ctypes.data),
               "abra_model_decode_streaming")
        return out

    def info(self) -> dict:
        st, wb, kb = C.c_void_p(), C.c_uint64(), C.c_uint64()
        _check(_lib.lib.abra_model_info(self.handle, C.byref(st), C.byref(wb), C.byref(kb)),
               "abra_model_info")
        return {"stream": st.value or 0, "weight_bytes": wb.value, "kv_bytes": kb.value}

    @property
    def stream(self) -> int:
        return self.info()["stream"]
