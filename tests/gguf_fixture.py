"""Test helper: a Qwen3 GGUF file holding exactly the seeded tensors of the
synthetic model (the generators of the oracle, with the runtime's tensor ids
and row offsets), so a model loaded from it must decode like the oracle
model of that seed."""
from __future__ import annotations

import numpy as np

import oracle as O
from abra_b200 import gguf as G


def qwen3_tensors(n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, seed, centered=1,
                  mix=False):
    from abra_b200.model import q6k_layers

    qd, kvd = n_heads * head_dim, n_kv_heads * head_dim
    tid = O.tensor_id
    q6 = set(q6k_layers(n_layers)) if mix else set()

    def q4(rows, cols, t, row0=0):
        return (cols, rows), G.GGML_Q4_K, O.gen_q4k(rows, cols, seed, t, row_offset=row0,
                                                      centered=bool(centered)).reshape(-1)

    def q6w(rows, cols, t, row0=0):
        return (cols, rows), G.GGML_Q6_K, O.gen_q6k(rows, cols, seed, t, row_offset=row0).reshape(-1)

    def f32(n, t):
        return (n,), G.GGML_F32, O.gen_norm_f32(n, seed, t).view(np.uint8)

    out = [("token_embd.weight", *(q6w if mix else q4)(vocab, hidden, tid(-1, 1))),
           ("output_norm.weight", *f32(hidden, tid(-1, 2)))]
    for l in range(n_layers):
        b = f"blk.{l}."
        out += [(b + "attn_norm.weight", *f32(hidden, tid(l, 0))),
                (b + "attn_q.weight", *q4(qd, hidden, tid(l, 1))),
                (b + "attn_k.weight", *q4(kvd, hidden, tid(l, 1), qd)),
                (b + "attn_v.weight", *(q6w if l in q6 else q4)(kvd, hidden, tid(l, 1), qd + kvd)),
                (b + "attn_q_norm.weight", *f32(head_dim, tid(l, 2))),
                (b + "attn_k_norm.weight", *f32(head_dim, tid(l, 3))),
                (b + "attn_output.weight", *q4(hidden, qd, tid(l, 4))),
                (b + "ffn_norm.weight", *f32(hidden, tid(l, 5))),
                (b + "ffn_gate.weight", *q4(ffn, hidden, tid(l, 6))),
                (b + "ffn_up.weight", *q4(ffn, hidden, tid(l, 7))),
                (b + "ffn_down.weight", *(q6w if l in q6 else q4)(hidden, ffn, tid(l, 8)))]
    return out


def qwen3_metadata(n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab,
                   rope_theta=1000000.0, eps=1e-6):
    return {
        "general.architecture": "qwen3",
        "general.name": "synthetic qwen3",
        "qwen3.block_count": G.Typed(G.U32, n_layers),
        "qwen3.context_length": G.Typed(G.U32, 40960),
        "qwen3.embedding_length": G.Typed(G.U32, hidden),
        "qwen3.feed_forward_length": G.Typed(G.U32, ffn),
        "qwen3.attention.head_count": G.Typed(G.U32, n_heads),
        "qwen3.attention.head_count_kv": G.Typed(G.U32, n_kv_heads),
        "qwen3.attention.key_length": G.Typed(G.U32, head_dim),
        "qwen3.attention.value_length": G.Typed(G.U32, head_dim),
        "qwen3.rope.freq_base": G.Typed(G.F32, rope_theta),
        "qwen3.attention.layer_norm_rms_epsilon": G.Typed(G.F32, eps),
        "tokenizer.ggml.model": "gpt2",
        "tokenizer.ggml.tokens": [f"tok{i}" for i in range(vocab)],
        "tokenizer.ggml.token_type": np.ones(vocab, dtype=np.int32),
    }


def write_qwen3(path, cfg: dict, seed: int, mix: bool = False, centered: int = 1, alignment=32):
    shape = {k: cfg[k] for k in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn",
                                 "vocab")}
    G.write_gguf(path, qwen3_metadata(**shape),
                 qwen3_tensors(**shape, seed=seed, centered=centered, mix=mix), alignment=alignment)
