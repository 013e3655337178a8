"""The decode oracle's architecture against an independent implementation.

The oracle (oracle/model_oracle.c) is the bit-exact target of the GPU decode
runtime, so a mistake in its reading of the architecture would pass the GPU
parity tests unnoticed.  Here the same seeded model is built in transformers'
Qwen3 (fp32, eager attention): Q4_K / Q6_K rows dequantized to fp32, the
seeded norm weights, tied embedding/output.  Both are fed the same 270
tokens (past the 256-position attention chunk).

The oracle quantizes activations to Q8_1 and keeps an fp16 KV cache, so the
logits agree to the precision of those formats, not bit for bit: the test
pins the semantics -- RMSNorm, QK-norm before RoPE, the NEOX rotation with
theta 1e6, the GQA grouping (q head h reads kv head h / group), causal
attention, SwiGLU, the residual stream, the final norm and the tied output,
and with the Q4_K_M map the Q6_K attn_v / ffn_down / table.  A negative
control (theta 1e4 in the independent model) shows the measure tells a
wrong rotation apart.  The reference runs this architecture through
llama.cpp, which has no Python form here; transformers is the independent
implementation at hand.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")

N_TOKENS = 270


def _independent_model(cfg: dict, theta: float = 1e6):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    L, H, nh, nkv = cfg["n_layers"], cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"]
    F, V, hd, s = cfg["ffn"], cfg["vocab"], 128, cfg["seed"]
    cen, mix = bool(cfg["centered"]), bool(cfg.get("mix", 0))
    qc = Qwen3Config(vocab_size=V, hidden_size=H, intermediate_size=F, num_hidden_layers=L,
                     num_attention_heads=nh, num_key_value_heads=nkv, head_dim=hd,
                     rope_theta=theta, rms_norm_eps=1e-6, tie_word_embeddings=True,
                     max_position_embeddings=cfg["max_ctx"], attention_bias=False)
    qc._attn_implementation = "eager"
    m = Qwen3ForCausalLM(qc).float().eval()

    def q4(rows, cols, tid, r0=0):
        w = O.gen_q4k(rows, cols, s, tid, r0, centered=cen)
        return torch.from_numpy(O.dequant_q4k(w).reshape(rows, cols))

    def q6(rows, cols, tid, r0=0):
        return torch.from_numpy(O.dequant_q6k(O.gen_q6k(rows, cols, s, tid, r0)).reshape(rows, cols))

    def norm(n, tid):
        return torch.from_numpy(O.gen_norm_f32(n, s, tid))

    qd, kvd = nh * hd, nkv * hd
    with torch.no_grad():
        m.model.embed_tokens.weight.copy_((q6 if mix else q4)(V, H, O.tensor_id(-1, 1)))
        m.model.norm.weight.copy_(norm(H, O.tensor_id(-1, 2)))
        for l, y in enumerate(m.model.layers):
            six = mix and O.lib.orc_q6k_layer(l, L)
            tid = O.tensor_id(l, 1)  # q | k | v rows of one tensor (v in Q6_K on q6 layers)
            wqk = q4(qd + kvd, H, tid)
            wv = q6(kvd, H, tid, qd + kvd) if six else q4(kvd, H, tid, qd + kvd)
            a = y.self_attn
            y.input_layernorm.weight.copy_(norm(H, O.tensor_id(l, 0)))
            a.q_proj.weight.copy_(wqk[:qd])
            a.k_proj.weight.copy_(wqk[qd:])
            a.v_proj.weight.copy_(wv)
            a.q_norm.weight.copy_(norm(hd, O.tensor_id(l, 2)))
            a.k_norm.weight.copy_(norm(hd, O.tensor_id(l, 3)))
            a.o_proj.weight.copy_(q4(H, qd, O.tensor_id(l, 4)))
            y.post_attention_layernorm.weight.copy_(norm(H, O.tensor_id(l, 5)))
            y.mlp.gate_proj.weight.copy_(q4(F, H, O.tensor_id(l, 6)))
            y.mlp.up_proj.weight.copy_(q4(F, H, O.tensor_id(l, 7)))
            y.mlp.down_proj.weight.copy_((q6 if six else q4)(H, F, O.tensor_id(l, 8)))
    assert m.lm_head.weight.data_ptr() == m.model.embed_tokens.weight.data_ptr()
    return m


def _compare(cfg: dict, theta: float = 1e6):
    toks = np.random.default_rng(cfg["seed"] + 1).integers(0, cfg["vocab"], N_TOKENS).astype(np.int32)
    c = O.OrcModel(**cfg)
    ours = np.stack([c.step(int(t), p, logits=True)[1] for p, t in enumerate(toks)])
    c.close()
    with torch.no_grad():
        ref = _independent_model(cfg, theta)(torch.from_numpy(toks.astype(np.int64))[None])
    ref = ref.logits[0].numpy()
    cos = (ours * ref).sum(1) / np.linalg.norm(ours, axis=1) / np.linalg.norm(ref, axis=1)
    top2 = np.sort(ref, axis=1)[:, -2:]
    margin = (top2[:, 1] - top2[:, 0]) / ref.std(axis=1)  # in units of the logits' spread
    return cos, margin, ours.argmax(1) == ref.argmax(1)


CASES = [
    # GQA group 4 (as Qwen3-4B's 32:8), two layers
    (dict(n_layers=2, hidden=512, n_heads=4, n_kv_heads=1, ffn=1024, vocab=2048, max_ctx=300,
          centered=1, seed=3), 0.998),
    # group 2, three layers
    (dict(n_layers=3, hidden=512, n_heads=4, n_kv_heads=2, ffn=768, vocab=1024, max_ctx=300,
          centered=1, seed=5), 0.998),
    # the Q4_K_M map on 8 layers: Q6_K attn_v / ffn_down in layers 0, 3, 7 and a Q6_K table
    (dict(n_layers=8, hidden=256, n_heads=2, n_kv_heads=1, ffn=512, vocab=1024, max_ctx=300,
          centered=1, seed=7, mix=1), 0.98),
]


@pytest.mark.parametrize("cfg,min_cos", CASES, ids=["gqa4", "gqa2", "q4_k_m"])
def test_oracle_model_agrees_with_transformers_qwen3(cfg, min_cos):
    cos, margin, same = _compare(cfg)
    assert cos.min() > min_cos, cos.min()
    assert np.median(cos) > 0.998, np.median(cos)
    # the greedy pick agrees wherever it is not a near tie
    assert same[margin > 0.5].all(), np.flatnonzero(~same & (margin > 0.5))
    assert same.mean() > 0.9


def test_a_wrong_rotation_is_told_apart():
    cos, _, _ = _compare(CASES[0][0], theta=1e4)
    assert cos.min() < 0.95, cos.min()


@pytest.mark.parametrize("mix", [False, True], ids=["q4_k", "q4_k_m"])
def test_gguf_file_read_by_transformers_decodes_like_the_oracle(tmp_path, mix):
    """A GGUF file written by abra_b200.gguf (the seeded tensors under the
    Qwen3 names and metadata) read by transformers' own GGUF loader, which
    dequantizes through the gguf package, gives a model whose logits agree
    with the oracle model of that seed: an independent reader takes our
    names, shapes, types and metadata for the model we mean."""
    gguf_utils = pytest.importorskip("transformers.modeling_gguf_pytorch_utils")
    pytest.importorskip("gguf")
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from gguf_fixture import write_qwen3

    shape = dict(n_layers=8 if mix else 2, hidden=256 if mix else 512, n_heads=2 if mix else 4,
                 n_kv_heads=1 if mix else 2, head_dim=128, ffn=512 if mix else 768, vocab=1024)
    path = tmp_path / "m.gguf"
    write_qwen3(path, shape, seed=5, mix=mix)
    meta = gguf_utils.load_gguf_checkpoint(str(path), return_tensors=False)["config"]
    assert meta["model_type"] == "qwen3" and meta["num_key_value_heads"] == shape["n_kv_heads"]
    qc = Qwen3Config(**{k: v for k, v in meta.items() if k not in ("model_type", "_model_name_or_path")})
    qc._attn_implementation = "eager"
    m = Qwen3ForCausalLM(qc).float().eval()
    tensors = gguf_utils.load_gguf_checkpoint(str(path), return_tensors=True, model_to_load=m)["tensors"]
    res = m.load_state_dict(tensors, strict=False)
    assert not res.unexpected_keys and set(res.missing_keys) <= {"lm_head.weight"}  # tied
    assert m.lm_head.weight.data_ptr() == m.model.embed_tokens.weight.data_ptr()

    cfg = {k: shape[k] for k in ("n_layers", "hidden", "n_heads", "n_kv_heads", "ffn", "vocab")}
    toks = np.random.default_rng(6).integers(0, shape["vocab"], 40).astype(np.int32)
    c = O.OrcModel(**cfg, max_ctx=64, centered=1, seed=5, mix=int(mix))
    ours = np.stack([c.step(int(t), p, logits=True)[1] for p, t in enumerate(toks)])
    c.close()
    with torch.no_grad():
        ref = m(torch.from_numpy(toks.astype(np.int64))[None]).logits[0].numpy()
    cos = (ours * ref).sum(1) / np.linalg.norm(ours, axis=1) / np.linalg.norm(ref, axis=1)
    assert cos.min() > 0.98 and np.median(cos) > 0.998, (cos.min(), np.median(cos))
