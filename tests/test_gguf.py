"""CPU tests of the GGUF v3 reader/writer and the Qwen3 mapping
(abra_b200/gguf.py): metadata of every value type, tensor data and
alignment round-trip; the model shape and the Q4_K / Q4_K_M type map are
read from the header; malformed files are refused."""
from __future__ import annotations

import struct

import numpy as np
import pytest

from abra_b200 import gguf as G
from gguf_fixture import qwen3_metadata, write_qwen3

SMALL = dict(n_layers=9, hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, vocab=300)


@pytest.mark.parametrize("alignment", [32, 64])
def test_round_trip_metadata_and_tensors(tmp_path, alignment):
    rng = np.random.default_rng(0)
    meta = {"a.u8": G.Typed(G.U8, 7), "a.i8": G.Typed(G.I8, -7), "a.u16": G.Typed(G.U16, 65535),
            "a.i16": G.Typed(G.I16, -300), "a.u32": G.Typed(G.U32, 1 << 31), "a.i32": G.Typed(G.I32, -5),
            "a.f32": G.Typed(G.F32, 0.5), "a.bool": True, "a.str": "héllo", "a.u64": 1 << 63,
            "a.i64": -(1 << 40), "a.f64": G.Typed(G.F64, 1e-300),
            "a.arr_i32": np.arange(5, dtype=np.int32), "a.arr_f32": np.linspace(0, 1, 3, dtype=np.float32),
            "a.arr_str": ["x", "", "yz"]}
    tensors = [("t.f32", (7,), G.GGML_F32, rng.standard_normal(7).astype(np.float32).view(np.uint8)),
               ("t.q4k", (512, 3), G.GGML_Q4_K, rng.integers(0, 256, 3 * 2 * 144, dtype=np.uint8)),
               ("t.q6k", (256, 5), G.GGML_Q6_K, rng.integers(0, 256, 5 * 210, dtype=np.uint8))]
    p = tmp_path / "x.gguf"
    G.write_gguf(p, meta, tensors, alignment=alignment)
    with G.read_gguf(p) as g:
        assert g.version == 3 and g.alignment == alignment and g.data_offset % alignment == 0
        assert g.metadata["a.u8"] == 7 and g.metadata["a.i8"] == -7 and g.metadata["a.u16"] == 65535
        assert g.metadata["a.u32"] == 1 << 31 and g.metadata["a.bool"] is True
        assert g.metadata["a.str"] == "héllo" and g.metadata["a.u64"] == 1 << 63
        assert g.metadata["a.i64"] == -(1 << 40) and g.metadata["a.f64"] == 1e-300
        assert g.metadata["a.f32"] == 0.5 and g.metadata["a.arr_str"] == ["x", "", "yz"]
        assert np.array_equal(g.metadata["a.arr_i32"], np.arange(5))
        assert list(g.tensors) == ["t.f32", "t.q4k", "t.q6k"]
        for name, dims, gt, data in tensors:
            t = g.tensors[name]
            assert t.dims == dims and t.ggml_type == gt and t.offset % alignment == 0
            assert np.array_equal(g.data(name), data)


def test_qwen3_shape_and_type_map_from_header(tmp_path):
    from abra_b200.model import Q4_K_M

    for mix, want in ((False, 0), (True, Q4_K_M)):
        p = tmp_path / f"m{int(mix)}.gguf"
        write_qwen3(p, SMALL, seed=1, mix=mix)
        with G.read_gguf(p) as g:
            cfg = G.model_config(g)
            assert {k: cfg[k] for k in SMALL} == SMALL
            assert cfg["rope_theta"] == 1e6 and abs(cfg["eps"] - 1e-6) < 1e-12
            assert G.type_flags(g, SMALL["n_layers"]) == want
            assert len(g.metadata["tokenizer.ggml.tokens"]) == SMALL["vocab"]
            assert sum(G.slot_of(n) is not None for n in g.tensors) == 2 + 11 * SMALL["n_layers"]


def test_other_type_mixes_and_untied_output_refused(tmp_path):
    from gguf_fixture import qwen3_tensors

    shape = {k: SMALL[k] for k in SMALL}
    t = qwen3_tensors(**shape, seed=1, mix=True)
    # one Q6_K ffn_down moved to a layer the Q4_K_M map keeps Q4_K
    t = [(n, d, G.GGML_Q6_K, np.zeros(d[1] * d[0] // 256 * 210, np.uint8)) if n == "blk.1.ffn_down.weight"
         else (n, d, gt, x) for n, d, gt, x in t]
    p = tmp_path / "bad.gguf"
    G.write_gguf(p, qwen3_metadata(**shape), t)
    with G.read_gguf(p) as g, pytest.raises(G.GGUFError, match="Q4_K_M"):
        G.type_flags(g, SMALL["n_layers"])
    t2 = qwen3_tensors(**shape, seed=1) + [("output.weight", (512, 300), G.GGML_Q4_K,
                                            np.zeros(300 * 2 * 144, np.uint8))]
    G.write_gguf(p, qwen3_metadata(**shape), t2)
    with G.read_gguf(p) as g, pytest.raises(G.GGUFError, match="untied"):
        G.model_config(g)


def test_slot_names():
    assert G.slot_of("token_embd.weight") == (-1, 1)
    assert G.slot_of("output_norm.weight") == (-1, 2)
    assert G.slot_of("blk.35.ffn_down.weight") == (35, 8)
    assert G.slot_of("blk.0.attn_v.weight") == (0, 10)
    assert G.slot_of("blk.x.attn_v.weight") is None and G.slot_of("blk.0.attn_v.bias") is None


def test_malformed_files_refused(tmp_path):
    p = tmp_path / "m.gguf"
    p.write_bytes(b"")
    with pytest.raises(G.GGUFError, match="not a GGUF"):
        G.read_gguf(p)
    p.write_bytes(b"GGML" + b"\0" * 40)
    with pytest.raises(G.GGUFError, match="not a GGUF"):
        G.read_gguf(p)
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 2, 0, 0))
    with pytest.raises(G.GGUFError, match="version"):
        G.read_gguf(p)
    G.write_gguf(p, {}, [("t", (256, 4), G.GGML_Q4_K, np.zeros(4 * 144, np.uint8))])
    p.write_bytes(p.read_bytes()[:-100])  # truncated data
    with pytest.raises(G.GGUFError, match="past the end"):
        G.read_gguf(p)
    with pytest.raises(G.GGUFError):
        G.write_gguf(p, {}, [("t", (256, 4), G.GGML_Q4_K, np.zeros(10, np.uint8))])


def test_load_tensor_refuses_without_a_model():
    from abra_b200 import _lib

    assert _lib.lib.abra_model_load_tensor(None, -1, 1, 12, 16, 144) == _lib.ABRA_E_INVALID


def test_close_with_a_live_tensor_view(tmp_path):
    p = tmp_path / "v.gguf"
    G.write_gguf(p, {}, [("t", (256, 1), G.GGML_Q4_K, np.arange(144, dtype=np.uint8))])
    g = G.read_gguf(p)
    view = g.data("t")
    g.close()  # does not raise while `view` is alive
    assert view[5] == 5


def test_from_gguf_refuses_before_creating_a_model(tmp_path):
    """An unsupported file is refused while reading the header: no model (and
    no CUDA call) is made."""
    from abra_b200.model import DecodeModel
    from gguf_fixture import qwen3_tensors

    shape = {k: SMALL[k] for k in SMALL}
    t = qwen3_tensors(**shape, seed=1) + [("output.weight", (512, 300), G.GGML_Q4_K,
                                           np.zeros(300 * 2 * 144, np.uint8))]
    p = tmp_path / "untied.gguf"
    G.write_gguf(p, qwen3_metadata(**shape), t)
    with pytest.raises(G.GGUFError, match="untied"):
        DecodeModel.from_gguf(p)
    meta = qwen3_metadata(**shape)
    meta["general.architecture"] = "llama"
    G.write_gguf(p, meta, qwen3_tensors(**shape, seed=1))
    with pytest.raises(G.GGUFError, match="qwen3"):
        DecodeModel.from_gguf(p)
