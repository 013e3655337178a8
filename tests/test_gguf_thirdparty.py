"""Cross-checks against the third-party `gguf` package (llama.cpp's own Python
tooling, installed in this image; not part of the reference): its decoders of
ggml's Q4_K and Q6_K blocks against the oracle's, and its GGUF reader/writer
against abra_b200.gguf, in both directions.  Skipped where it is absent."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from abra_b200 import gguf as G

gguf = pytest.importorskip("gguf")


@pytest.mark.parametrize("qtype,gen,deq,nbytes", [
    ("Q4_K", lambda: O.gen_q4k(37, 768, 3, 81), O.dequant_q4k, 144),
    ("Q4_K", lambda: O.gen_q4k(37, 768, 3, 82, centered=True), O.dequant_q4k, 144),
    ("Q6_K", lambda: O.gen_q6k(37, 768, 3, 83), O.dequant_q6k, 210),
])
def test_block_decoders_agree(qtype, gen, deq, nbytes):
    """The oracle's reading of the block layouts equals the gguf package's,
    value for value."""
    w = gen().reshape(-1, nbytes)
    ours = deq(w)
    theirs = gguf.quants.dequantize(w, getattr(gguf.GGMLQuantizationType, qtype)).reshape(-1)
    assert ours.shape == theirs.shape
    assert np.array_equal(ours, theirs.astype(np.float32))


def test_our_files_read_by_gguf(tmp_path):
    rng = np.random.default_rng(1)
    q4 = rng.integers(0, 256, 3 * 144 * 2, dtype=np.uint8)
    q6 = rng.integers(0, 256, 5 * 210, dtype=np.uint8)
    f32 = rng.standard_normal(12).astype(np.float32)
    p = tmp_path / "ours.gguf"
    G.write_gguf(p, {"general.architecture": "qwen3", "qwen3.block_count": G.Typed(G.U32, 36),
                     "qwen3.rope.freq_base": G.Typed(G.F32, 1e6), "tok": ["a", "bc"]},
                 [("w4", (512, 3), G.GGML_Q4_K, q4), ("w6", (256, 5), G.GGML_Q6_K, q6),
                  ("n", (12,), G.GGML_F32, f32.view(np.uint8))])
    r = gguf.GGUFReader(p)
    fields = r.fields
    assert bytes(fields["general.architecture"].parts[-1]).decode() == "qwen3"
    assert int(fields["qwen3.block_count"].parts[-1][0]) == 36
    assert float(fields["qwen3.rope.freq_base"].parts[-1][0]) == 1e6
    t = {x.name: x for x in r.tensors}
    assert t["w4"].tensor_type == gguf.GGMLQuantizationType.Q4_K and list(t["w4"].shape) == [512, 3]
    assert t["w6"].tensor_type == gguf.GGMLQuantizationType.Q6_K and list(t["w6"].shape) == [256, 5]
    assert np.array_equal(np.asarray(t["w4"].data).view(np.uint8).reshape(-1), q4)
    assert np.array_equal(np.asarray(t["w6"].data).view(np.uint8).reshape(-1), q6)
    assert np.array_equal(np.asarray(t["n"].data).reshape(-1), f32)


def test_gguf_files_read_by_ours(tmp_path):
    rng = np.random.default_rng(2)
    p = tmp_path / "theirs.gguf"
    w = gguf.GGUFWriter(p, "qwen3")
    w.add_uint32("qwen3.block_count", 2)
    w.add_float32("qwen3.attention.layer_norm_rms_epsilon", 1e-6)
    q4 = rng.integers(0, 256, (4, 2 * 144), dtype=np.uint8)
    w.add_tensor("blk.0.attn_q.weight", q4, raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    n = rng.standard_normal(256).astype(np.float32)
    w.add_tensor("blk.0.attn_norm.weight", n)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with G.read_gguf(p) as g:
        assert g.metadata["general.architecture"] == "qwen3"
        assert g.metadata["qwen3.block_count"] == 2
        t = g.tensors["blk.0.attn_q.weight"]
        assert t.ggml_type == G.GGML_Q4_K and t.dims == (512, 4)
        assert np.array_equal(g.data("blk.0.attn_q.weight"), q4.reshape(-1))
        assert np.array_equal(g.data("blk.0.attn_norm.weight").view(np.float32), n)
        assert G.slot_of("blk.0.attn_q.weight") == (0, 1)
