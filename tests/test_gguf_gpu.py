"""GPU: a model loaded from a GGUF file decodes exactly like the oracle
model whose tensors the file holds (logits bit-identical at every step), for
the all-Q4_K and the Q4_K_M type maps.  The model is created with another
seed first, so every slot must have been overwritten by the file."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from gguf_fixture import write_qwen3

pytestmark = pytest.mark.gpu

SMALL = dict(n_layers=9, hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, vocab=3000)


@pytest.mark.parametrize("mix", [False, True])
def test_model_from_gguf_matches_oracle(tmp_path, mix):
    from abra_b200.model import DecodeModel

    p = tmp_path / "q.gguf"
    write_qwen3(p, SMALL, seed=7, mix=mix)
    with DecodeModel.from_gguf(p, max_ctx=64) as m:
        assert m.cfg.seed == 0  # the seeded weights were all replaced
        c = O.OrcModel(seed=7, centered=1, mix=int(mix), max_ctx=64, **SMALL)
        prompt = np.random.default_rng(3).integers(0, SMALL["vocab"], 5).astype(np.int32)
        m.reset(prompt)
        tok = None
        for pos in range(20):
            feed = int(prompt[pos]) if pos < 5 else tok
            tok, want = c.step(feed, pos, logits=True)
            m.step(1)
            assert np.array_equal(m.logits().view(np.uint32), want.view(np.uint32)), f"pos {pos}"
        c.close()


def test_wrong_type_for_a_slot_is_refused(tmp_path):
    """A Q6_K file loaded into an all-Q4_K model: the first Q6_K tensor is refused."""
    from abra_b200 import gguf as G
    from abra_b200.model import DecodeModel

    p = tmp_path / "q.gguf"
    write_qwen3(p, SMALL, seed=7, mix=True)
    with G.read_gguf(p) as g, DecodeModel(max_ctx=16, **SMALL) as m:
        with pytest.raises(G.GGUFError, match="type differs"):
            G.load_into(m, g)
