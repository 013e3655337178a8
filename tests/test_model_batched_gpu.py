"""Batched decode (32 sequences in lockstep, every GEMV on the tcgen05
tensor cores): each sequence's greedy tokens and logits must equal those of
the batch-1 model run on the same prompt, bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _batch1(cfg, prompt, n_steps):
    from abra_b200.model import DecodeModel

    with DecodeModel(**cfg) as m:
        m.reset(prompt)
        m.step(n_steps)
        m.sync()
        return m.tokens(n_steps + 1), m.logits()


@pytest.mark.parametrize("cfg,n_steps,check", [
    (dict(n_layers=2, vocab=4096, max_ctx=96, centered=1, seed=3), 40, range(32)),
    (dict(max_ctx=48, centered=1, seed=1), 12, (0, 13, 31)),
], ids=["small", "qwen3_4b"])
def test_batched_matches_batch1(dev, cfg, n_steps, check):
    import abra_b200 as A
    from abra_b200.model import BatchedDecodeModel

    prompts = np.random.default_rng(5).integers(0, cfg.get("vocab", 151936), (32, 9)).astype(np.int32)
    with BatchedDecodeModel(32, **cfg) as mb:
        mb.reset(prompts)
        mb.step(n_steps)
        mb.sync()
        toks, lg = mb.tokens(n_steps + 1), mb.logits()
    assert A.device_error() == 0
    for i in check:
        t1, l1 = _batch1(cfg, prompts[i], n_steps)
        assert np.array_equal(toks[i], t1), f"sequence {i}: tokens differ"
        assert np.array_equal(lg[i], l1), f"sequence {i}: logits differ"


def test_batched_rejects_other_sizes():
    from abra_b200 import AbraError
    from abra_b200.model import BatchedDecodeModel

    with pytest.raises(AbraError):
        BatchedDecodeModel(16, n_layers=1, vocab=512, max_ctx=16)
