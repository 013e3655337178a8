"""CPU tests of prompt-lookup drafting (abra_lookup_draft), against a
restatement of the reference's draft() (tests/lookup_decode.cpp:39-51) on
random histories with repeats and the edge cases it handles."""
from __future__ import annotations

import numpy as np
import pytest


def ref_draft(history, key, limit):
    """tests/lookup_decode.cpp:39-51, restated."""
    if limit <= 0 or len(history) < 2 * key:
        return []
    suffix = len(history) - key
    for pos in range(suffix - key, -1, -1):
        if history[pos:pos + key] == history[suffix:suffix + key]:
            n = min(limit, suffix - pos - key)
            return history[pos + key:pos + key + n] if n > 0 else []
    return []


@pytest.mark.parametrize("key", [1, 2, 3])
def test_draft_matches_the_reference_rule(key):
    from abra_b200.model import lookup_draft

    rng = np.random.default_rng(key)
    for trial in range(400):
        n = int(rng.integers(0, 60))
        h = rng.integers(0, 4 if trial % 2 else 12, n).tolist()
        limit = int(rng.integers(0, 20))
        assert lookup_draft(h, key, limit).tolist() == ref_draft(h, key, limit), (h, key, limit)


def test_draft_edge_cases():
    from abra_b200.model import lookup_draft

    assert lookup_draft([], 2, 5).size == 0
    assert lookup_draft([1, 2, 3], 2, 5).size == 0           # shorter than 2 key
    assert lookup_draft([1, 2, 1, 2], 2, 0).size == 0        # no room
    assert lookup_draft([1, 2, 1, 2], 2, 5).size == 0        # match right before: nothing follows
    assert lookup_draft([1, 2, 7, 1, 2], 2, 5).tolist() == [7]
    assert lookup_draft([1, 2, 7, 8, 1, 2, 9, 1, 2], 2, 5).tolist() == [9]  # most recent match


def test_verify_and_lookup_refuse_without_a_model():
    from abra_b200 import _lib

    assert _lib.lib.abra_model_verify(None, None, 0, None, None) == _lib.ABRA_E_INVALID
    assert _lib.lib.abra_model_generate_lookup(None, None, 0, 1, 2, 8, None, None) == _lib.ABRA_E_INVALID
