"""Property tests (hypothesis) of the canonical order on random shapes:
for Q4_K and Q6_K rows of any superblock count, the GEMV is the fixed tree
of the eight K-slice sums, every 2/4/8-way K-shard split recombines to the
same bits, and the result is within 1e-5 of sum|w||x| of the f64 oracle."""
from __future__ import annotations

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

import oracle as O

CASES = st.tuples(st.sampled_from(["q4k", "q6k"]), st.integers(1, 9), st.integers(1, 41),
                  st.integers(1, 3), st.integers(0, 2**20))


@settings(max_examples=30, deadline=None)
@given(case=CASES)
def test_canonical_order_invariants(case):
    kind, N, nsb, ncols, seed = case
    K = nsb * 256
    xq = O.quantize_q8_1(O.gen_normal_f32((ncols, K), seed))
    if kind == "q4k":
        w = O.gen_q4k(N, K, seed, 1, centered=bool(seed & 1))
        y, v = O.gemv(w, xq, K), O.gemv_slices(w, xq, K)
        y64, s = O.gemv_f64(w, xq, K), O.absdot_f64(w, xq, K)
    else:
        w = O.gen_q6k(N, K, seed, 2)
        y, v = O.q6k_gemv(w, xq, K), O.q6k_gemv_slices(w, xq, K)
        y64, s = O.q6k_gemv_f64(w, xq, K), O.q6k_absdot_f64(w, xq, K)
    assert np.array_equal(O.tree8(v), y)
    for world in (2, 4, 8):
        per = 8 // world
        parts = [O.kshard_partial(v, r * per, per) for r in range(world)]
        assert np.array_equal(O.delta_tree(parts), y)
    assert (np.abs(y.astype(np.float64) - y64) <= 1e-5 * np.maximum(s, 1e-30)).all()
