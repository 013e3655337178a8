"""Property tests of the GGUF writer/reader (hypothesis): random metadata of
every value type and random tensor sets round-trip through our reader, and
through the gguf package's reader where it is installed."""
from __future__ import annotations

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from abra_b200 import gguf as G

KEY = st.text(alphabet="abcdefghijklmnopqrstuvwxyz._", min_size=1, max_size=24)
SCALARS = st.one_of(
    st.builds(lambda v: G.Typed(G.U8, v), st.integers(0, 255)),
    st.builds(lambda v: G.Typed(G.I16, v), st.integers(-2**15, 2**15 - 1)),
    st.builds(lambda v: G.Typed(G.U32, v), st.integers(0, 2**32 - 1)),
    st.builds(lambda v: G.Typed(G.I32, v), st.integers(-2**31, 2**31 - 1)),
    st.integers(-2**63, 2**63 - 1),
    st.booleans(),
    st.text(max_size=40),
    st.builds(lambda v: G.Typed(G.F64, v), st.floats(allow_nan=False)),
    st.lists(st.text(max_size=8), max_size=6),
    st.builds(lambda v: np.array(v, dtype=np.int32), st.lists(st.integers(-2**31, 2**31 - 1), max_size=6)),
)
TENSOR = st.tuples(st.sampled_from([G.GGML_F32, G.GGML_Q4_K, G.GGML_Q6_K]),
                   st.integers(1, 3), st.integers(1, 4))


def _plain(v):
    v = v.value if isinstance(v, G.Typed) else v
    return v.tolist() if isinstance(v, np.ndarray) else v


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(meta=st.dictionaries(KEY, SCALARS, max_size=8), shapes=st.lists(TENSOR, max_size=4),
       alignment=st.sampled_from([32, 64, 128]), seed=st.integers(0, 2**16))
def test_random_files_round_trip(tmp_path, meta, shapes, alignment, seed):
    meta.pop("general.alignment", None)
    rng = np.random.default_rng(seed)
    tensors = []
    for i, (gt, rows, blocks) in enumerate(shapes):
        per, size = G.GGML_BLOCKS[gt]
        dims = (blocks * per, rows)
        data = rng.integers(0, 256, rows * blocks * size, dtype=np.uint8)
        tensors.append((f"t{i}", dims, gt, data))
    p = tmp_path / f"r{seed}.gguf"
    G.write_gguf(p, meta, tensors, alignment=alignment)
    with G.read_gguf(p) as g:
        assert g.alignment == alignment
        for k, v in meta.items():
            got = g.metadata[k]
            assert _plain(got) == _plain(v), k
        for name, dims, gt, data in tensors:
            t = g.tensors[name]
            assert (t.dims, t.ggml_type) == (dims, gt)
            assert np.array_equal(g.data(name), data)
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(p)
    theirs = {t.name: t for t in r.tensors}
    for name, dims, gt, data in tensors:
        assert np.array_equal(np.asarray(theirs[name].data).view(np.uint8).reshape(-1), data)
