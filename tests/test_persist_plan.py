"""Host-side checks of the persistent decode kernel's plan (no GPU).

abra_persist_plan walks every weight copy each CTA's warps would issue over
one token -- per layer the q|k|v, o, gate/up and down units, then
the tied output -- and checks it against its shared-memory ring slot (bounds,
16-byte alignment, the mbarrier transaction limit) and against its weight
tensor; it follows every lane of a unit through its superblock reads, its
staging-buffer writes and the row sums' reads (the kernel's lane map); and it
checks the ticket walk by which each warp refills the slot
it finished (from the start, and NSLOT tickets ahead of every ticket) against
the sequential phase-by-phase order.  The sizes are the decode model's shapes
on B200's 148 SMs and on other SM counts, so that the grid split leaves
ragged row ranges."""
from __future__ import annotations

import pytest

from abra_b200._lib import ABRA_E_UNSUPPORTED, AbraError
from abra_b200.model import persist_plan

QWEN = dict(n_layers=36)
SHAPES = [
    QWEN,
    dict(n_layers=2, vocab=4096),
    dict(n_layers=9, hidden=512, n_heads=4, n_kv_heads=2, ffn=1024, vocab=3000),
    dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=1, ffn=768, vocab=1000),
    dict(n_layers=2, hidden=256, n_heads=2, n_kv_heads=2, ffn=512, vocab=1000),
    dict(n_layers=0, vocab=300),
    # wide activations: the eight-slot ring (the refill walk NSLOT = 8 ahead)
    dict(n_layers=3, hidden=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=5000),
]


@pytest.mark.parametrize("sms", [148, 132, 7, 1])
@pytest.mark.parametrize("shape", SHAPES)
def test_every_copy_fits_its_slot_and_tensor(shape, sms):
    p = persist_plan(sms, **shape)
    assert p["smem"] <= 227 * 1024 - 1024
    assert p["ring_bytes"] % (8 * 16) == 0
    assert p["copies"] > 0


def test_wide_shape_uses_eight_slots():
    """A 4096-wide model with a 14336-wide FFN leaves room for eight ring
    slots only; its plan (every copy, and the walk by which each warp refills
    the slot it finished with the unit eight tickets ahead) is checked like
    the sixteen-slot plans."""
    p = persist_plan(148, n_layers=3, hidden=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=5000)
    assert p["ring_bytes"] == 8 * 8 * 1456


def test_qwen_plan():
    """The Qwen3-4B shape: eight rows of a 2560-wide matrix per ring slot for
    q|k|v and the output, four rows of o (K=4096) and of gate/up (two
    matrices), two rows of down (K=9728)."""
    p = persist_plan(148, **QWEN)
    rows = (p["rows_qkv"], p["rows_o"], p["rows_gate_up"], p["rows_down"], p["rows_output"])
    assert rows == (8, 4, 4, 2, 8)
    assert p["ring_bytes"] == 16 * 8 * 1456  # sixteen slots


@pytest.mark.parametrize("shape", [
    dict(n_heads=12, n_kv_heads=4),              # 3 q heads per kv head
    dict(hidden=16384, n_heads=128, ffn=16384),  # activations beyond the shared-memory plan
])
def test_unsupported_shapes_are_refused(shape):
    with pytest.raises(AbraError) as e:
        persist_plan(148, n_layers=1, **shape)
    assert e.value.code == ABRA_E_UNSUPPORTED
