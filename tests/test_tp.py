"""Tensor-parallel split, host side (no GPU): the shard plan of every world
size tiles the model, K-shard partial sums recombine to the unsharded bits
(oracle arithmetic), and the arena-handle exchange works over gloo with two
ranks.  The GPU halves are in test_tp_gpu.py."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import oracle as O

WORLDS = [1, 2, 4, 8]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", WORLDS)
def test_shard_plan_tiles_the_model(world):
    from abra_b200.model import default_config, shard_info

    c = default_config()
    shards = [shard_info(r, world) for r in range(world)]
    qh = [s.q_heads for s in shards]
    assert sum(qh) == c.n_heads and sum(s.kv_heads for s in shards) == c.n_kv_heads
    for r, s in enumerate(shards):
        assert s.q_head_lo == r * s.q_heads and s.kv_head_lo == r * s.kv_heads
        # every rank keeps whole GQA groups
        assert s.q_heads // s.kv_heads == c.n_heads // c.n_kv_heads
    assert [s.ffn_lo for s in shards][0] == 0 and shards[-1].ffn_hi == c.ffn
    assert [s.vocab_lo for s in shards][0] == 0 and shards[-1].vocab_hi == c.vocab
    for a, b in zip(shards, shards[1:]):
        assert a.ffn_hi == b.ffn_lo and a.vocab_hi == b.vocab_lo
        assert a.sl_base + a.sl_cnt == b.sl_base
    from abra_b200 import slice_start

    nsb_f, nsb_o = c.ffn // 256, c.n_heads * c.head_dim // 256
    for s in shards:
        # FFN units and o columns sit exactly on canonical K-slices
        assert s.ffn_lo == slice_start(nsb_f, s.sl_base) * 256
        assert s.ffn_hi == slice_start(nsb_f, s.sl_base + s.sl_cnt) * 256
        assert s.q_head_lo * c.head_dim == slice_start(nsb_o, s.sl_base) * 256


def test_shard_plan_rejects_bad_splits():
    from abra_b200 import AbraError
    from abra_b200.model import shard_info

    for rank, world in [(0, 3), (2, 2), (-1, 2), (0, 16)]:
        with pytest.raises(AbraError):
            shard_info(rank, world)
    with pytest.raises(AbraError):
        shard_info(0, 8, n_kv_heads=4, n_heads=16)  # 4 kv heads cannot split 8 ways


@pytest.mark.parametrize("N,K", [(48, 4096), (40, 9728), (16, 2304)])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_kshard_partials_recombine_bit_exact(N, K, world):
    """Each rank's partial (its canonical slices, the rest +0.0, the same
    tree) summed in the fixed tree equals the unsharded canonical sum."""
    w = O.gen_q4k(N, K, 4, 21)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K), 8))
    slices = O.gemv_slices(w, xq, K)
    full = O.gemv(w, xq, K)
    assert np.array_equal(O.tree8(slices), full)
    per = 8 // world
    parts = [O.kshard_partial(slices, r * per, per) for r in range(world)]
    assert np.array_equal(O.delta_tree(parts), full)


def _exchange_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from abra_b200.model import IPC_HANDLE_BYTES, exchange_handles, shard_info

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        mine = bytes([rank + 1]) * IPC_HANDLE_BYTES
        allh = exchange_handles(mine, world)
        plans = [None] * world
        dist.all_gather_object(plans, shard_info(rank, world).as_dict())
        with open(os.path.join(out_dir, f"rank{rank}.npz"), "wb") as f:
            np.savez(f, handles=np.frombuffer(allh, dtype=np.uint8),
                     vocab=np.array([[p["vocab_lo"], p["vocab_hi"]] for p in plans]))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_two_ranks(tmp_path):
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    mp.spawn(_exchange_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    want = b"".join(bytes([r + 1]) * 64 for r in range(world))
    for r in range(world):
        d = np.load(tmp_path / f"rank{r}.npz")
        assert d["handles"].tobytes() == want
        assert d["vocab"].tolist() == [[0, 75968], [75968, 151936]]


def _slice(cfg, rank, world, layer, slot):
    import ctypes as C

    from abra_b200 import _lib

    out = (C.c_int64 * 8)()
    rc = _lib.lib.abra_tp_tensor_slice(C.byref(cfg), rank, world, layer, slot, out)
    assert rc == _lib.ABRA_OK, _lib.lib.abra_model_last_error()
    return dict(zip(("type", "N", "K", "rb", "r0", "nr", "b0", "nb"), list(out)))


ROW_SPLIT = {1: "q", 9: "k", 10: "v", 6: "gate", 7: "up"}
K_SPLIT = {4: "o", 8: "down"}
WHOLE = {0: "attn_norm", 2: "q_norm", 3: "k_norm", 5: "ffn_norm"}


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_gguf_tensor_slices_tile_every_tensor(world):
    """What each rank keeps of a GGUF tensor (abra_model_load_tensor's cut):
    row-split tensors partition the rows, K-split ones each row's bytes
    along the canonical slices, the rest are whole on every rank -- the same
    placement as the seeded weights (heads, FFN units, K-slices)."""
    from abra_b200.model import default_config, shard_info

    cfg = default_config()
    for layer, slots in ((-1, {1: "embd", 2: "out_norm"}), (0, {**ROW_SPLIT, **K_SPLIT, **WHOLE}),
                         (35, {**ROW_SPLIT, **K_SPLIT})):
        for slot, name in slots.items():
            sl = [_slice(cfg, r, world, layer, slot) for r in range(world)]
            assert len({(s["type"], s["N"], s["K"], s["rb"]) for s in sl}) == 1, name
            N, rb = sl[0]["N"], sl[0]["rb"]
            if slot in ROW_SPLIT and layer >= 0:
                spans = sorted((s["r0"], s["r0"] + s["nr"]) for s in sl)
                assert spans[0][0] == 0 and spans[-1][1] == N, name
                assert all(a[1] == b[0] for a, b in zip(spans, spans[1:])), name
                assert all(s["b0"] == 0 and s["nb"] == rb for s in sl)
            elif slot in K_SPLIT and layer >= 0:
                spans = sorted((s["b0"], s["b0"] + s["nb"]) for s in sl)
                assert spans[0][0] == 0 and spans[-1][1] == rb, name
                assert all(a[1] == b[0] for a, b in zip(spans, spans[1:])), name
                assert all(s["r0"] == 0 and s["nr"] == N for s in sl)
            else:
                assert all((s["r0"], s["nr"], s["b0"], s["nb"]) == (0, N, 0, rb) for s in sl), name
        for r in range(world):
            sh = shard_info(r, world)
            q = _slice(cfg, r, world, 0, 1)
            assert (q["r0"], q["nr"]) == (sh.q_head_lo * 128, sh.q_heads * 128)
            g = _slice(cfg, r, world, 0, 6)
            assert (g["r0"], g["r0"] + g["nr"]) == (sh.ffn_lo, sh.ffn_hi)
            d = _slice(cfg, r, world, 0, 8)
            assert (d["b0"] // 144 * 256, (d["b0"] + d["nb"]) // 144 * 256) == (sh.ffn_lo, sh.ffn_hi)
            o = _slice(cfg, r, world, 0, 4)
            nsb_o = 4096 // 256
            assert o["b0"] // 144 == O.slice_starts(nsb_o)[sh.sl_base]


def test_gguf_tensor_slices_of_the_q4_k_m_map():
    from abra_b200.model import Q4_K_M, default_config, q6k_layers

    cfg = default_config(flags=Q4_K_M)
    q6 = set(q6k_layers(36))
    assert _slice(cfg, 0, 1, -1, 1)["type"] == 14
    for layer in range(36):
        assert _slice(cfg, 0, 1, layer, 10)["type"] == (14 if layer in q6 else 12)
        assert _slice(cfg, 0, 1, layer, 8)["type"] == (14 if layer in q6 else 12)
        assert _slice(cfg, 0, 1, layer, 1)["type"] == 12
    assert _slice(cfg, 0, 1, 0, 8)["rb"] == 9728 // 256 * 210
