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
