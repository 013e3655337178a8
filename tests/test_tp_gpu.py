"""Tensor-parallel decode on the GPU.

One GPU: the row-parallel (K-sharded) MMVQ gives each rank's partial sums
bit for bit as the oracle forms them, and the fixed-tree sum of the ranks'
partials equals the unsharded MMVQ.

Two or more GPUs: the tensor-parallel model (world = 2, 4, 8, one process
per GPU, arena handles exchanged over gloo) produces the same greedy tokens
and the same logits, bit for bit, as the one-GPU model.  Skipped when the
box has fewer GPUs than the world size.
"""
from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest

import oracle as O
from conftest import to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,K_full", [(2560, 4096), (2560, 9728), (300, 2304)])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_kshard_mmvq_bit_exact(dev, N, K_full, world):
    import torch
    import abra_b200 as A

    nsb = K_full // 256
    w = O.gen_q4k(N, K_full, 6, 33).reshape(N, nsb, 144)
    xq = O.quantize_q8_1(O.gen_normal_f32((1, K_full), 12)).reshape(nsb * 8, 36)
    slices = O.gemv_slices(w.reshape(-1), xq.reshape(-1), K_full)
    full = O.gemv(w.reshape(-1), xq.reshape(-1), K_full, nthreads=8)
    per = 8 // world
    parts = []
    for r in range(world):
        lo, hi = A.slice_start(nsb, r * per), A.slice_start(nsb, (r + 1) * per)
        K = (hi - lo) * 256
        dw = to_dev(np.ascontiguousarray(w[:, lo:hi]).reshape(-1), dev)
        dx = to_dev(np.ascontiguousarray(xq[lo * 8:hi * 8]).reshape(-1), dev)
        dy = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
        A.mmvq_kshard(dw, dx, dy, N, K, K_full, r * per, per)
        torch.cuda.synchronize()
        y = dy.cpu().numpy().reshape(1, N)
        assert np.array_equal(y, O.kshard_partial(slices, r * per, per)), f"rank {r}"
        parts.append(y)
    assert np.array_equal(O.delta_tree(parts), full)
    assert A.device_error() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SMALL = dict(n_layers=2, vocab=4096, max_ctx=64, centered=1, seed=3)
FULL = dict(max_ctx=48, centered=1, seed=1)


def _tp_worker(rank, world, port, cfg, n_steps, prompt):
    import torch
    import torch.distributed as dist

    import abra_b200 as A
    from abra_b200.model import DecodeModel

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=180))
    m = None
    try:
        m = DecodeModel(rank=rank, world=world, **cfg)
        m.reset(prompt)
        m.step(n_steps)
        m.sync()
        toks = m.tokens(n_steps + 1)
        logits = m.logits()
        err = A.device_error()
        got = [None] * world
        dist.all_gather_object(got, (toks, logits, err))
        dist.barrier()  # every rank is done stepping before any arena is freed
        m.close()
        m = None
        dist.barrier()
        if rank == 0:
            assert all(g[2] == 0 for g in got), "a bounded cross-rank wait gave up"
            ref = DecodeModel(**cfg)
            ref.reset(prompt)
            ref.step(n_steps)
            ref.sync()
            ref_toks = ref.tokens(n_steps + 1)
            ref_logits = ref.logits()
            ref.close()
            for r, g in enumerate(got):
                assert np.array_equal(g[0], ref_toks), f"rank {r} tokens differ"
            tp_logits = np.concatenate([g[1] for g in got])
            assert np.array_equal(tp_logits, ref_logits), "logits differ from one GPU"
    finally:
        if m is not None:
            # leave together: peers push into this rank's arena until they
            # have finished their steps
            try:
                dist.barrier()
            finally:
                m.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("cfg,n_steps", [(SMALL, 24), (FULL, 12)], ids=["small", "qwen3_4b"])
def test_tp_model_matches_one_gpu(world, cfg, n_steps):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    prompt = np.random.default_rng(world).integers(0, cfg.get("vocab", 151936), 9).astype(np.int32)
    mp.spawn(_tp_worker, args=(world, _free_port(), cfg, n_steps, prompt), nprocs=world, join=True)


def _tp_batched_worker(rank, world, port, cfg, n_steps, prompts):
    import torch
    import torch.distributed as dist

    import abra_b200 as A
    from abra_b200.model import BatchedDecodeModel

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=180))
    m = None
    try:
        m = BatchedDecodeModel(batch=32, rank=rank, world=world, **cfg)
        m.reset(prompts)
        m.step(n_steps)
        m.sync()
        n_prompt = prompts.shape[1]
        toks = m.tokens(n_prompt + n_steps)
        logits = m.logits()
        err = A.device_error()
        got = [None] * world
        dist.all_gather_object(got, (toks, logits, err))
        dist.barrier()  # every rank is done stepping before any arena is freed
        m.close()
        m = None
        dist.barrier()
        if rank == 0:
            assert all(g[2] == 0 for g in got), "a bounded cross-rank wait gave up"
            ref = BatchedDecodeModel(batch=32, **cfg)
            ref.reset(prompts)
            ref.step(n_steps)
            ref.sync()
            ref_toks = ref.tokens(n_prompt + n_steps)
            ref_logits = ref.logits()
            ref.close()
            for r, g in enumerate(got):
                assert np.array_equal(g[0], ref_toks), f"rank {r} tokens differ"
            tp_logits = np.concatenate([g[1] for g in got], axis=1)
            assert np.array_equal(tp_logits, ref_logits), "logits differ from one GPU"
    finally:
        if m is not None:
            try:
                dist.barrier()
            finally:
                m.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("cfg,n_steps", [(SMALL, 10), (FULL, 6)], ids=["small", "qwen3_4b"])
def test_tp_batched_model_matches_one_gpu(world, cfg, n_steps):
    """Batch 32 on the tensor cores split over world GPUs: every sequence's
    tokens and every logit equal the one-GPU batch-32 model's, bit for bit
    (o/down partial sums pushed from the tcgen05 MMVQ epilogue, the per-
    sequence argmax keys merged across ranks)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    prompts = np.random.default_rng(100 + world).integers(0, cfg.get("vocab", 151936), (32, 5)).astype(np.int32)
    mp.spawn(_tp_batched_worker, args=(world, _free_port(), cfg, n_steps, prompts), nprocs=world, join=True)
