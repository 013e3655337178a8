"""Failure detection on the host, as gloo ranks on CPU (no GPU, no fault):
the tensor-parallel runtime exchanges its arena handles through
torch.distributed, and a rank that never joins, or that leaves between
steps, must turn into an error on the others within the process group's
short timeout -- not a hang."""
from __future__ import annotations

import datetime
import os
import socket
import time

import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _record(out_dir, rank, text):
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(text)


def _worker(rank, world, port, out_dir, mode):
    import torch.distributed as dist

    from abra_b200.model import IPC_HANDLE_BYTES, exchange_handles

    if mode == "never_joins" and rank == 1:
        _record(out_dir, rank, "did not join")
        return
    t0 = time.time()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=5))
    except Exception as exc:  # the group never formed
        _record(out_dir, rank, f"init raised {type(exc).__name__} after {time.time() - t0:.1f}s")
        return
    if mode == "leaves" and rank == 1:
        _record(out_dir, rank, "left")
        os._exit(0)  # gone between steps, with nothing in flight
    t0 = time.time()
    try:
        exchange_handles(bytes([rank + 1]) * IPC_HANDLE_BYTES, world)
        _record(out_dir, rank, "exchanged")
    except Exception as exc:
        _record(out_dir, rank, f"exchange raised {type(exc).__name__} after {time.time() - t0:.1f}s")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("mode", ["never_joins", "leaves"])
def test_missing_rank_becomes_an_error(tmp_path, mode):
    import torch.multiprocessing as mp

    t0 = time.time()
    ctx = mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), mode), nprocs=2,
                             join=False, start_method="spawn")
    while not ctx.join(timeout=120):
        pass
    text = (tmp_path / "rank0.txt").read_text()
    assert "raised" in text, text
    assert time.time() - t0 < 120
