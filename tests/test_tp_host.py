"""Host side of tensor parallelism on CPU: two gloo ranks exchange their
exchange-buffer handles through mogemma_b200._core.gather_handles, the call
init_model_tp makes before mg_tp_connect (which then maps the handles in rank
order).  No GPU is involved."""

from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _rank(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mogemma_b200 import _core  # noqa: PLC0415

        mine = bytes([rank + 1]) * _core.TP_HANDLE_BYTES
        got = _core.gather_handles(mine)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_handles_gathered_in_rank_order(world: int) -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = [bytes([r + 1]) * 64 for r in range(world)]
    assert all(results[r] == expect for r in range(world))
