"""Host logic of the N-sharded projection on CPU ranks (gloo, world size 2 and 4): shard
boundaries, per-rank projection and the all-gather reassembly, against the FP64 oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muse_bf16_proj_b200.sharded import ShardedProjection, shard_rows
from oracle import contract_ref as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_project(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    wb = w.contiguous().view(torch.int16).numpy().view(np.uint16)
    return torch.from_numpy(O.ref_kernel(xb, wb).view(np.int16)).view(torch.bfloat16)


def _worker(rank, world, port, m, n, k, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn((m, k), generator=g).to(torch.bfloat16)
        sp = ShardedProjection(w, n, project_fn=_oracle_project)
        y_local = sp.project(x)
        assert y_local.shape == (m, n // world)
        y = sp.gather(y_local)
        ym = sp.gather(y_local, rank_major=True)
        full = _oracle_project(x, w)
        results[rank] = (torch.equal(y.view(torch.int16), full.view(torch.int16)),
                         torch.equal(ym.permute(1, 0, 2).reshape(m, n).view(torch.int16), full.view(torch.int16)),
                         (sp.r0, sp.r1))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_projection_gloo(world):
    m, n, k = 5, 64 * world, 256
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), m, n, k, results), nprocs=world, join=True,
                       start_method="spawn")
    assert sorted(results.keys()) == list(range(world))
    for rank in range(world):
        ok_full, ok_rank_major, (r0, r1) = results[rank]
        assert ok_full and ok_rank_major
        assert (r0, r1) == (rank * n // world, (rank + 1) * n // world)


def test_shard_rows():
    assert shard_rows(57344, 8, 7) == (50176, 57344)
    assert shard_rows(57344, 1, 0) == (0, 57344)
    with pytest.raises(ValueError):
        shard_rows(100, 3, 0)
    with pytest.raises(ValueError):
        shard_rows(100, 2, 2)
