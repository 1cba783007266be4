"""Host logic of the N-sharded projection on CPU ranks (gloo, world size 2 and 4): shard
boundaries, per-rank projection and the all-gather reassembly, against the FP64 oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muse_bf16_proj_b200.sharded import RowParallelProjection, ShardedProjection, shard_k, shard_rows
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


def _oracle_partial(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x . W^T in FP64, rounded to FP32: a rank's row-parallel partial."""
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    wb = w.contiguous().view(torch.int16).numpy().view(np.uint16)
    return torch.from_numpy(O.ref_product(xb, wb).astype(np.float32))


def _row_worker(rank, world, port, m, n, k, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn((m, k), generator=g).to(torch.bfloat16)
        rp = RowParallelProjection(w, k, project_fn=_oracle_partial)
        part = rp.partial(x)
        assert part.dtype == torch.float32 and part.shape == (m, n)
        y_cols = rp.reduce(part.clone())
        y_full = rp.reduce(part.clone(), scatter=False)
        xb = x.view(torch.int16).numpy().view(np.uint16)
        wb = w.view(torch.int16).numpy().view(np.uint16)
        ref = O.ref_kernel(xb, wb)
        full_bits = y_full.view(torch.int16).numpy().view(np.uint16)
        ok_full = O.check_implementation(xb, wb, full_bits, ref_bits=ref)[0]
        rel = O.relative_l2(O.bf16_to_f32(full_bits), O.bf16_to_f32(ref))
        per = n // world
        same = torch.equal(y_cols.view(torch.int16), y_full[:, rank * per:(rank + 1) * per].view(torch.int16))
        results[rank] = (ok_full, rel, same, (rp.k0, rp.k1))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_projection_gloo(world):
    """K-sharded partials in FP32, summed across ranks, rounded once: within the reference's check
    and 1e-3 of the FP64 product; the reduce-scatter slice equals the all-reduce's columns."""
    m, n, k = 6, 64 * world, 128 * world
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    mp.start_processes(_row_worker, args=(world, _free_port(), m, n, k, results), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        ok_full, rel, same, (k0, k1) = results[rank]
        assert ok_full and rel <= 1e-3 and same
        assert (k0, k1) == (rank * k // world, (rank + 1) * k // world)


def test_shard_k():
    assert shard_k(8192, 8, 7) == (7168, 8192)
    with pytest.raises(ValueError):
        shard_k(1000, 2, 0)  # 500 is not a multiple of 64



def _exchange_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from muse_bf16_proj_b200.sharded import exchange_peer_entries
        entry = {"y": (bytes([rank]) * 64, 512 * rank), "ctl": (bytes([100 + rank]) * 64, 0), "rank": rank,
                 "host": "node0"}
        got = exchange_peer_entries(entry)
        ok = [e["rank"] for e in got] == list(range(world)) and all(
            e["y"] == (bytes([q]) * 64, 512 * q) for q, e in enumerate(got))
        # A rank on another node must be refused on every rank (no IPC across hosts).
        bad = dict(entry, host="node1" if rank == world - 1 else "node0")
        try:
            exchange_peer_entries(bad)
            refused = False
        except RuntimeError:
            refused = True
        results[rank] = (ok, refused)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_peer_entries_gloo(world):
    """The fused all-gather's one-time exchange of IPC handles: every rank gets every rank's entry in
    rank order, and ranks on different hosts are refused."""
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_exchange_worker, args=(world, _free_port(), results), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        assert results[rank] == (True, True), (rank, results[rank])


def test_gather_plan():
    from muse_bf16_proj_b200 import _lib as L
    from muse_bf16_proj_b200.sharded import gather_plan
    p = gather_plan(1, 7168, 8192)  # the MLP-up shard at P = 8, decode: 56 tiles x 5 fill one wave
    assert (p.kernel, p.tile_n, p.split, p.stages) == (L.KERNEL_TC_TILE, 16, 5, 6)
    assert p.flags == L.FLAG_PDL | L.FLAG_GLOBAL_SPLIT
    p = gather_plan(1, 28672, 8192)  # P = 2: 224 tiles already fill a wave at two CTAs an SM
    assert (p.tile_n, p.split, p.flags) == (16, 1, L.FLAG_PDL)
    p = gather_plan(16, 512, 4096)  # the unpooler slice: few W tiles, K split 16 ways
    assert (p.tile_n, p.split) == (16, 16)
    p = gather_plan(100, 2048, 64)  # K = one block: no split
    assert (p.tile_n, p.split, p.flags) == (128, 1, L.FLAG_PDL)
    assert gather_plan(8192, 7168, 8192).kernel == L.KERNEL_TC_GEMM2
