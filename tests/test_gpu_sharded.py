"""The sharded projections on 2, 4 and 8 GPUs with NCCL, checked against the FP64 oracle: N-sharded
(each rank runs the sm_100a kernels on its W shard, the all-gather rebuilds y) and K-sharded (FP32
partials, reduce-scatter / all-reduce). A world size is skipped when the box has fewer GPUs."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from muse_bf16_proj_b200.sharded import ShardedProjection
        from oracle import contract_ref as O

        out = {}
        for m, n, k in ((1, 2048, 4096), (16, 4096, 4096), (512, 2048, 2048)):
            g = torch.Generator().manual_seed(m + n)
            w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
            x = torch.randn((m, k), generator=g).to(torch.bfloat16)
            sp = ShardedProjection(w.cuda(), n, verbose=False)
            y = sp.gather(sp.project(x.cuda()))
            torch.cuda.synchronize()
            yb = y.cpu().view(torch.int16).numpy().view(np.uint16)
            xb = x.view(torch.int16).numpy().view(np.uint16)
            wb = w.view(torch.int16).numpy().view(np.uint16)
            ok, msg, _ = O.check_implementation(xb, wb, yb)
            out[(m, n, k)] = (ok, msg)
        # Row-parallel: K-sharded FP32 partials, NCCL reduce-scatter, BF16 column slices.
        from muse_bf16_proj_b200.sharded import RowParallelProjection
        for m, n, k in ((1, 8192, 2048), (16, 8192, 2048), (200, 4096, 4096)):
            g = torch.Generator().manual_seed(3 * m + n)
            w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
            x = torch.randn((m, k), generator=g).to(torch.bfloat16)
            rp = RowParallelProjection(w.cuda(), k)
            y_full = rp.reduce(rp.partial(x.cuda()), scatter=False)
            y_cols = rp.reduce(rp.partial(x.cuda()))
            torch.cuda.synchronize()
            xb = x.view(torch.int16).numpy().view(np.uint16)
            wb = w.view(torch.int16).numpy().view(np.uint16)
            ok, msg, _ = O.check_implementation(xb, wb, y_full.cpu().view(torch.int16).numpy().view(np.uint16))
            per = n // world
            # The reduce-scatter and the all-reduce may add the ranks' FP32 partials in different orders
            # (NCCL picks the algorithm), so the BF16 results may differ by a rounding step: one unit in
            # the last place of BF16 (2^-8 relative; near zero, FP32 rounding of the partials' scale).
            cols = y_cols.cpu().float()
            ref = y_full.cpu()[:, rank * per:(rank + 1) * per].float()
            same = bool(((cols - ref).abs() <= ref.abs() * 2.0 ** -7 + 1e-5 * ref.abs().max()).all())
            out[("row", m, n, k)] = (ok and same, msg if ok else msg + "; column slice differs beyond one BF16 step")
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_projection_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True, start_method="spawn")
    for rank in range(world):
        assert results[rank], f"rank {rank} reported nothing"
        for shape, (ok, msg) in results[rank].items():
            assert ok, f"rank {rank} {shape}: {msg}"
