"""Failure detection of the sharded projections on the host (gloo ranks on CPU, world size 2, no
GPU): when a rank never reaches a collective, or leaves before it, the other rank's all-gather
(column-parallel) or reduce (row-parallel) ends with an error within the process group's timeout
instead of waiting for good. The failure is made on the host: a rank that sleeps past the timeout
without taking the collective, or one that raises before it."""

import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muse_bf16_proj_b200.sharded import RowParallelProjection, ShardedProjection
from oracle import contract_ref as O

PG_TIMEOUT_S = 3.0
BOUND_S = 30.0  # the surviving rank must have its error well before this


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _project(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    wb = w.contiguous().view(torch.int16).numpy().view(np.uint16)
    return torch.from_numpy(O.ref_kernel(xb, wb).view(np.int16)).view(torch.bfloat16)


def _partial(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    wb = w.contiguous().view(torch.int16).numpy().view(np.uint16)
    return torch.from_numpy(O.ref_product(xb, wb).astype(np.float32))


def _worker(rank, world, port, kind, how, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=PG_TIMEOUT_S))
    out = {"raised": False, "elapsed": 0.0, "msg": ""}
    try:
        g = torch.Generator().manual_seed(5)
        m, n, k = 4, 64 * world, 128 * world
        w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn((m, k), generator=g).to(torch.bfloat16)
        if kind == "columns":
            sp = ShardedProjection(w, n, project_fn=_project)
            local = sp.project(x)
            step = lambda: sp.gather(local)  # noqa: E731
        else:
            rp = RowParallelProjection(w, k, project_fn=_partial)
            part = rp.partial(x)
            step = lambda: rp.reduce(part.clone())  # noqa: E731
        if rank == world - 1:  # the failing rank: it never takes the collective
            if how == "raise":
                raise RuntimeError("rank failed before the collective")
            time.sleep(2 * PG_TIMEOUT_S + 2)
            return
        t0 = time.monotonic()
        try:
            step()
        except Exception as e:  # the error the survivor must see
            out.update(raised=True, msg=repr(e)[:300])
        out["elapsed"] = time.monotonic() - t0
    except RuntimeError as e:
        out["msg"] = repr(e)[:300]
    finally:
        results[rank] = out
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("kind", ["columns", "rows"])
@pytest.mark.parametrize("how", ["never_joins", "raise"])
def test_survivor_errors_instead_of_hanging(kind, how):
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    t0 = time.monotonic()
    mp.start_processes(_worker, args=(world, _free_port(), kind, how, results), nprocs=world, join=True,
                       start_method="spawn")
    assert time.monotonic() - t0 < 120
    survivor = results[0]
    assert survivor["raised"], f"rank 0's collective returned although rank 1 never joined: {survivor}"
    assert survivor["elapsed"] < BOUND_S, survivor
    msg = survivor["msg"].lower()
    # A transport error, not some other failure: gloo words a peer that left as a closed, reset or
    # broken connection depending on which side of the socket notices first.
    assert any(s in msg for s in ("timed out", "timeout", "closed", "reset", "broken pipe", "connection")), survivor
    if how == "never_joins":  # it waited out the process group's timeout, no longer
        assert survivor["elapsed"] >= 0.8 * PG_TIMEOUT_S, survivor
    if how == "raise":
        assert "rank failed before the collective" in results[1]["msg"]
