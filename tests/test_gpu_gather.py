"""The projection with its all-gather fused into the epilogue (muse_proj_bf16_tiles_gather).

On one GPU: world 1 (the epilogue writes a column window of a wider y_full) must equal the plain
tile-kernel call bit for bit, over repeated calls (the control block's epoch advances each call),
for the tile kernel (plain and K split through scratch) and the pair GEMM; and a peer that never
joins (a second control block on the same GPU that no kernel writes) must end the launch with the
arrival timeout in the device error word instead of a hang, this rank's own columns still written.
On 2, 4 and 8 GPUs (as many as the box has): every rank's y_full holds every rank's columns,
against the FP64 oracle and bit for bit against each rank's plain call. Peer pointers come from CUDA IPC handles; no TMA or bulk copy
reads a peer's memory.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muse_bf16_proj_b200 import _lib
from oracle import contract_ref as O

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _packed(w: torch.Tensor, stream: int) -> torch.Tensor:
    n, k = w.shape
    tiles = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device=w.device)
    _lib.pack_tiles(w.data_ptr(), tiles.data_ptr(), n, k, stream)
    return tiles


def _plain(x, tiles, m, n, k, plan, stream):
    y = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    need = _lib.scratch_bytes(m, n, k, plan)
    scratch = torch.zeros(max(need, 1), dtype=torch.uint8, device=x.device)
    _lib.proj_bf16_tiles(x.data_ptr(), tiles.data_ptr(), y.data_ptr(), m, n, k, plan, stream,
                         scratch.data_ptr() if need else 0, need)
    return y


def _tile_plan(tile_n, split):
    flags = _lib.FLAG_PDL | (_lib.FLAG_GLOBAL_SPLIT if split > 1 else 0)
    return _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=tile_n, split=split, flags=flags)


CASES = [
    (1, 2048, 4096, _tile_plan(16, 1)),
    (5, 1024, 4096, _tile_plan(16, 8)),
    (40, 512, 2048, _tile_plan(64, 4)),
    (300, 1024, 1024, _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2)),
    (512, 768, 2048, _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2)),
]


@pytest.mark.parametrize("m,n,k,plan", CASES)
def test_world1_window_equals_plain_call(m, n, k, plan):
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(17 * m + n)
    w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16).cuda()
    tiles = _packed(w, stream)
    col0, ldy = 64, n + 128  # this "rank" owns columns 64 .. 64 + n of a wider output
    y_full = torch.full((m, ldy), 7.0, dtype=torch.bfloat16, device="cuda")
    ctl = torch.zeros(_lib.peer_ctl_bytes(), dtype=torch.uint8, device="cuda")
    gat = _lib.MuseGather()
    gat.world, gat.rank, gat.ldy, gat.col0 = 1, 0, ldy, col0
    gat.y[0], gat.ctl[0] = y_full.data_ptr(), ctl.data_ptr()
    need = _lib.scratch_bytes(m, n, k, plan)
    scratch = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    for call in range(3):
        x = torch.randn((m, k), generator=g).to(torch.bfloat16).cuda()
        _lib.proj_bf16_tiles_gather(x.data_ptr(), tiles.data_ptr(), m, n, k, gat, plan, stream,
                                    scratch.data_ptr() if need else 0, need)
        assert _lib.device_error(stream) == 0
        ref = _plain(x, tiles, m, n, k, plan, stream)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(y_full[:, col0:col0 + n]), _bits(ref)), f"call {call}"
        outside = torch.cat([y_full[:, :col0], y_full[:, col0 + n:]], dim=1)
        assert bool((outside == 7.0).all()), "columns outside the window were written"
        ok, msg, _ = O.check_implementation(_bits(x), _bits(w), _bits(ref))
        assert ok, msg
    epoch = int(ctl[:4].view(torch.int32).item())
    assert epoch == 3, f"control block epoch {epoch} after 3 calls"


def test_peer_that_never_joins_times_out():
    stream = torch.cuda.current_stream().cuda_stream
    m, n, k = 4, 1024, 2048
    g = torch.Generator().manual_seed(99)
    w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16).cuda()
    x = torch.randn((m, k), generator=g).to(torch.bfloat16).cuda()
    tiles = _packed(w, stream)
    plan = _tile_plan(16, 1)
    # Rank 0 of 2; "rank 1" is a buffer and control block on this GPU that no kernel ever writes.
    y0 = torch.zeros((m, 2 * n), dtype=torch.bfloat16, device="cuda")
    y1 = torch.zeros((m, 2 * n), dtype=torch.bfloat16, device="cuda")
    ctl = torch.zeros((2, _lib.peer_ctl_bytes()), dtype=torch.uint8, device="cuda")
    gat = _lib.MuseGather()
    gat.world, gat.rank, gat.ldy, gat.col0 = 2, 0, 2 * n, 0
    gat.y[0], gat.y[1] = y0.data_ptr(), y1.data_ptr()
    gat.ctl[0], gat.ctl[1] = ctl[0].data_ptr(), ctl[1].data_ptr()
    _lib.device_error(stream)  # start from a clear error word
    _lib.proj_bf16_tiles_gather(x.data_ptr(), tiles.data_ptr(), m, n, k, gat, plan, stream)
    with pytest.raises(_lib.MuseError) as err:
        _lib.device_error(stream)
    assert "0x401" in str(err.value) or "1025" in str(err.value)
    ref = _plain(x, tiles, m, n, k, plan, stream)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(y0[:, :n]), _bits(ref)), "own columns must still be written"
    assert bool((y1 == 0).all()), "nothing may be written to a peer that never arrived"
    assert _lib.device_error(stream) == 0


def test_late_peer_after_a_timeout_ends_with_an_error():
    """Two "ranks" on one GPU, run one after the other: rank 0's call times out waiting for rank 1's
    arrival (0x401) and, having written only its own copy, publishes no done flag; rank 1 then
    arrives late, sees rank 0's arrival, stores its slice and waits for rank 0's done flag, which
    never comes: its call must end with 0x402, not complete as if y_full held every slice."""
    stream = torch.cuda.current_stream().cuda_stream
    m, n, k = 4, 1024, 2048
    g = torch.Generator().manual_seed(7)
    w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16).cuda()
    x = torch.randn((m, k), generator=g).to(torch.bfloat16).cuda()
    tiles = _packed(w, stream)
    plan = _tile_plan(16, 1)
    y = [torch.zeros((m, 2 * n), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ctl = torch.zeros((2, _lib.peer_ctl_bytes()), dtype=torch.uint8, device="cuda")
    _lib.device_error(stream)  # start from a clear error word
    for rank, expect in ((0, "0x401"), (1, "0x402")):
        gat = _lib.MuseGather()
        gat.world, gat.rank, gat.ldy, gat.col0 = 2, rank, 2 * n, rank * n
        gat.y[0], gat.y[1] = y[0].data_ptr(), y[1].data_ptr()
        gat.ctl[0], gat.ctl[1] = ctl[0].data_ptr(), ctl[1].data_ptr()
        _lib.proj_bf16_tiles_gather(x.data_ptr(), tiles.data_ptr(), m, n, k, gat, plan, stream)
        with pytest.raises(_lib.MuseError) as err:
            _lib.device_error(stream)
        assert expect in str(err.value), (rank, str(err.value))
    assert _lib.device_error(stream) == 0


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
    out = {}
    try:
        from muse_bf16_proj_b200.sharded import FusedGatherProjection, shard_rows
        stream = torch.cuda.current_stream().cuda_stream
        for m, n, k in ((1, 4096, 4096), (16, 2048, 8192), (77, 1024, 2048), (300, 2048, 1024)):
            g = torch.Generator().manual_seed(m + n + k)
            w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16)
            fg = FusedGatherProjection(w.cuda(), n, max_rows=512)
            r0, r1 = shard_rows(n, world, rank)
            good, msg = True, ""
            for call in range(4):  # repeated calls: the epoch protocol, fresh x every call
                x = torch.randn((m, k), generator=g).to(torch.bfloat16)
                y = fg.project(x.cuda())
                mine = _plain(x.cuda(), fg.tiles, m, r1 - r0, k, fg.plan(m), stream)
                torch.cuda.synchronize()
                code = _lib.device_error(stream)
                ok, msg, _ = O.check_implementation(_bits(x), _bits(w), _bits(y))
                same = np.array_equal(_bits(y[:, r0:r1]), _bits(mine))
                if code or not ok or not same:
                    good = False
                    msg = f"call {call}: device code {code}, oracle {ok} ({msg}), own slice bit-equal {same}"
                    break
            fg.close()
            out[(m, n, k)] = (good, msg)
    except Exception as e:  # reported through the results dict
        out["error"] = (False, repr(e))
    finally:
        results[rank] = out
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gather_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True, start_method="spawn")
    for rank in range(world):
        assert results[rank], f"rank {rank} reported nothing"
        for shape, (ok, msg) in results[rank].items():
            assert ok, f"rank {rank} {shape}: {msg}"
