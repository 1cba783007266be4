"""Column-parallel (N-sharded) and row-parallel (K-sharded) projections across the GPUs of one node.

Rows of W are independent, so rank r of P holds W[r0:r1] (``shard_rows``), x is replicated and each
rank computes its slice y[:, r0:r1] with the single-GPU kernels. The only collective is the
optional all-gather of y, for callers that need the whole output: ``all_gather_into_tensor`` into a
rank-major [P, M, N/P] buffer (one NCCL call over NVLink), then one strided copy to [M, N].
A caller that can consume the rank-major layout skips the copy (``gather(..., rank_major=True)``).

No counterpart in the reference (its shapes are TP8 per-GPU slices and it runs no collective,
baseline.py:11); the layout follows the column-parallel split of the reference's qkv_gate
(reference.py:16).

Row-parallel (``RowParallelProjection``, the TP split of the reference's `o` projection,
reference.py:17): rank r holds W[:, r0:r1] and the matching columns of x, computes the FP32 partial
x[:, r0:r1] . W[:, r0:r1]^T (``muse_proj_bf16_tiles_f32``: no rounding before the sum), and one
reduce-scatter over NCCL sums the ranks' partials in FP32 and leaves rank r the columns
[r N/P, (r+1) N/P) of y, rounded to BF16 once (or an all-reduce for the whole y).
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """[r0, r1) of the N rows rank `rank` of `world` holds: equal shards, N % world == 0."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n % world:
        raise ValueError(f"N={n} does not split evenly across {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def gather_columns(y_local: torch.Tensor, world: int, group=None, rank_major: bool = False,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """All ranks' [M, N/P] slices -> [M, N] (or the rank-major [P, M, N/P] buffer)."""
    if world == 1:
        return y_local.unsqueeze(0) if rank_major else y_local
    m, npr = y_local.shape
    buf = torch.empty((world, m, npr), dtype=y_local.dtype, device=y_local.device)
    if y_local.is_cuda:
        dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    else:  # gloo: list form
        dist.all_gather(list(buf.unbind(0)), y_local.contiguous(), group=group)
    if rank_major:
        return buf
    full = out if out is not None else torch.empty((m, world * npr), dtype=y_local.dtype, device=y_local.device)
    full.view(m, world, npr).copy_(buf.permute(1, 0, 2))
    return full


class ShardedProjection:
    """One rank's part of y = x . W^T with W split along N.

    ``project(x)`` -> this rank's [M, N/P] slice (the single-GPU path: ``project_fn`` defaults to
    ``submission.project`` on the state built by ``prepare``). ``gather(y_local)`` -> the full
    [M, N] (or [P, M, N/P] with ``rank_major=True``)."""

    def __init__(self, w_full_or_shard: torch.Tensor, n_full: int, group=None, shard_given: bool = False,
                 project_fn: Callable | None = None, name: str = "w", **prepare_kw):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_full = n_full
        self.r0, self.r1 = shard_rows(n_full, self.world, self.rank)
        shard = w_full_or_shard if shard_given else w_full_or_shard[self.r0:self.r1]
        if shard.shape[0] != self.r1 - self.r0:
            raise ValueError(f"shard has {shard.shape[0]} rows, expected {self.r1 - self.r0}")
        self.name = name
        self.shard = shard.contiguous()
        if project_fn is None:
            from . import submission
            self.state = submission.prepare({name: self.shard}, **prepare_kw)
            self._project = lambda x, out=None: submission.project(x, self.state, name, out=out)
        else:
            self.state = None

            def _project(x, out=None):
                y = project_fn(x, self.shard)
                if out is None:
                    return y
                out.copy_(y)  # the caller's buffer holds the result, as on the kernel path
                return out

            self._project = _project

    def project(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._project(x, out)

    def gather(self, y_local: torch.Tensor, rank_major: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
        return gather_columns(y_local, self.world, self.group, rank_major, out)


def shard_k(k: int, world: int, rank: int) -> tuple[int, int]:
    """[k0, k1) of the K columns rank `rank` of `world` holds: equal shards, a multiple of 64 each."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if k % (64 * world):
        raise ValueError(f"K={k} does not split into {world} shards of a multiple of 64")
    per = k // world
    return rank * per, (rank + 1) * per


def reduce_columns(y_partial: torch.Tensor, world: int, group=None, scatter: bool = True) -> torch.Tensor:
    """The sum over ranks of FP32 [M, N] partials: rank r's columns [r N/P, (r+1) N/P) (scatter) or
    all of y, rounded to BF16 after the FP32 sum."""
    m, n = y_partial.shape
    if world == 1:
        return y_partial.to(torch.bfloat16)
    if n % world:
        raise ValueError(f"N={n} does not split across {world} ranks")
    if not scatter:
        dist.all_reduce(y_partial, group=group)
        return y_partial.to(torch.bfloat16)
    per = n // world
    rank_major = y_partial.view(m, world, per).permute(1, 0, 2).contiguous()  # [P, M, N/P]
    if y_partial.is_cuda:
        out = torch.empty((m, per), dtype=torch.float32, device=y_partial.device)
        dist.reduce_scatter_tensor(out, rank_major, group=group)
    else:  # gloo has no reduce-scatter: all-reduce, keep this rank's part
        dist.all_reduce(rank_major, group=group)
        out = rank_major[dist.get_rank(group)]
    return out.to(torch.bfloat16)


def _tile_plan_f32(m: int, n: int, k: int):
    """A tile-kernel plan for the FP32 partial: tokens per tile the power of two >= M (16..256), K
    split so the grid roughly covers the SMs."""
    from . import _lib
    bnt = 16
    while bnt < m and bnt < 256:
        bnt *= 2
    tiles = -(-n // 128) * -(-m // bnt)
    split = max(1, min(8, 148 // max(tiles, 1), k // 64))
    return _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=bnt, split=split, stages=6 if bnt <= 64 else 0,
                         flags=(_lib.FLAG_GLOBAL_SPLIT if split > 1 else 0) | _lib.FLAG_PDL)


class RowParallelProjection:
    """One rank's part of y = x . W^T with W split along K.

    ``partial(x)`` -> this rank's FP32 [M, N] partial (x full or already this rank's columns);
    ``reduce(y_partial)`` -> BF16 y[:, r N/P:(r+1) N/P] (or all of y with ``scatter=False``).
    ``project_fn(x_shard, w_shard) -> FP32`` replaces the GPU kernel (CPU tests)."""

    def __init__(self, w_full_or_shard: torch.Tensor, k_full: int, group=None, shard_given: bool = False,
                 project_fn: Callable | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.k_full = k_full
        self.k0, self.k1 = shard_k(k_full, self.world, self.rank)
        shard = w_full_or_shard if shard_given else w_full_or_shard[:, self.k0:self.k1]
        if shard.shape[1] != self.k1 - self.k0:
            raise ValueError(f"shard has {shard.shape[1]} columns, expected {self.k1 - self.k0}")
        self.shard = shard.contiguous()
        self.n = self.shard.shape[0]
        self.project_fn = project_fn
        self.tiles = None
        self.scratch = None
        if project_fn is None:
            from . import _lib
            n, k = self.shard.shape
            self.tiles = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device=self.shard.device)
            _lib.pack_tiles(self.shard.data_ptr(), self.tiles.data_ptr(), n, k,
                            torch.cuda.current_stream(self.shard.device).cuda_stream)
            self._plans: dict = {}

    def partial(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[1] == self.k_full and self.world > 1:
            x = x[:, self.k0:self.k1]
        x = x.contiguous()
        if self.project_fn is not None:
            return self.project_fn(x, self.shard)
        from . import _lib
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.shard.shape[1]:
            raise ValueError(f"x must be BF16 [M, {self.shard.shape[1]}] (this rank's K columns), got "
                             f"{x.dtype} {tuple(x.shape)}")
        if x.device != self.tiles.device:
            raise ValueError(f"x is on {x.device}, this rank's shard on {self.tiles.device}")
        m, k = x.shape
        plan = self._plans.get(m)
        if plan is None:
            plan = self._plans[m] = _tile_plan_f32(m, self.n, k)
        need = _lib.scratch_bytes(m, self.n, k, plan)
        if need and (self.scratch is None or self.scratch.numel() < need):
            self.scratch = torch.zeros(need, dtype=torch.uint8, device=x.device)
        y = torch.empty((m, self.n), dtype=torch.float32, device=x.device)
        _lib.proj_bf16_tiles_f32(x.data_ptr(), self.tiles.data_ptr(), y.data_ptr(), m, self.n, k, plan,
                                 torch.cuda.current_stream(x.device).cuda_stream,
                                 self.scratch.data_ptr() if need else 0, need)
        return y

    def reduce(self, y_partial: torch.Tensor, scatter: bool = True) -> torch.Tensor:
        return reduce_columns(y_partial, self.world, self.group, scatter)



def gather_plan(m: int, n_local: int, k: int, sms: int = 148):
    """Plan for the fused all-gather projection (``muse_proj_bf16_tiles_gather`` runs the tile
    kernel or the pair GEMM): above 256 tokens the pair GEMM; else 128-row W tiles x the smallest
    power-of-two token tile >= M (16 .. 128), K split through scratch. The split is the one whose
    grid wastes the least of its last wave (two CTAs an SM with the 6-stage ring of 16- and 32-token
    tiles), each extra split charged 10 % for its partial sums, pipeline fill and ticket (measured
    on B200 with the all-gather epilogue: 224 tiles at M = 1 run best unsplit, 32 tiles split 8 ways)."""
    from . import _lib as L
    p = L.MusePlan()
    if m > 256:
        p.kernel = L.KERNEL_TC_GEMM2
        return p
    tile_n = 16
    while tile_n < m and tile_n < 128:
        tile_n *= 2
    tiles = -(-n_local // 128) * -(-m // tile_n)
    nkb = -(-k // 64)
    per_sm = 2 if tile_n <= 32 else 1
    best, best_cost = 1, None
    for split in range(1, min(16, nkb) + 1):
        waves = -(-(tiles * split) // (sms * per_sm))
        cost = waves / split * (1 + 0.1 * (split - 1))
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = split, cost
    p.kernel = L.KERNEL_TC_TILE
    p.tile_n = tile_n
    p.stages = 6 if per_sm == 2 else 0
    p.split = best
    p.flags = L.FLAG_PDL | (L.FLAG_GLOBAL_SPLIT if best > 1 else 0)
    return p


def exchange_peer_entries(entry: dict, group=None) -> list[dict]:
    """Every rank's ``entry`` (IPC handles and offsets of its output and control block, its device
    and host), in rank order. Peers must be GPUs of one node: a host mismatch raises."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return [entry]
    out = [None] * world
    dist.all_gather_object(out, entry, group=group)
    hosts = {e["host"] for e in out}
    if len(hosts) != 1:
        raise RuntimeError(f"the fused all-gather needs every rank on one node (hosts {sorted(hosts)})")
    return out


class FusedGatherProjection:
    """Column-parallel projection whose all-gather is fused into the kernel's epilogue.

    Each rank holds W[r0:r1] (``shard_rows``) as packed tiles and owns y_full [max_rows, N] plus a
    small control block; the buffers are exchanged once as CUDA IPC handles. ``project(x)`` runs
    ``muse_proj_bf16_tiles_gather``: the kernel stores every output value of this rank's columns
    into all ranks' y_full over NVLink as it finishes them, so there is no NCCL step and no
    staging copy; it returns y_full[:M], complete on this rank's stream when the launch ends.
    The view is overwritten by the next call; every rank makes the same calls in the same order.
    """

    def __init__(self, w_full_or_shard: torch.Tensor, n_full: int, max_rows: int, group=None,
                 shard_given: bool = False):
        from . import _lib as L
        import socket
        self._L = L
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > L.MAX_PEERS:
            raise ValueError(f"the fused all-gather spans at most {L.MAX_PEERS} ranks (got {self.world})")
        self.n_full, self.max_rows = n_full, max_rows
        self.r0, self.r1 = shard_rows(n_full, self.world, self.rank)
        self.n = self.r1 - self.r0
        if self.n % 8:
            raise ValueError(f"each rank's {self.n} columns must be a multiple of 8")
        shard = w_full_or_shard if shard_given else w_full_or_shard[self.r0:self.r1]
        if shard.dtype != torch.bfloat16 or not shard.is_cuda or shard.shape[0] != self.n:
            raise ValueError(f"need a BF16 CUDA shard of {self.n} rows (got {shard.dtype}, {tuple(shard.shape)})")
        self.k = shard.shape[1]
        dev = shard.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        shard = shard.contiguous()
        self.tiles = torch.empty(L.tiles_bytes(self.n, self.k), dtype=torch.uint8, device=dev)
        L.pack_tiles(shard.data_ptr(), self.tiles.data_ptr(), self.n, self.k, stream)
        self.y_full = torch.empty((max_rows, n_full), dtype=torch.bfloat16, device=dev)
        self.ctl = torch.zeros(L.peer_ctl_bytes(), dtype=torch.uint8, device=dev)
        self._scratch = torch.zeros(0, dtype=torch.uint8, device=dev)
        self._plans = {}  # M -> (plan, scratch bytes)
        torch.cuda.synchronize(dev)  # buffers zeroed and W packed before any peer can see them
        yh, yo = L.ipc_export(self.y_full.data_ptr())
        ch, co = L.ipc_export(self.ctl.data_ptr())
        entries = exchange_peer_entries({"y": (yh, yo), "ctl": (ch, co), "rank": self.rank,
                                         "host": socket.gethostname()}, group)
        self._opened = []  # (pointer, offset) of peers' buffers opened here
        g = L.MuseGather()
        g.world, g.rank, g.ldy, g.col0 = self.world, self.rank, n_full, self.r0
        try:
            for p, e in enumerate(entries):
                if p == self.rank:
                    g.y[p], g.ctl[p] = self.y_full.data_ptr(), self.ctl.data_ptr()
                    continue
                for field in ("y", "ctl"):
                    ptr = L.ipc_open(*e[field])
                    self._opened.append((ptr, e[field][1]))
                    if field == "y":
                        g.y[p] = ptr
                    else:
                        g.ctl[p] = ptr
        except Exception:
            self._close_opened()
            raise
        self.gather = g
        self._barrier()  # every rank's peers are open before anyone's first call

    def _barrier(self):
        if self.world > 1:
            dist.barrier(group=self.group)

    def _close_opened(self):
        while self._opened:
            ptr, off = self._opened.pop()
            self._L.ipc_close(ptr, off)

    def plan(self, m: int):
        return gather_plan(m, self.n, self.k, self._L.sm_count())

    def project(self, x: torch.Tensor, plan=None, tiles: torch.Tensor | None = None) -> torch.Tensor:
        """y_full[:M] after x . W^T with every rank's columns. `tiles`: packed tiles of another W
        shard of the same shape (muse_pack_tiles) to use instead of this one's."""
        L = self._L
        if tiles is None:
            tiles = self.tiles
        elif tiles.numel() * tiles.element_size() != self.tiles.numel() or tiles.device != self.tiles.device:
            raise ValueError("tiles must be a packed shard of the same shape on the same device")
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.k or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous BF16 [M, {self.k}] tensor")
        if x.device != self.tiles.device:
            raise ValueError(f"x is on {x.device}, this rank's shard on {self.tiles.device}")
        m = x.shape[0]
        if not 0 < m <= self.max_rows:
            raise ValueError(f"M={m} outside 1..{self.max_rows} (the y_full buffer's rows)")
        if not self._opened and self.world > 1:
            raise RuntimeError("closed")
        if plan is None:
            cached = self._plans.get(m)
            if cached is None:
                p = self.plan(m)
                cached = self._plans[m] = (p, L.scratch_bytes(m, self.n, self.k, p))
            plan, need = cached
        else:
            need = L.scratch_bytes(m, self.n, self.k, plan)
        if need > self._scratch.numel():
            self._scratch = torch.zeros(need, dtype=torch.uint8, device=x.device)
        L.proj_bf16_tiles_gather(x.data_ptr(), tiles.data_ptr(), m, self.n, self.k, self.gather, plan,
                                 torch.cuda.current_stream(x.device).cuda_stream,
                                 self._scratch.data_ptr() if need else 0, need)
        return self.y_full[:m]

    def close(self):
        """Unmaps the peers' buffers (after every rank's work on them has finished)."""
        torch.cuda.synchronize(self.y_full.device)
        self._barrier()
        self._close_opened()
        self._barrier()  # no rank frees its buffers while a peer still maps them
