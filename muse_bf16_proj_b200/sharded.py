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
            self._project = lambda x, out=None: project_fn(x, self.shard)

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

