"""Column-parallel (N-sharded) projection across the GPUs of one node.

Rows of W are independent, so rank r of P holds W[r0:r1] (``shard_rows``), x is replicated and each
rank computes its slice y[:, r0:r1] with the single-GPU kernels. The only collective is the
optional all-gather of y, for callers that need the whole output: ``all_gather_into_tensor`` into a
rank-major [P, M, N/P] buffer (one NCCL call over NVLink), then one strided copy to [M, N].
A caller that can consume the rank-major layout skips the copy (``gather(..., rank_major=True)``).

No counterpart in the reference (its shapes are TP8 per-GPU slices and it runs no collective,
baseline.py:11); the layout follows the column-parallel split of the reference's qkv_gate
(reference.py:16).
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
