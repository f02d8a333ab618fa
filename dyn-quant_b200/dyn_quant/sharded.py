"""Row-sharded split GEMV across the GPUs of one node.

The rows (d_out) of a dynamic-precision GEMV are independent, so P ranks each
hold a contiguous slice of the rows, run the fused split GEMV on their slice
with the full, replicated activation vector, and exchange only the output
slices.  The exchange is one NCCL all-gather over NVLink: the cheap statistics
and the outlier mask are recomputed on every rank from the same x, with a
reduction order that does not depend on the slice, so every rank applies the
same mask.

One process per GPU (torch.distributed with the "nccl" backend for the
plumbing).  The partition and the gather are plain functions so that their
logic can be exercised on CPU ranks (gloo) with any local GEMV.
"""
from __future__ import annotations

from typing import Callable, Tuple

import torch
import torch.distributed as dist

from dyn_quant import DynQuantLinear

ROW_BLOCK = 16  # rows per MMA row block: slices are whole row blocks


def shard_rows(d_out: int, world: int, rank: int) -> Tuple[int, int, int]:
    """Rows [r0, r1) of `rank` and the padded slice height (equal on every rank).

    Slices are whole 16-row blocks; the last ranks may hold fewer (or no) real
    rows, and every slice is padded to the same height for the all-gather."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    blocks = (d_out + ROW_BLOCK - 1) // ROW_BLOCK
    per = (blocks + world - 1) // world
    rows_per = per * ROW_BLOCK
    r0 = min(d_out, rank * rows_per)
    r1 = min(d_out, r0 + rows_per)
    return r0, r1, rows_per


def gather_rows(y_local: torch.Tensor, d_out: int, rows_per: int, group=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather the ranks' output slices into y [d_out] (y_local: this rank's
    rows, at most rows_per of them)."""
    world = dist.get_world_size(group)
    if y_local.numel() > rows_per:
        raise ValueError("local slice taller than the padded slice")
    if y_local.numel() < rows_per:
        pad = torch.zeros(rows_per, dtype=y_local.dtype, device=y_local.device)
        pad[: y_local.numel()] = y_local
        y_local = pad
    full = out if out is not None and out.numel() == world * rows_per else torch.empty(
        world * rows_per, dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(full, y_local.contiguous(), group=group)
    return full[:d_out]


class ShardedDynQuantLinear(torch.nn.Module):
    """DynQuantLinear with its rows split over the ranks of `group`.

    load_weight() takes the full [d_out, d_in] FP16 weight (every rank passes
    the same matrix, or at least the rank's rows) and keeps this rank's slice;
    forward(x) returns the full y [d_out] on every rank.
    """

    def __init__(self, d_in: int, d_out: int, outlier_k: float = 3.0, group=None,
                 local_gemv: Callable[[torch.Tensor], torch.Tensor] | None = None) -> None:
        super().__init__()
        self.d_in, self.d_out, self.outlier_k, self.group = d_in, d_out, outlier_k, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.r0, self.r1, self.rows_per = shard_rows(d_out, self.world, self.rank)
        self.local = DynQuantLinear(d_in, max(self.r1 - self.r0, 0), outlier_k) if self.r1 > self.r0 else None
        self._local_gemv = local_gemv  # test hook: a local GEMV other than the kernel
        self._gather_buf = None

    def load_weight(self, weight: torch.Tensor) -> None:
        if weight.shape != (self.d_out, self.d_in):
            raise ValueError(f"expected weight ({self.d_out}, {self.d_in}), got {tuple(weight.shape)}")
        if self.local is not None:
            self.local.load_weight(weight[self.r0:self.r1].contiguous())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._local_gemv is not None:
            y_local = self._local_gemv(x)
        elif self.local is not None:
            y_local = self.local(x)
        else:
            y_local = torch.empty(0, dtype=torch.float16, device=x.device)
        if self._gather_buf is None or self._gather_buf.device != x.device:
            self._gather_buf = torch.empty(self.world * self.rows_per, dtype=torch.float16, device=x.device)
        return gather_rows(y_local.to(torch.float16), self.d_out, self.rows_per, self.group, self._gather_buf)
