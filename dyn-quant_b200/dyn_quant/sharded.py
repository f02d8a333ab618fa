"""Row-sharded split GEMV across the GPUs of one node.

The rows (d_out) of a dynamic-precision GEMV are independent, so P ranks each
hold a contiguous slice of the rows, run the fused split GEMV on their slice
with the full, replicated activation vector, and exchange only the output
slices.  The cheap statistics and the outlier mask are recomputed on every
rank from the same x, with a reduction order that does not depend on the
slice, so every rank applies the same mask.  The exchange is either

  "nccl": one NCCL all-gather over NVLink after the GEMV, or
  "peer": fused into the GEMV kernel (dq_split_gemv_gather): every output
          row also goes straight into every other rank's gather region as
          one 32-bit word (the FP16 value and the call's 16-bit tag), and
          each CTA copies the same rows of the other ranks' slices from its
          own region into y once their words carry the call's tag (bounded
          waits): one kernel per call, no fences, and no rank reads another's
          memory.

One process per GPU (torch.distributed for the plumbing).  The partition and
the NCCL gather are plain functions so that their logic can be exercised on
CPU ranks (gloo) with any local GEMV.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, List, Tuple

import torch
import torch.distributed as dist

from dyn_quant import DynQuantLinear, _lib

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
                out: torch.Tensor | None = None, pad: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather the ranks' output slices into y [d_out] (y_local: this rank's
    rows, at most rows_per of them).  out ([world * rows_per]) and pad
    ([rows_per], for a slice shorter than rows_per; its tail must be zero)
    are preallocated buffers; without them the call allocates its own."""
    world = dist.get_world_size(group)
    if y_local.numel() > rows_per:
        raise ValueError("local slice taller than the padded slice")
    if y_local.numel() < rows_per:
        if pad is None or pad.numel() != rows_per:
            pad = torch.zeros(rows_per, dtype=y_local.dtype, device=y_local.device)
        pad[: y_local.numel()].copy_(y_local.reshape(-1))
        y_local = pad
    full = out if out is not None and out.numel() == world * rows_per else torch.empty(
        world * rows_per, dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(full, y_local.contiguous(), group=group)
    return full[:d_out]


class _DeviceBytes:
    """A raw device allocation seen by torch (no copy, no ownership)."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


class PeerGather:
    """The gather regions of one row-sharded weight matrix, mapped on every rank.

    Each rank allocates its region (dq_device_alloc) and zero-fills it; the
    64-byte CUDA IPC handles are exchanged over the process group and every
    rank maps the others' regions (plain peer access, no multicast).  All
    ranks construct it together (collective), and must then make the same
    calls in the same order."""

    def __init__(self, rows_per: int, d_total: int, group=None, device=None) -> None:
        L = _lib.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_GATHER_RANKS:
            raise ValueError(f"at most {_lib.MAX_GATHER_RANKS} ranks")
        nbytes = L.dq_gather_region_bytes(rows_per)
        if nbytes == 0:
            raise ValueError(f"bad slice height {rows_per}")
        own = C.c_void_p()
        _lib.check(L.dq_device_alloc(nbytes, C.byref(own)), "dq_device_alloc")
        self._own = own.value
        self._opened: List[int] = []
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        torch.as_tensor(_DeviceBytes(self._own, nbytes), device=dev).zero_()
        handle = C.create_string_buffer(64)
        _lib.check(L.dq_ipc_handle(C.c_void_p(self._own), handle), "dq_ipc_handle")
        handles: List[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        regions = []
        for q, h in enumerate(handles):
            if q == self.rank:
                regions.append(self._own)
                continue
            p = C.c_void_p()
            _lib.check(L.dq_ipc_open(h, C.byref(p)), "dq_ipc_open")
            self._opened.append(p.value)
            regions.append(p.value)
        region = (C.c_void_p * _lib.MAX_GATHER_RANKS)(*(regions + [None] * (_lib.MAX_GATHER_RANKS - self.world)))
        self.desc = _lib.DqGather(self.rank, self.world, rows_per, d_total, region)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)  # every region zeroed and mapped before any rank calls

    def close(self) -> None:
        """Unmap the peers' regions and free this one (collective: after every
        rank's last call)."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        L = _lib.lib()
        for p in self._opened:
            _lib.check(L.dq_ipc_close(C.c_void_p(p)), "dq_ipc_close")
        self._opened = []
        dist.barrier(group=self.group)
        _lib.check(L.dq_device_free(C.c_void_p(self._own)), "dq_device_free")
        self._own = None


class ShardedDynQuantLinear(torch.nn.Module):
    """DynQuantLinear with its rows split over the ranks of `group`.

    load_weight() takes the full [d_out, d_in] FP16 weight (every rank passes
    the same matrix, or at least the rank's rows) and keeps this rank's slice;
    forward(x) returns the full y [d_out] on every rank.  gather: "nccl" (an
    all-gather after the GEMV) or "peer" (gathered inside the GEMV kernel; the
    last ranks' slices are zero-padded to the common height, and close() ends
    the module's use collectively).
    """

    def __init__(self, d_in: int, d_out: int, outlier_k: float = 3.0, group=None,
                 local_gemv: Callable[[torch.Tensor], torch.Tensor] | None = None, gather: str = "nccl") -> None:
        super().__init__()
        if gather not in ("nccl", "peer"):
            raise ValueError(f"gather must be 'nccl' or 'peer', not {gather!r}")
        self.d_in, self.d_out, self.outlier_k, self.group, self.gather = d_in, d_out, outlier_k, group, gather
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.r0, self.r1, self.rows_per = shard_rows(d_out, self.world, self.rank)
        if gather == "peer":
            self.local = DynQuantLinear(d_in, self.rows_per, outlier_k)
        else:
            self.local = DynQuantLinear(d_in, max(self.r1 - self.r0, 0), outlier_k) if self.r1 > self.r0 else None
        self._local_gemv = local_gemv  # test hook: a local GEMV other than the kernel
        self._gather_buf = None
        self._pad_buf = None
        self._peer: PeerGather | None = None
        self._ws = None

    def load_weight(self, weight: torch.Tensor) -> None:
        if weight.shape != (self.d_out, self.d_in):
            raise ValueError(f"expected weight ({self.d_out}, {self.d_in}), got {tuple(weight.shape)}")
        if self.gather == "peer":
            rows = torch.zeros(self.rows_per, self.d_in, dtype=weight.dtype, device=weight.device)
            rows[: self.r1 - self.r0] = weight[self.r0:self.r1]
            self.local.load_weight(rows)
        elif self.local is not None:
            self.local.load_weight(weight[self.r0:self.r1].contiguous())

    def _forward_peer(self, x: torch.Tensor) -> torch.Tensor:
        L = _lib.lib()
        if self._peer is None:
            self._peer = PeerGather(self.rows_per, self.d_out, self.group, x.device)
            self._ws = torch.zeros(L.dq_workspace_bytes(self.rows_per, self.d_in), dtype=torch.uint8,
                                   device=x.device)
        lin = self.local
        x = x.reshape(-1).to(torch.float16).contiguous()
        y = torch.empty(self.d_out, dtype=torch.float16, device=x.device)
        w = _lib.weights(lin.packed.data_ptr(), lin.scales.data_ptr(), lin.zeros.data_ptr(), None,
                         lin.fp16_w.data_ptr(), lin.d_out, lin.d_in, lin._native.data_ptr())
        _lib.check(L.dq_split_gemv_gather(C.byref(w), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                          float(self.outlier_k), C.c_void_p(self._ws.data_ptr()), self._ws.numel(),
                                          C.byref(self._peer.desc),
                                          C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)),
                   "dq_split_gemv_gather")
        return y

    def close(self) -> None:
        """End a "peer" module's use on every rank (collective)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.gather == "peer" and self._local_gemv is None:
            return self._forward_peer(x)
        if self._local_gemv is not None:
            y_local = self._local_gemv(x)
        elif self.local is not None:
            y_local = self.local(x)
        else:
            y_local = torch.empty(0, dtype=torch.float16, device=x.device)
        if self._gather_buf is None or self._gather_buf.device != x.device:
            self._gather_buf = torch.empty(self.world * self.rows_per, dtype=torch.float16, device=x.device)
            self._pad_buf = torch.zeros(self.rows_per, dtype=torch.float16, device=x.device)
        return gather_rows(y_local.to(torch.float16), self.d_out, self.rows_per, self.group, self._gather_buf,
                           self._pad_buf)
