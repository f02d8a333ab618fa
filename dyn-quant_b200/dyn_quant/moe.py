"""Mixture-of-experts FFN decode step on the dynamic-precision split GEMV.

Mixtral-style experts, y = w2 (silu(w1 x) * (w3 x)), top-k routing: each
(token, expert) pair is the reference's split GEMV of that token through the
expert's three matrices, each vector with its own statistics and outlier mask.
Here the tokens routed to one expert go through the batched split GEMV
together (the expert's weights stream once for all of them).  w1 and w3 read
the same x, so they are stacked into one [2 d_ff, d_model] matrix: one call,
one plan of the tokens' outliers, and each row's result is the split GEMV of
that row of w1 or w3.  The gated activation is one kernel on the stacked
output (dq_silu_mul_pairs) and the weighted outputs are added into an FP32
buffer (dq_moe_combine).  With the experts spread over the ranks
of a process group, every rank runs its own experts on the tokens routed to
them and the partial outputs are summed with one all-reduce.

Routing (which experts, with which weights) is fixed per step by a
``MoERouting`` built on the host, so a step issues kernel launches only and
can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Dict, Iterable, List, Sequence

import torch
import torch.distributed as dist

from dyn_quant import DynQuantLinear, _lib


class MoERouting:
    """Per-expert token lists of a top-k routing.

    experts: [T, k] expert index of each token's choices; weights: [T, k]
    combine weights.  Built once on the host; ``tokens[e]`` (int32) and
    ``weight[e]`` (float32) are the rows routed to expert e and their weights
    (a token lists an expert at most once)."""

    def __init__(self, experts: torch.Tensor, weights: torch.Tensor, n_experts: int,
                 device: torch.device | str | None = None) -> None:
        ex = experts.detach().cpu().long()
        wt = weights.detach().cpu().float()
        if ex.shape != wt.shape or ex.dim() != 2:
            raise ValueError("experts and weights must both be [tokens, k]")
        if ex.numel() and (ex.min() < 0 or ex.max() >= n_experts):
            raise ValueError("expert index out of range")
        self.n_tokens, self.k = ex.shape
        self.n_experts = n_experts
        dev = torch.device(device) if device is not None else experts.device
        self.tokens: Dict[int, torch.Tensor] = {}
        self.tokens64: Dict[int, torch.Tensor] = {}
        self.weight: Dict[int, torch.Tensor] = {}
        for e in range(n_experts):
            rows, slots = (ex == e).nonzero(as_tuple=True)
            if len(set(rows.tolist())) != len(rows):
                raise ValueError(f"a token selects expert {e} twice")
            if rows.numel():
                self.tokens[e] = rows.to(torch.int32).to(dev)
                self.tokens64[e] = rows.to(dev)
                self.weight[e] = wt[rows, slots].contiguous().to(dev)

    def count(self, e: int) -> int:
        t = self.tokens.get(e)
        return 0 if t is None else int(t.numel())

    def stacked(self, experts: Sequence[int]):
        """The rows routed to the given experts, one expert after another:
        (token indices int64 on the device, per-expert counts).  Cached per
        expert list, so a CUDA graph captured after the first call reuses it."""
        key = tuple(experts)
        hit = self.__dict__.setdefault("_stacked", {}).get(key)
        if hit is None:
            rows = torch.cat([self.tokens64[e] for e in experts]) if experts else None
            hit = (rows, [self.count(e) for e in experts])
            self._stacked[key] = hit
        return hit


def silu_mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp16(silu(a) * b), silu(v) = v / (1 + exp(-v)) in FP32 (dq_silu_mul)."""
    if a.shape != b.shape or a.dtype != torch.float16 or b.dtype != torch.float16:
        raise RuntimeError("silu_mul takes two float16 tensors of one shape")
    a, b = a.contiguous(), b.contiguous()
    h = torch.empty_like(a)
    _lib.check(_lib.lib().dq_silu_mul(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(h.data_ptr()),
                                      a.numel(), C.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)),
               "dq_silu_mul")
    return h


def silu_mul_pairs(ab: torch.Tensor) -> torch.Tensor:
    """[rows, 2d] float16 (w1 x | w3 x per row) -> fp16(silu(first half) *
    second half), [rows, d] (dq_silu_mul_pairs)."""
    if ab.dtype != torch.float16 or ab.dim() != 2 or ab.shape[1] % 16 != 0:
        raise RuntimeError("silu_mul_pairs takes a [rows, 2d] float16 tensor, d a multiple of 8")
    ab = ab.contiguous()
    d = ab.shape[1] // 2
    h = torch.empty(ab.shape[0], d, dtype=torch.float16, device=ab.device)
    _lib.check(_lib.lib().dq_silu_mul_pairs(C.c_void_p(ab.data_ptr()), C.c_void_p(h.data_ptr()), ab.shape[0], d,
                                            C.c_void_p(torch.cuda.current_stream(ab.device).cuda_stream)),
               "dq_silu_mul_pairs")
    return h


def combine_(out: torch.Tensor, y: torch.Tensor, rows: torch.Tensor, weight: torch.Tensor) -> None:
    """out[rows[i]] += weight[i] * y[i] in place (out float32 [T, d], y float16 [m, d])."""
    if y.numel() == 0:
        return
    y = y.contiguous()
    _lib.check(_lib.lib().dq_moe_combine(C.c_void_p(y.data_ptr()), C.c_void_p(rows.data_ptr()),
                                         C.c_void_p(weight.data_ptr()), C.c_void_p(out.data_ptr()),
                                         int(y.shape[0]), int(y.shape[1]),
                                         C.c_void_p(torch.cuda.current_stream(out.device).cuda_stream)),
               "dq_moe_combine")


class MoEFFN(torch.nn.Module):
    """The experts of one MoE FFN layer, or this rank's share of them.

    experts: the expert indices held here (default: all).  load_expert(e, w1,
    w3, w2) quantizes expert e's FP16 matrices ([d_ff, d_model], [d_ff,
    d_model], [d_model, d_ff]), w1 and w3 stacked as w13[e] ([2 d_ff,
    d_model]: rows 0 .. d_ff-1 are w1's, the rest w3's); forward(x, routing,
    group) returns the combined output [T, d_model] (float16) on every rank of
    group (the sum over the ranks' experts)."""

    def __init__(self, n_experts: int, d_model: int, d_ff: int, outlier_k: float = 3.0,
                 experts: Iterable[int] | None = None) -> None:
        super().__init__()
        self.n_experts, self.d_model, self.d_ff, self.outlier_k = n_experts, d_model, d_ff, outlier_k
        self.local: List[int] = sorted(experts) if experts is not None else list(range(n_experts))
        self.w13 = torch.nn.ModuleDict({str(e): DynQuantLinear(d_model, 2 * d_ff, outlier_k) for e in self.local})
        self.w2 = torch.nn.ModuleDict({str(e): DynQuantLinear(d_ff, d_model, outlier_k) for e in self.local})

    def load_expert(self, e: int, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor) -> None:
        self.w13[str(e)].load_weight(torch.cat([w1, w3]).contiguous())
        self.w2[str(e)].load_weight(w2)

    def gate_up(self, e: int, x: torch.Tensor) -> torch.Tensor:
        """[w1 x | w3 x] of the rows of x ([m, d_model] -> [m, 2 d_ff], float16)."""
        return self.w13[str(e)](x).reshape(x.shape[0], -1)

    def expert(self, e: int, x: torch.Tensor) -> torch.Tensor:
        """The expert's FFN on the rows of x ([m, d_model] -> [m, d_model], float16)."""
        return self.w2[str(e)](silu_mul_pairs(self.gate_up(e, x)))

    def forward(self, x: torch.Tensor, routing: MoERouting, group=None, out: torch.Tensor | None = None
                ) -> torch.Tensor:
        """Combined output [T, d_model] float16.  When this module holds only
        some of the experts, the ranks of group (default: the default group)
        hold the others and the partial outputs are all-reduced."""
        if out is None:
            out = torch.zeros(x.shape[0], self.d_model, dtype=torch.float32, device=x.device)
        else:
            out.zero_()
        reduce = len(self.local) < self.n_experts
        if x.is_cuda and self._grouped(x, routing, out):
            if reduce:
                dist.all_reduce(out, group=group)
            return out.to(torch.float16)
        return moe_forward(x, routing, self.local, self.expert, out, reduce, group).to(torch.float16)

    def _grouped(self, x: torch.Tensor, routing: MoERouting, out: torch.Tensor) -> bool:
        """The local experts' step with grouped batched calls: one call for
        every expert's w13 on its tokens, one gated activation over all rows,
        one call for every w2, then the combine expert by expert (the order of
        moe_forward, so out gets the same additions in the same order).
        Returns False (nothing done) where the grouped call does not apply:
        more than 16 experts here, or more than 16 tokens on one expert."""
        es = [e for e in self.local if routing.count(e) > 0]
        if not es or len(es) > _lib.MAX_GROUPS or any(routing.count(e) > _lib.MAX_BATCH for e in es):
            return len(es) == 0
        if x.dtype != torch.float16:
            x = x.to(torch.float16)
        rows, counts = routing.stacked(es)
        xg = x.index_select(0, rows).contiguous()
        n = xg.shape[0]
        D, F = self.d_model, self.d_ff
        h13 = torch.empty(n, 2 * F, dtype=torch.float16, device=x.device)
        y2 = torch.empty(n, D, dtype=torch.float16, device=x.device)
        ws = self._workspace(x.device, max(counts), len(es))
        stream = torch.cuda.current_stream(x.device).cuda_stream
        offs = [0]
        for c in counts:
            offs.append(offs[-1] + c)
        for layers, src, dst, d_src, d_dst in ((self.w13, xg, h13, D, 2 * F), (self.w2, None, y2, F, D)):
            if src is None:
                src = silu_mul_pairs(h13)
            st = _lib.batched_grouped([_weights_of(layers[str(e)]) for e in es],
                                      [src.data_ptr() + 2 * d_src * o for o in offs[:-1]],
                                      [dst.data_ptr() + 2 * d_dst * o for o in offs[:-1]], counts,
                                      self.outlier_k, ws.data_ptr(), ws.numel(), stream)
            _lib.check(st, "dq_split_gemv_batched_grouped")
        for i, e in enumerate(es):
            combine_(out, y2[offs[i]:offs[i + 1]], routing.tokens[e], routing.weight[e])
        return True

    def _workspace(self, device: torch.device, m_max: int, groups: int) -> torch.Tensor:
        L = _lib.lib()
        need = max(L.dq_workspace_bytes_batched_grouped(2 * self.d_ff, self.d_model, m_max, groups),
                   L.dq_workspace_bytes_batched_grouped(self.d_model, self.d_ff, m_max, groups))
        ws = self.__dict__.get("_ws")
        if ws is None or ws.device != device or ws.numel() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=device)
            self.__dict__["_ws"] = ws
        return ws


def _weights_of(lin: DynQuantLinear):
    """The dq_weights_t of a loaded DynQuantLinear (its FP16 weights are the
    row-major matrix or the transpose of the column-major mirror)."""
    f = lin.fp16_w
    d_out, d_in = f.shape
    cm = d_out > 1 and f.stride() == (1, d_out)
    return _lib.weights(lin.packed.data_ptr(), lin.scales.data_ptr(), lin.zeros.data_ptr(),
                        None if cm else f.data_ptr(), f.data_ptr() if cm else None, d_out, d_in,
                        lin._native.data_ptr())


def moe_forward(x: torch.Tensor, routing: MoERouting, local: Sequence[int],
                expert: Callable[[int, torch.Tensor], torch.Tensor], out: torch.Tensor, reduce: bool,
                group=None) -> torch.Tensor:
    """Run the local experts on their routed tokens and add their weighted
    outputs into out (float32 [T, d]), experts in the order of local; with
    reduce, sum out over the ranks of group.  expert(e, xe) is expert e's FFN
    on the rows xe."""
    if x.dtype != torch.float16:
        x = x.to(torch.float16)
    for e in local:
        rows = routing.tokens.get(e)
        if rows is None:
            continue
        xe = x.index_select(0, routing.tokens64[e]).contiguous()
        ye = expert(e, xe).reshape(xe.shape[0], -1)
        if out.is_cuda:
            combine_(out, ye, rows, routing.weight[e])
        else:  # CPU ranks (tests of the distribution logic)
            out.index_add_(0, rows.long(), routing.weight[e][:, None] * ye.float())
    if reduce:
        dist.all_reduce(out, group=group)
    return out
