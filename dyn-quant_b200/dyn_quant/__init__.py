"""dyn_quant: fused dynamic-precision W4A16 GEMV for NVIDIA B200 (sm_100a).

Drop-in for the reference package of the same name (dyn-quant,
dyn_quant/__init__.py:1-179): the same functions, the same DynQuantLinear
module, the same argument meaning and the same RuntimeError behaviour, over
hand-written sm_100a kernels (libdq_b200.so, C ABI in include/dq_abi.h).

Exports:
  DynQuantLinear   nn.Module: load_weight() quantizes on the GPU; forward()
                   runs the fused split-precision GEMV.
  quantize()       FP16 weight -> (packed INT4, scales, zeros, fp16 copy).
  split_gemv()     fused dynamic-precision GEMV (functional API).
  int4_gemv()      dense INT4 GEMV baseline.
  reference_gemv() FP16 dense GEMV.
  detect_outliers() the detector the split GEMV applies, standalone.

There is no CPU path: every function raises if the extension is not built.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn

try:
    from dyn_quant import _C  # noqa: F401

    _EXTENSION_LOADED = True
    _IMPORT_ERROR: Exception | None = None
except ImportError as e:  # pragma: no cover - exercised only without a build
    _EXTENSION_LOADED = False
    _IMPORT_ERROR = e

__all__ = [
    "DynQuantLinear",
    "quantize",
    "split_gemv",
    "int4_gemv",
    "reference_gemv",
    "detect_outliers",
    "build_colmajor",
    "build_native",
]

GROUP_SIZE = 128


def _require_extension() -> None:
    """dyn_quant/__init__.py:26-31 of the reference: fail loudly without the extension."""
    if not _EXTENSION_LOADED:
        raise RuntimeError(
            "dyn_quant C extension not found. Build it with: python dyn-quant_b200/build.py"
            + (f" ({_IMPORT_ERROR})" if _IMPORT_ERROR else ""))


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The kernels read x with 16-byte loads; re-home a misaligned view."""
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def quantize(weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Quantize an FP16 weight matrix to packed INT4 format (on the GPU, bit-exact
    with the reference's host quantizer, src/quant_format.cuh:58-97).

    Args:
        weight: [d_out, d_in] float16 tensor on CUDA.

    Returns:
        (packed, scales, zeros, fp16_copy):
          packed    [d_out, d_in//2] uint8, two INT4 values per byte (even column low nibble)
          scales    [d_out, d_in//128] float16, per-group scale
          zeros     [d_out, d_in//128] float16, per-group zero-point
          fp16_copy [d_out, d_in] float16, original weights for outlier columns
    """
    _require_extension()
    if weight.dtype != torch.float16:
        weight = weight.to(torch.float16)
    if not weight.is_contiguous():
        weight = weight.contiguous()
    return _C.quantize_weights(_aligned(weight))


def build_colmajor(weight: torch.Tensor) -> torch.Tensor:
    """Column-major FP16 mirror [d_in, d_out] of a [d_out, d_in] weight.

    Its transpose (``mirror.t()``) is a [d_out, d_in] view that split_gemv accepts
    as ``fp16_w`` and uses for coalesced outlier-column reads."""
    _require_extension()
    if weight.dtype != torch.float16:
        weight = weight.to(torch.float16)
    if not weight.is_contiguous():
        weight = weight.contiguous()
    return _C.build_colmajor(_aligned(weight))


def split_gemv(
    packed: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    fp16_w: torch.Tensor,
    x: torch.Tensor,
    outlier_k: float = 3.0,
    native: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused dynamic-precision GEMV with runtime outlier detection.

    Outlier channels (|x_i - mean| > outlier_k * std) use the FP16 weight
    columns; the rest use INT4 dequantization; one FP32 accumulation, one FP16
    write, one kernel launch.

    Args:
        packed:    [d_out, d_in//2] uint8 packed INT4 weights.
        scales:    [d_out, d_in//128] float16 per-group scales.
        zeros:     [d_out, d_in//128] float16 per-group zero-points.
        fp16_w:    [d_out, d_in] float16 original weights: contiguous, or the
                   transpose of a column-major mirror (see build_colmajor).
        x:         [d_in] float16 activation vector, or [m, d_in] for m
                   vectors at once (each with its own outlier mask; the
                   reference accepts one vector only).
        outlier_k: sigma threshold for outlier detection (default 3.0).
        native:    optional unit layout from build_native(packed, scales,
                   zeros) -- the fast path (one bulk copy per unit).  Built
                   here when a batch of vectors is given without it.

    Returns:
        y: [d_out] float16 output vector ([m, d_out] for a batch).
    """
    _require_extension()
    if x.dim() == 2 and x.numel() != fp16_w.shape[1]:
        return _split_gemv_rows(packed, scales, zeros, fp16_w, x, outlier_k, native)
    return _C.split_gemv(packed, scales, zeros, fp16_w, _aligned(x), float(outlier_k), native)


MAX_BATCH = 16  # vectors per batched kernel call


def _split_gemv_rows(packed, scales, zeros, fp16_w, x, outlier_k, native):
    """Rows of x [m, d_in] through the batched kernel, up to 16 rows per call."""
    if x.dtype != torch.float16:
        x = x.to(torch.float16)
    x = x.contiguous()
    if x.shape[1] != fp16_w.shape[1]:
        raise RuntimeError(f"x must be [m, d_in] with d_in={fp16_w.shape[1]}, got {tuple(x.shape)}")
    if x.shape[0] == 0:
        return x.new_empty((0, fp16_w.shape[0]))
    if native is None:
        native = _C.build_native(packed, scales, zeros)
    outs = [_C.split_gemv_batched(packed, scales, zeros, fp16_w, _aligned(x[i:i + MAX_BATCH].contiguous()),
                                  float(outlier_k), native)
            for i in range(0, x.shape[0], MAX_BATCH)]
    return outs[0] if len(outs) == 1 else torch.cat(outs)


def int4_gemv(
    packed: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    fp16_w: torch.Tensor,
    x: torch.Tensor,
    native: torch.Tensor | None = None,
) -> torch.Tensor:
    """Dense INT4 GEMV without outlier handling (fp16_w used only for shape)."""
    _require_extension()
    return _C.int4_gemv(packed, scales, zeros, fp16_w, _aligned(x), native)


def build_native(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor) -> torch.Tensor:
    """The unit layout the GEMV kernels stream with one bulk copy per 16-row x
    512-column unit: packed codes in lane order plus interleaved (scale, zero),
    a reordering of (packed, scales, zeros) (a uint8 tensor)."""
    _require_extension()
    return _C.build_native(packed, scales, zeros)


def reference_gemv(fp16_w: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """FP16 dense GEMV with FP32 accumulation: y = fp16_w @ x."""
    _require_extension()
    return _C.reference_gemv(_aligned(fp16_w), _aligned(x))


def detect_outliers(x: torch.Tensor, outlier_k: float = 3.0):
    """The outlier detector the split GEMV applies, standalone.

    Returns (mask, indices, stats): mask [d_in] bool, indices int32 in the
    reference's list order (stripe class (c//32)%4 == 0 ascending, then 1, 2, 3),
    stats float32 [mean, threshold, unbiased variance, M2].  Synchronises to
    read the count."""
    _require_extension()
    if x.dtype != torch.float16:
        x = x.to(torch.float16)
    x = _aligned(x.contiguous().reshape(-1))
    words, idx, cnt, stats = _C.detect_outliers(x, float(outlier_k))
    n = int(cnt.item())
    bits = (words.view(-1, 1) >> torch.arange(32, device=x.device, dtype=torch.int32)) & 1
    return bits.reshape(-1).bool(), idx[:n], stats


class DynQuantLinear(nn.Module):
    """Linear layer using the fused INT4/FP16 split-precision GEMV.

    load_weight() quantizes the weights on the GPU and builds the column-major
    FP16 mirror used for outlier columns; forward() detects outlier channels of
    x at run time (no calibration) and runs one fused kernel.

    ``fp16_w`` is the [d_out, d_in] transpose view of the column-major mirror:
    same shape and values as the reference's row-major copy, one copy in memory.

    Args:
        d_in:      Input feature dimension.
        d_out:     Output feature dimension.
        outlier_k: Sigma threshold for outlier detection (default 3.0).
    """

    def __init__(self, d_in: int, d_out: int, outlier_k: float = 3.0) -> None:
        super().__init__()
        self.d_in = d_in
        self.d_out = d_out
        self.outlier_k = outlier_k
        self._quantized = False
        self.register_buffer("packed", None)
        self.register_buffer("scales", None)
        self.register_buffer("zeros", None)
        self.register_buffer("fp16_w", None)
        # load-time unit layout the kernels stream (rebuilt from packed/scales/zeros, not saved)
        self.register_buffer("_native", None, persistent=False)

    def load_weight(self, weight: torch.Tensor) -> None:
        """Quantize and store an FP16 weight matrix.

        Args:
            weight: [d_out, d_in] float16 CUDA tensor.
        """
        assert weight.shape == (self.d_out, self.d_in), (
            f"Expected weight shape ({self.d_out}, {self.d_in}), got {tuple(weight.shape)}")
        _require_extension()
        if weight.dtype != torch.float16:
            weight = weight.to(torch.float16)
        weight = _aligned(weight.contiguous())
        packed, scales, zeros, _ = _C.quantize_weights(weight, with_copy=False)
        self.packed = packed
        self.scales = scales
        self.zeros = zeros
        self.fp16_w = _C.build_colmajor(weight).t()
        self._native = _C.build_native(packed, scales, zeros)
        self._quantized = True

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y = W_split x for one activation vector, or for each row of a batch.

        Args:
            x:   [d_in] float16 activation vector, or [m, d_in] (each row with
                 its own outlier mask; up to 16 rows share one weight stream).
            out: optional tensor to write y into (same shape as y, float16),
                 e.g. a slice of one buffer that gathers several layers'
                 outputs for a single copy to the host.  Not in the reference
                 API, which always allocates y.

        Returns:
            y: [d_out] float16 ([m, d_out] for a batch); `out` when given.
        """
        fast = self.__dict__.get("_fast")
        b = self._buffers
        if (fast is not None and fast[1] is b["packed"] and fast[2] is b["fp16_w"] and fast[3] is b["_native"]
                and fast[4] is b["scales"] and fast[5] is b["zeros"] and fast[6] == self.outlier_k):
            y = fast[0].forward(x, out)
            if y is not None:
                return y
        if not self._quantized:
            raise RuntimeError("Call load_weight() before forward()")
        self._refresh_fast()
        if x.dtype != torch.float16:
            x = x.to(torch.float16)
        if not x.is_contiguous():
            x = x.contiguous()
        y = split_gemv(self.packed, self.scales, self.zeros, self.fp16_w, x, self.outlier_k, self._native)
        if out is None:
            return y
        if out.shape != y.shape:
            raise RuntimeError(f"out has shape {tuple(out.shape)}, expected {tuple(y.shape)}")
        return out.copy_(y)

    def _refresh_fast(self) -> None:
        # The prebuilt weights handle for single vectors (checked once, then
        # only x is checked per call), keyed on the buffer objects and k it
        # was built from: forward() uses it only while all of them are the
        # ones the module holds now.
        b = self._buffers
        key = (b["packed"], b["fp16_w"], b["_native"], b["scales"], b["zeros"], self.outlier_k)
        fast = self.__dict__.get("_fast")
        if fast is not None and all(u is v for u, v in zip(fast[1:6], key[:5])) and fast[6] == key[5]:
            return
        self._fast = None
        if any(t is None or not t.is_cuda for t in key[:5]):
            return
        try:
            handle = _C.SplitLinear(key[0], key[3], key[4], key[1], key[2], float(self.outlier_k))
        except RuntimeError:
            return  # not a layout the handle takes: the general path checks and reports
        self._fast = (handle,) + key

    def _apply(self, fn, *args, **kwargs):
        self.__dict__["_fast"] = None  # .to() / .cuda() replace the buffers the handle refers to
        return super()._apply(fn, *args, **kwargs)

    def __getstate__(self):
        state = self.__dict__.copy()
        state["_fast"] = None  # the handle is rebuilt on the first forward()
        return state

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        # A fresh module holds None buffers; materialise them from the checkpoint
        # (rebuilding the column-major mirror) so load_state_dict round-trips.
        names = ("packed", "scales", "zeros", "fp16_w")
        if not self._quantized and all(prefix + n in state_dict for n in names):
            _require_extension()
            dev = state_dict[prefix + "packed"].device
            if dev.type != "cuda":
                dev = torch.device("cuda", torch.cuda.current_device())
            self.packed = state_dict[prefix + "packed"].to(dev).contiguous()
            self.scales = state_dict[prefix + "scales"].to(dev, torch.float16).contiguous()
            self.zeros = state_dict[prefix + "zeros"].to(dev, torch.float16).contiguous()
            w = state_dict[prefix + "fp16_w"].to(dev, torch.float16).contiguous()
            self.fp16_w = _C.build_colmajor(_aligned(w)).t()
            self._native = _C.build_native(self.packed, self.scales, self.zeros)
            self._quantized = True
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)

    def extra_repr(self) -> str:
        return f"d_in={self.d_in}, d_out={self.d_out}, outlier_k={self.outlier_k}"
