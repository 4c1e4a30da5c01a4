"""Weight-only INT8 / INT4 quantization on the B200.

Drop-in for the reference's engine/quantization.py: same names, same
``QuantizedWeight`` fields and validation, same packed layout and error
class.  What changes is where the work happens:

* ``quantize_int8_per_channel`` / ``quantize_int4_per_group`` pack on the GPU
  (``ksh_pack_int8`` / ``ksh_pack_int4``), byte-identical to the reference;
* ``QuantizedLinear.forward`` never materialises the dequantized weight: it
  calls the fused dequant-GEMV (decode) / GEMM (prefill) kernels.

Layouts (identical to the reference, quantization.py:37-49):

* INT8: payload int8 [out, in], scales fp16 [out]
* INT4: payload uint8 [out, in_padded/2], low nibble = even k, scales fp16
  [out, in_padded/G]
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import _lib
from ._lib import call, ptr, stream_ptr


class QuantizationError(ValueError):
    """Raised on invalid weight, scale, or group-size inputs (quantization.py:69)."""


def _device(w: torch.Tensor) -> torch.device:
    if w.is_cuda:
        return w.device
    if not torch.cuda.is_available():
        raise _lib.KshipraLibraryError("quantization runs on the GPU; no CUDA device is available")
    return torch.device("cuda", torch.cuda.current_device())


@dataclass
class QuantizedWeight:
    """Quantized weight plus the metadata to use it (quantization.py:78-172)."""

    payload: torch.Tensor
    scales: torch.Tensor
    scheme: str
    original_shape: Tuple[int, int]
    group_size: Optional[int] = None
    in_features_padded: Optional[int] = None

    def __post_init__(self) -> None:
        # validation rules of quantization.py:108-152
        if self.scheme not in ("int8_per_channel", "int4_per_group"):
            raise QuantizationError(f"unknown scheme {self.scheme!r}")
        out_features, _ = self.original_shape
        if self.scales.shape[0] != out_features:
            raise QuantizationError(
                f"scales.shape[0] = {self.scales.shape[0]} does not match out_features = {out_features}")
        if self.scheme == "int8_per_channel":
            if self.payload.dtype != torch.int8:
                raise QuantizationError(f"INT8 payload must be int8, got {self.payload.dtype}")
            if self.scales.dim() != 1:
                raise QuantizationError(
                    f"INT8 scales must be 1-D [out_features], got {tuple(self.scales.shape)}")
            if tuple(self.payload.shape) != tuple(self.original_shape):
                raise QuantizationError(
                    f"INT8 payload shape {tuple(self.payload.shape)} != original_shape {self.original_shape}")
        else:
            if self.payload.dtype != torch.uint8:
                raise QuantizationError(f"INT4 payload must be uint8, got {self.payload.dtype}")
            if self.group_size is None or self.in_features_padded is None:
                raise QuantizationError("INT4 requires group_size and in_features_padded")
            groups = self.in_features_padded // self.group_size
            if tuple(self.scales.shape) != (out_features, groups):
                raise QuantizationError(
                    f"INT4 scales shape {tuple(self.scales.shape)} != ({out_features}, {groups})")
            cols = self.in_features_padded // 2
            if tuple(self.payload.shape) != (out_features, cols):
                raise QuantizationError(
                    f"INT4 payload shape {tuple(self.payload.shape)} != ({out_features}, {cols})")

    def storage_bytes(self) -> int:
        return (self.payload.numel() * self.payload.element_size()
                + self.scales.numel() * self.scales.element_size())

    def dequantize(self, dtype: torch.dtype = torch.float16) -> torch.Tensor:
        """Materialise the weight (API parity; the forward path never calls this)."""
        if self.scheme == "int8_per_channel":
            w = self.payload.to(torch.float32) * self.scales.to(torch.float32).unsqueeze(1)
        else:
            n, kp, g = self.original_shape[0], self.in_features_padded, self.group_size
            lo = (self.payload & 0x0F).to(torch.int16)
            hi = ((self.payload >> 4) & 0x0F).to(torch.int16)
            u = torch.stack([lo, hi], dim=-1).reshape(n, kp)
            q = torch.where(u >= 8, u - 16, u).to(torch.float32)
            s = self.scales.to(torch.float32).repeat_interleave(g, dim=1)
            w = (q * s)[:, : self.original_shape[1]]
        return w.to(dtype)


def _validate_weight(w: torch.Tensor) -> None:
    # quantization.py:180-190
    if w.dim() != 2:
        raise QuantizationError(f"weight must be 2-D, got {w.dim()}-D")
    if w.shape[0] == 0 or w.shape[1] == 0:
        raise QuantizationError(f"weight must have non-zero dims, got {tuple(w.shape)}")


def _raise_if_nonfinite(flags: torch.Tensor) -> None:
    if int(flags.item()) & 1:
        raise QuantizationError("weight contains non-finite values")


def quantize_int8_per_channel(w: torch.Tensor) -> QuantizedWeight:
    """Symmetric per-output-channel INT8 (quantization.py:196-223), packed on the GPU."""
    _validate_weight(w)
    dev = _device(w)
    wf = w.detach().to(device=dev, dtype=torch.float32).contiguous()
    n, k = wf.shape
    payload = torch.empty((n, k), dtype=torch.int8, device=dev)
    scales = torch.empty((n,), dtype=torch.float16, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        call("ksh_pack_int8", ptr(wf), n, k, ptr(payload), ptr(scales), ptr(flags), stream_ptr())
    _raise_if_nonfinite(flags)
    return QuantizedWeight(payload=payload, scales=scales, scheme="int8_per_channel",
                           original_shape=(n, k))


def quantize_int4_per_group(w: torch.Tensor, group_size: int = 128) -> QuantizedWeight:
    """Symmetric per-group INT4, nibble-packed (quantization.py:238-318), on the GPU."""
    _validate_weight(w)
    if group_size <= 0 or group_size % 2 != 0:
        raise QuantizationError(f"group_size must be a positive even integer, got {group_size}")
    dev = _device(w)
    wf = w.detach().to(device=dev, dtype=torch.float32).contiguous()
    n, k = wf.shape
    ng = (k + group_size - 1) // group_size
    kp = ng * group_size
    payload = torch.empty((n, kp // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((n, ng), dtype=torch.float16, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        call("ksh_pack_int4", ptr(wf), n, k, group_size, ptr(payload), ptr(scales), ptr(flags),
             stream_ptr())
    _raise_if_nonfinite(flags)
    return QuantizedWeight(payload=payload, scales=scales, scheme="int4_per_group",
                           original_shape=(n, k), group_size=group_size, in_features_padded=kp)


# ---------------------------------------------------------------------------
# Fused linear launches (shared by QuantizedLinear and the model)
# ---------------------------------------------------------------------------

class Workspace:
    """Grow-only device scratch for the tensor-core GEMM path."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device) -> Tuple[Optional[int], int]:
        if nbytes <= 0:
            return None, 0
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        return self.buf.data_ptr(), self.buf.numel()


_WS = Workspace()


def linear_launch(x2d: torch.Tensor, qw: Optional[QuantizedWeight], w_f32: Optional[torch.Tensor],
                  bias: Optional[torch.Tensor], out: torch.Tensor,
                  residual: Optional[torch.Tensor] = None, ws: Workspace = _WS,
                  norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6) -> torch.Tensor:
    """out[m, n] = x' @ W^T (+ bias) (+ residual), W quantized or fp32;
    x' = RMSNorm(x2d; norm_w, eps) when norm_w is given, else x2d."""
    m, k = x2d.shape
    n = out.shape[1]
    wsz = int(_lib.lib().ksh_linear_workspace_size(m, k, n))
    wp, wb = ws.get(wsz, x2d.device)
    s = stream_ptr()
    nw = ptr(norm_w)
    if qw is None:
        call("ksh_linear_f32", ptr(x2d), m, k, nw, eps, ptr(w_f32), ptr(bias), ptr(residual),
             ptr(out), n, wp, wb, s)
    elif qw.scheme == "int8_per_channel":
        call("ksh_qlinear_w8", ptr(x2d), m, k, nw, eps, ptr(qw.payload), ptr(qw.scales),
             ptr(bias), ptr(residual), ptr(out), n, wp, wb, s)
    else:
        call("ksh_qlinear_w4", ptr(x2d), m, k, nw, eps, ptr(qw.payload), ptr(qw.scales),
             qw.group_size, qw.in_features_padded, ptr(bias), ptr(residual), ptr(out), n, wp,
             wb, s)
    return out


def swiglu_launch(x2d: torch.Tensor, qw: Optional[QuantizedWeight], w_f32: Optional[torch.Tensor],
                  inter: int, out: torch.Tensor, ws: Workspace = _WS,
                  norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6) -> torch.Tensor:
    """out[m, j] = silu(x' W_gate^T)[m, j] * (x' W_up^T)[m, j]; W holds gate rows then
    up rows; x' = RMSNorm(x2d) when norm_w is given."""
    m, k = x2d.shape
    wsz = int(_lib.lib().ksh_linear_workspace_size(m, k, 2 * inter))
    wp, wb = ws.get(wsz, x2d.device)
    s = stream_ptr()
    nw = ptr(norm_w)
    if qw is None:
        call("ksh_linear_swiglu_f32", ptr(x2d), m, k, nw, eps, ptr(w_f32), ptr(out), inter, wp,
             wb, s)
    elif qw.scheme == "int8_per_channel":
        call("ksh_qlinear_swiglu_w8", ptr(x2d), m, k, nw, eps, ptr(qw.payload), ptr(qw.scales),
             ptr(out), inter, wp, wb, s)
    else:
        call("ksh_qlinear_swiglu_w4", ptr(x2d), m, k, nw, eps, ptr(qw.payload), ptr(qw.scales),
             qw.group_size, qw.in_features_padded, ptr(out), inter, wp, wb, s)
    return out


class QuantizedLinear(nn.Module):
    """Drop-in for ``nn.Linear`` with quantized weights (quantization.py:352-402).

    ``forward`` runs the fused dequant kernels: x fp32 ``[..., in]`` on the
    GPU -> fp32 ``[..., out]``.
    """

    def __init__(self, linear: nn.Linear, scheme: str = "int8", group_size: int = 128) -> None:
        super().__init__()
        if not isinstance(linear, nn.Linear):
            raise QuantizationError(f"expected nn.Linear, got {type(linear).__name__}")
        if scheme not in ("int8", "int4"):
            raise QuantizationError(f"scheme must be 'int8' or 'int4', got {scheme!r}")
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.scheme = scheme
        w = linear.weight.detach()
        if scheme == "int8":
            self.weight = quantize_int8_per_channel(w)
        else:
            self.weight = quantize_int4_per_group(w, group_size)
        if linear.bias is not None:
            self.register_buffer("bias", linear.bias.detach().to(
                device=self.weight.payload.device, dtype=torch.float32).clone())
        else:
            self.bias = None

    @classmethod
    def from_quantized(cls, qw: QuantizedWeight, bias: Optional[torch.Tensor] = None,
                       scheme: Optional[str] = None) -> "QuantizedLinear":
        obj = cls.__new__(cls)
        nn.Module.__init__(obj)
        obj.out_features, obj.in_features = qw.original_shape
        obj.scheme = scheme or ("int8" if qw.scheme == "int8_per_channel" else "int4")
        obj.weight = qw
        if bias is not None:
            obj.register_buffer("bias", bias)
        else:
            obj.bias = None
        return obj

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(x, "x")
        if x.dtype != torch.float32:
            raise QuantizationError(f"activations must be fp32, got {x.dtype}")
        lead = x.shape[:-1]
        x2d = x.reshape(-1, self.in_features).contiguous()
        out = torch.empty((x2d.shape[0], self.out_features), dtype=torch.float32, device=x.device)
        with torch.cuda.device(x.device):
            linear_launch(x2d, self.weight, None, self.bias, out)
        return out.view(*lead, self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"scheme={self.scheme}, storage_bytes={self.weight.storage_bytes()}")
