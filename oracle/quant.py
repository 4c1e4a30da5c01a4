"""numpy restatement of the reference weight-only quantizers.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows engine/quantization.py of the reference:

* ``quantize_int8_per_channel``  -- quantization.py:196-223
* ``quantize_int4_per_group``    -- quantization.py:238-318
* ``dequantize_int8`` / ``dequantize_int4`` -- quantization.py:226-230, 321-344

Arithmetic notes (these are what make the result byte-exact):

* the scale is ``fp16(max(fp32(absmax) / 127, fp32(1e-8)))`` with a true
  IEEE fp32 division and round-to-nearest-even into fp16;
* the quantizer divides by the fp16-rounded scale widened back to fp32
  (quantization.py:215, :298), rounds half-to-even (``torch.round``) and
  clamps;
* when the fp16 scale underflows to 0, ``w / 0`` is +-inf (clamped to the
  range end) and ``0 / 0`` is NaN, which torch's float->int8 conversion maps
  to 0 -- probed on the reference's torch build and pinned by the golden
  fixtures.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def _validate(w: np.ndarray) -> None:
    # quantization.py:180-190 (_validate_weight)
    if w.ndim != 2:
        raise ValueError(f"weight must be 2-D, got {w.ndim}-D")
    if w.shape[0] == 0 or w.shape[1] == 0:
        raise ValueError(f"weight must have non-zero dims, got {w.shape}")
    if not np.isfinite(w).all():
        raise ValueError("weight contains non-finite values")


def _scale_fp16(absmax: np.ndarray, qmax: float) -> np.ndarray:
    s32 = absmax.astype(F32) / F32(qmax)            # fp32 IEEE division
    s32 = np.maximum(s32, F32(1e-8))                # clamp_min(1e-8) in fp32
    return s32.astype(np.float16)                   # RNE


def _round_clamp(r: np.ndarray, lo: int, hi: int) -> np.ndarray:
    q = np.rint(r)                                  # half-to-even, like torch.round
    q = np.clip(q, lo, hi)                          # NaN propagates
    q = np.where(np.isnan(q), F32(0), q)            # NaN -> 0 on conversion
    return q.astype(np.int8)


def quantize_int8_per_channel(w: np.ndarray):
    """Returns (payload int8 [N,K], scales fp16 [N])."""
    w = np.asarray(w, dtype=F32)
    _validate(w)
    s16 = _scale_fp16(np.abs(w).max(axis=1), 127.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = w / s16.astype(F32)[:, None]
    return _round_clamp(r, -127, 127), s16


def quantize_int4_per_group(w: np.ndarray, group_size: int = 128):
    """Returns (payload uint8 [N, Kp/2], scales fp16 [N, Kp/G], Kp)."""
    w = np.asarray(w, dtype=F32)
    _validate(w)
    if group_size <= 0 or group_size % 2 != 0:
        raise ValueError(f"group_size must be a positive even integer, got {group_size}")
    n, k = w.shape
    ng = (k + group_size - 1) // group_size
    kp = ng * group_size
    wp = np.zeros((n, kp), dtype=F32)
    wp[:, :k] = w
    wg = wp.reshape(n, ng, group_size)
    s16 = _scale_fp16(np.abs(wg).max(axis=2), 7.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = wg / s16.astype(F32)[:, :, None]
    q = _round_clamp(r, -8, 7).reshape(n, kp)
    u = q.view(np.uint8) & np.uint8(0x0F)
    packed = (u[:, 0::2] | (u[:, 1::2] << np.uint8(4))).astype(np.uint8)
    return packed, s16, kp


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """uint8 [N, Kp/2] -> int8 [N, Kp] (low nibble = even k)."""
    lo = (packed & 0x0F).astype(np.int16)
    hi = ((packed >> 4) & 0x0F).astype(np.int16)
    u = np.stack([lo, hi], axis=-1).reshape(packed.shape[0], -1)
    return np.where(u >= 8, u - 16, u).astype(np.int8)


def dequantize_int8(payload: np.ndarray, scales: np.ndarray) -> np.ndarray:
    return payload.astype(F32) * scales.astype(F32)[:, None]


def dequantize_int4(packed: np.ndarray, scales: np.ndarray, in_features: int,
                    group_size: int) -> np.ndarray:
    q = unpack_int4(packed).astype(F32)
    s = np.repeat(scales.astype(F32), group_size, axis=1)
    return (q * s)[:, :in_features]
