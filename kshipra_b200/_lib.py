"""ctypes binding of ``libkshipra_b200.so`` (the C ABI in include/kshipra_b200.h).

The library is the only compute path: there is no CPU or PyTorch fallback.
``lib()`` raises ``KshipraLibraryError`` if the shared library is missing or a
symbol is absent; every call goes through ``call()``, which raises on a
non-zero status.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libkshipra_b200.so")

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float

# name -> (restype, argtypes); mirrors include/kshipra_b200.h
SIGNATURES = {
    "ksh_abi_version": (I32, []),
    "ksh_status_string": (ctypes.c_char_p, [I32]),
    "ksh_last_cuda_error": (I32, []),
    "ksh_set_pdl": (I32, [I32]),
    "ksh_set_gemv_resident": (I32, [I32]),
    "ksh_set_gemv_tc": (I32, [I32]),
    "ksh_set_gemv_dp4a": (I32, [I32]),
    "ksh_set_gemm_mid": (I32, [I32]),
    "ksh_set_gemm_predeq": (I64, [I64]),
    "ksh_set_decode_split": (I32, [I32]),
    "ksh_kernel_launches": (ctypes.c_uint64, []),
    "ksh_pack_int8": (I32, [P, I64, I64, P, P, P, P]),
    "ksh_pack_int4": (I32, [P, I64, I64, I64, P, P, P, P]),
    "ksh_linear_workspace_size": (I64, [I64, I64, I64]),
    "ksh_qlinear_w8": (I32, [P, I64, I64, P, F32, P, P, P, P, P, I64, P, I64, P]),
    "ksh_qlinear_w4": (I32, [P, I64, I64, P, F32, P, P, I64, I64, P, P, P, I64, P, I64, P]),
    "ksh_linear_f32": (I32, [P, I64, I64, P, F32, P, P, P, P, I64, P, I64, P]),
    "ksh_qlinear_swiglu_w8": (I32, [P, I64, I64, P, F32, P, P, P, I64, P, I64, P]),
    "ksh_qlinear_swiglu_w4": (I32, [P, I64, I64, P, F32, P, P, I64, I64, P, I64, P, I64, P]),
    "ksh_linear_swiglu_f32": (I32, [P, I64, I64, P, F32, P, P, I64, P, I64, P]),
    "ksh_embedding": (I32, [P, I64, P, I64, I64, P, P, P]),
    "ksh_rmsnorm": (I32, [P, P, P, I64, I64, F32, P]),
    "ksh_rope_kv_write": (I32, [P, I64, I64, I64, I64, P, P, P, P, I64, P, P, I64, I64, I64,
                                I64, P, P]),
    "ksh_paged_attention_workspace_size": (I64, [I64, I64, I64, I64, I64, I64]),
    "ksh_paged_attention": (I32, [P, I64, I64, P, I64, I64, I64, I64, I64, P, I64, P, P, I64,
                                  I64, I64, P, P, I64, P, P]),
    "ksh_decode_attention": (I32, [P, I64, I64, I64, I64, P, P, P, P, I64, P, I64, I64, I64,
                                   I64, P, I64, I64, P, P, P]),
    "ksh_decode_attention_workspace_size": (I64, [I64, I64, I64, I64]),
    "ksh_decode_attention_ws": (I32, [P, I64, I64, I64, I64, P, P, P, P, I64, P, I64, I64, I64,
                                      I64, P, I64, I64, P, P, I64, P, P]),
    "ksh_set_decode_gsplit": (I32, [I32]),
    "ksh_lm_head_workspace_size": (I64, [I64, I64]),
    "ksh_lm_head_argmax": (I32, [P, I64, I64, P, F32, P, I64, P, P, P, I64, P]),
    "ksh_lm_head_argmax_noalloc_max_bytes": (I64, []),
    "ksh_lm_head_argmax_noalloc": (I32, [P, I64, I64, P, F32, P, I64, P, P, P]),
    "ksh_argmax_rows": (I32, [P, I64, I64, P, P]),
    "ksh_decode_advance": (I32, [P, I64, P, P, P, P, P, I64, I64, P, I64, P, P, P]),
    "ksh_check_bounded_wait": (I32, [I64, I32, P, P, P, P]),
    "ksh_peer_allreduce_buffer_floats": (I64, [I64, I32]),
    "ksh_peer_allreduce_epoch_words": (I64, []),
    "ksh_peer_allreduce_f32": (I32, [P, I32, I32, I64, I64, I32, P, P, P, P]),
    "ksh_lm_head_tc_workspace_size": (I64, [I64, I64, I64]),
    "ksh_lm_head_split_weight": (I32, [P, I64, I64, P, P, P, P, P]),
    "ksh_lm_head_argmax_tc": (I32, [P, I64, I64, P, F32, P, P, P, I64, P, P, P, I64, P]),
}


class KshipraLibraryError(RuntimeError):
    """The CUDA library is missing, stale or a call failed."""


_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise KshipraLibraryError(
                    f"{LIB_PATH} is not built; run `python -m kshipra_b200.build` "
                    "(there is no CPU fallback)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                try:
                    fn = getattr(h, name)
                except AttributeError as e:
                    raise KshipraLibraryError(f"symbol {name} missing from {LIB_PATH}") from e
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def call(name: str, *args) -> int:
    st = getattr(lib(), name)(*args)
    if st != 0:
        msg = lib().ksh_status_string(st).decode()
        extra = ""
        if st == -3:
            extra = f" (cudaError {lib().ksh_last_cuda_error()})"
        raise KshipraLibraryError(f"{name} failed: {msg}{extra}")
    return st


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, name: str = "tensor") -> None:
    if not t.is_cuda:
        raise KshipraLibraryError(f"{name} must be a CUDA tensor (no CPU path)")
