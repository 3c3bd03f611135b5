"""ctypes binding of ``libflashvsr_b200.so`` (the sm_100a C ABI in ``include/flashvsr_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every op
raises.  Status codes map to Python exceptions with the same types the
reference raises for the same conditions (``ValueError``/``AssertionError``-like
argument errors become ``ValueError``, unsupported modes ``NotImplementedError``,
CUDA failures ``RuntimeError``).
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _build

FVB_OK = 0
FVB_ERR_INVALID = 1
FVB_ERR_UNSUPPORTED = 2
FVB_ERR_CUDA = 3

FVB_SCALE_TENSOR = 0
FVB_SCALE_ROW = 1
FVB_EPI_NONE = 0
FVB_EPI_GELU_AMAX = 1

_lib = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/flashvsr_b200.h
_SIGS = {
    "fvb_abi_version": (_int, []),
    "fvb_last_error": (ctypes.c_char_p, []),
    "fvb_device_error": (_int, [ctypes.POINTER(ctypes.c_uint)]),
    "fvb_quant_fp8_workspace_bytes": (_sz, [_i64, _i64, _int]),
    "fvb_quant_fp8": (_int, [_vp, _i64, _i64, _vp, _vp, _int, _vp, _vp]),
    "fvb_gelu_quant_fp8": (_int, [_vp, _i64, _i64, _vp, _vp, _int, _vp, _vp]),
    "fvb_quant_fp8_tensor_noalloc": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "fvb_fp8_gemm": (_int, [_vp, _vp, _int, _vp, _vp, _int, _vp, _i64, _i64, _i64, _vp, _int, _vp, _vp]),
    "fvb_quant_fp8_with_amax": (_int, [_vp, _i64, _i64, _vp, _int, _vp, _vp, _vp]),
    "fvb_fp8_ffn_workspace_bytes": (_sz, [_i64, _i64]),
    "fvb_fp8_ffn": (_int, [_vp, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _vp, _vp, _vp]),
    "fvb_fp8_ffn_residual": (_int, [_vp, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64,
                                    _i64, _vp, _vp, _vp, _vp, _vp]),
    "fvb_rms_rope": (_int, [_vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _int, _vp, _vp, _vp]),
    "fvb_qkv_rope_window": (_int, [_vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32,
                                   _f32, _vp, _vp, _vp, _vp, _vp]),
    "fvb_ln_modulate": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp, _vp, _vp]),
    "fvb_ln_modulate_adaln": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp, _vp, _vp,
                                     _vp]),
    "fvb_layer_norm": (_int, [_vp, _vp, _vp, _i64, _i64, _f32, _vp, _vp, _vp, _vp]),
    "fvb_gate_add_ln_modulate": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp,
                                         _vp, _vp, _vp]),
    "fvb_gate_add_layer_norm": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp,
                                        _vp, _vp, _vp]),
    "fvb_gate_add": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "fvb_mask_to_csr": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "fvb_bsa_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp, _vp]),
    "fvb_window_partition": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _int, _vp, _vp]),
    "fvb_copy_window_h2d": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "fvb_draft_mask_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "fvb_draft_block_mask": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "fvb_causal_topk_mask": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp, _vp]),
    "fvb_block_mean_pool": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "fvb_block_mean_pool2": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _vp, _vp]),
    "fvb_causal_topk_pooled_csr": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp,
                                          _vp, _vp]),
    "fvb_causal_topk_pooled": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp]),
}


class FvbError(RuntimeError):
    """A CUDA-side failure reported by the C ABI."""


def lib_path() -> str:
    return _build.LIB_PATH


def load():
    """Load (building first if the sources are newer) and return the ctypes library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if _build.needs_build():
            if os.environ.get("FVB_NO_BUILD") == "1" and os.path.exists(path):
                pass
            else:
                _build.build()
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols():
    return list(_SIGS)


def _raise(rc: int, name: str):
    msg = (load().fvb_last_error() or b"").decode(errors="replace")
    if rc == FVB_ERR_INVALID:
        raise ValueError(f"{name}: {msg}")
    if rc == FVB_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{name}: {msg}")
    raise FvbError(f"{name}: {msg}")


def _kernels_per_call(name: str, args) -> int:
    """How many of this library's kernels one C-ABI call launches."""
    if name == "fvb_quant_fp8":
        return 2 if args[5] == FVB_SCALE_TENSOR else 1
    if name == "fvb_gelu_quant_fp8":
        return 3 if args[5] == FVB_SCALE_TENSOR else 1
    if name in ("fvb_fp8_ffn", "fvb_fp8_ffn_residual"):
        return 3
    if name == "fvb_draft_block_mask":
        return 4
    if name == "fvb_causal_topk_mask":
        return 3
    if name in ("fvb_device_error", "fvb_abi_version", "fvb_last_error", "fvb_copy_window_h2d"):
        return 0  # no kernel (fvb_copy_window_h2d is a copy-engine transfer)
    return 1


_count = None


def start_launch_count():
    global _count
    _count = 0


def stop_launch_count() -> int:
    global _count
    n, _count = _count or 0, None
    return n


def call(name: str, *args):
    global _count
    rc = getattr(load(), name)(*args)
    if rc != FVB_OK:
        _raise(rc, name)
    if _count is not None:
        _count += _kernels_per_call(name, args)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(
                "flashvsr_sm89_ops_b200 runs on CUDA tensors only (sm_100a); "
                f"got a tensor on {t.device}")


def device_error() -> int:
    v = ctypes.c_uint(0)
    call("fvb_device_error", ctypes.byref(v))
    return int(v.value)
