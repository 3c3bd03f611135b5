"""FP8 (E4M3) dynamic activation quantisation on the sm_100a library.

Drop-in for ``flashvsr_sm89_ops.fp8_quant`` (fp8_quant.py:13-55): same name,
same return convention ``(codes, scale)`` with ``scale = amax / 448`` kept on
the GPU (no host sync), computed as the reference's torch expression evaluates on a CUDA
tensor: ``amax * fl(1/448)``.  ``mode="token"`` adds one scale per row.
"""
from __future__ import annotations

import os

import torch

from . import _lib

FP8_MAX = 448.0

_MODES = {"tensor": _lib.FVB_SCALE_TENSOR, "token": _lib.FVB_SCALE_ROW, "row": _lib.FVB_SCALE_ROW,
          "channel": _lib.FVB_SCALE_ROW}


def default_act_mode() -> str:
    """Activation granularity used by FP8Linear/FP8FFN when none is given.

    ``FS89_FP8_SCALE=tensor`` selects the reference's per-tensor numerics (bit-exact
    codes); the default ``token`` is the B200 pack's per-token x per-channel mode.
    """
    v = os.environ.get("FS89_FP8_SCALE", "token").lower()
    return "tensor" if v == "tensor" else "token"


def mode_code(mode: str) -> int:
    try:
        return _MODES[mode]
    except KeyError:
        raise ValueError(f"unknown FP8 scale mode {mode!r} (tensor|token)") from None


def _prep(x2: torch.Tensor, name: str) -> torch.Tensor:
    _lib.require_cuda(x2)
    if x2.dim() != 2:
        raise ValueError(f"{name}: expected a 2-D [M, K] tensor, got {tuple(x2.shape)}")
    if x2.dtype != torch.bfloat16:
        raise ValueError(f"{name}: expected bf16 input, got {x2.dtype}")
    return x2 if x2.is_contiguous() else x2.contiguous()


def _run(fn: str, x2: torch.Tensor, mode: str):
    x2 = _prep(x2, fn)
    M, K = x2.shape
    code = mode_code(mode)
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x2.device)
    scale = torch.empty((M if code == _lib.FVB_SCALE_ROW else 1,), dtype=torch.float32,
                        device=x2.device)
    ws = None
    if code == _lib.FVB_SCALE_TENSOR:
        ws = torch.empty(64, dtype=torch.float32, device=x2.device)
    _lib.call(fn, _lib.ptr(x2), M, K, _lib.ptr(q), _lib.ptr(scale), code, _lib.ptr(ws),
              _lib.stream_of(x2))
    return q, scale


def quantize_fp8(x2: torch.Tensor, mode: str = "tensor"):
    """x2: [M, K] bf16 -> (e4m3 codes [M, K], fp32 scale [1] or [M] on the GPU).

    s = max(amax, 1e-12)/448; codes = e4m3(clamp(x/s, +-448)); returned scale =
    amax * fl(1/448) (the reference's `amax / FP8_MAX` on a CUDA tensor).
    """
    return _run("fvb_quant_fp8", x2, mode)


def fused_gelu_quant_fp8(y2: torch.Tensor, mode: str = "tensor"):
    """y2: [M, K] bf16 -> (fp8, scale), equal to quantize_fp8(F.gelu(y2, approximate='tanh')).

    Drop-in for flashvsr_sm89_ops.fp8_ffn.fused_gelu_quant_fp8 (fp8_ffn.py:57-72).
    """
    return _run("fvb_gelu_quant_fp8", y2, mode)
