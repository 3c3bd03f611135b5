"""FP8 (E4M3) Linear on a hand-written tcgen05 GEMM (sm_100a).

Drop-in for ``flashvsr_sm89_ops.fp8_linear`` (fp8_linear.py:16-67):
``FP8Linear(linear)`` quantises the weight once and runs every forward as
dynamic activation quantisation + ``fvb_fp8_gemm`` (no cuBLASLt, no
``torch._scaled_mm``).  ``convert_linears_fp8(model, parts)`` matches the same
module names.  Granularity: ``"tensor"`` reproduces the reference's per-tensor
scales; ``"token"`` (default, or ``FS89_FP8_SCALE``) uses per-token activation
and per-output-channel weight scales.
"""
from __future__ import annotations

import re

import torch
import torch.nn as nn

from . import _lib
from .fp8_quant import FP8_MAX, default_act_mode, mode_code, quantize_fp8


def quantize_weight(w: torch.Tensor, mode: str):
    """One-time weight quantisation, the eager formula of fp8_linear.py:17-22.

    w_scale = (|w|.amax()/448).clamp(min=1e-12) (per tensor, or per output row for
    "token"/"channel"), codes = (w / w_scale).to(e4m3) in the weight's dtype.
    Runs once at conversion time on the weight's device, like the reference.
    """
    w = w.detach()
    if mode == "tensor":
        s = (w.abs().amax() / FP8_MAX).clamp(min=1e-12).float()
        return (w / s).to(torch.float8_e4m3fn), s.reshape(1)
    s = (w.abs().amax(dim=1) / FP8_MAX).clamp(min=1e-12).float()
    return (w / s[:, None]).to(torch.float8_e4m3fn), s.contiguous()


def fp8_mm(x8: torch.Tensor, sx: torch.Tensor, w8: torch.Tensor, sw: torch.Tensor,
           bias: torch.Tensor | None, out: torch.Tensor | None = None,
           epilogue: int = _lib.FVB_EPI_NONE, amax_out: torch.Tensor | None = None):
    """out[M,N] = bf16(x8 w8^T * sx * sw + bias) on the tcgen05 GEMM.

    sx has 1 (per-tensor) or M (per-token) entries, sw 1 or N entries.
    """
    _lib.require_cuda(x8, w8)
    M, K = x8.shape
    N = w8.shape[0]
    if w8.shape[1] != K:
        raise ValueError(f"fp8_mm: K mismatch {tuple(x8.shape)} x {tuple(w8.shape)}")
    a_mode = _lib.FVB_SCALE_ROW if (sx.numel() == M and M > 1) else _lib.FVB_SCALE_TENSOR
    w_mode = _lib.FVB_SCALE_ROW if (sw.numel() == N and N > 1) else _lib.FVB_SCALE_TENSOR
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x8.device)
    if bias is not None and bias.dtype != torch.bfloat16:
        bias = bias.to(torch.bfloat16)
    _lib.call("fvb_fp8_gemm", _lib.ptr(x8), _lib.ptr(sx), a_mode, _lib.ptr(w8), _lib.ptr(sw),
              w_mode, _lib.ptr(bias), M, N, K, _lib.ptr(out), epilogue, _lib.ptr(amax_out),
              _lib.stream_of(x8))
    return out


class FP8Linear(nn.Module):
    """nn.Linear replacement with E4M3 weights and a tcgen05 FP8 GEMM (fp8_linear.py:16-42)."""

    def __init__(self, linear: nn.Linear, mode: str | None = None):
        super().__init__()
        self.mode = mode or default_act_mode()
        mode_code(self.mode)
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        q, s = quantize_weight(linear.weight, self.mode)
        self.weight = nn.Parameter(q, requires_grad=False)
        self.register_buffer("w_scale", s, persistent=False)
        if linear.bias is not None:
            self.bias = nn.Parameter(linear.bias.detach().to(torch.bfloat16).clone(),
                                     requires_grad=False)
        else:
            self.bias = None

    def _mm(self, x8, s, out=None):
        return fp8_mm(x8, s, self.weight, self.w_scale, self.bias, out=out)

    def forward(self, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x8, s = quantize_fp8(x2, self.mode)
        y = self._mm(x8, s)
        return y.reshape(*shape[:-1], y.shape[-1])

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}, scales={self.mode}"


def convert_linears_fp8(model: nn.Module, parts=("ffn", "self", "cross"), mode: str | None = None) -> int:
    """Swap DiT-block Linears whose names match `parts` for FP8Linear; returns the count.

    Same selection as fp8_linear.py:45-67: blocks.N.self_attn.[qkvo],
    blocks.N.cross_attn.[qkvo], blocks.N.ffn.[02].
    """
    pats = []
    if "self" in parts:
        pats.append(re.compile(r"^blocks\.\d+\.self_attn\.[qkvo]$"))
    if "cross" in parts:
        pats.append(re.compile(r"^blocks\.\d+\.cross_attn\.[qkvo]$"))
    if "ffn" in parts:
        pats.append(re.compile(r"^blocks\.\d+\.ffn\.[02]$"))
    n = 0
    for name, mod in list(model.named_modules()):
        if type(mod) is not nn.Linear or not any(p.match(name) for p in pats):
            continue
        parent_name, _, leaf = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, leaf, FP8Linear(mod, mode=mode))
        n += 1
    return n
