"""FFN with the GELU -> FP8 mid-section fused into the up-projection's epilogue.

Drop-in for ``flashvsr_sm89_ops.fp8_ffn`` (fp8_ffn.py:75-115).  The B200 chain
is: quantise x -> tcgen05 GEMM-1 whose epilogue applies bias, GELU(tanh), the
bf16 rounding and the per-row (or per-tensor) amax -> one vectorised pass that
turns the GELU output into E4M3 codes with the finished amax -> tcgen05 GEMM-2.
Codes equal quantize_fp8(F.gelu(h)) exactly as in the reference.
"""
from __future__ import annotations

import re

import torch
import torch.nn as nn

from . import _lib
from .fp8_linear import FP8Linear
from .fp8_quant import fused_gelu_quant_fp8, mode_code, quantize_fp8  # noqa: F401 (re-export)


def ffn_fp8(x8, sx, lin0: FP8Linear, lin2: FP8Linear, out=None, workspace=None,
            residual=None, gate=None):
    """Pre-quantised input -> FFN output through fvb_fp8_ffn (one C-ABI call).

    residual ([M, D] bf16, with gate [D] bf16 or None): return the DiT block's gated
    residual update bf16(residual + bf16(gate * FFN(x))) instead (fvb_fp8_ffn_residual: the
    add runs in the down-projection's epilogue), bit for bit fused_gate_add(residual, gate,
    FFN(x))."""
    M, D = x8.shape
    F = lin0.weight.shape[0]
    if lin0.mode != lin2.mode:
        raise ValueError("FP8FFN: both linears must share one scale mode")
    code = mode_code(lin0.mode)
    if out is None:
        out = torch.empty((M, lin2.weight.shape[0]), dtype=torch.bfloat16, device=x8.device)
    need = _lib.load().fvb_fp8_ffn_workspace_bytes(M, F)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=x8.device)
    a_code = _lib.FVB_SCALE_ROW if (sx.numel() == M and M > 1) else _lib.FVB_SCALE_TENSOR
    if a_code != code and M > 1:
        raise ValueError("FP8FFN: activation scale granularity does not match the module")
    if residual is not None:
        residual = residual.reshape(M, -1)
        if residual.dtype != torch.bfloat16 or not residual.is_contiguous():
            raise ValueError("ffn_fp8: residual must be a contiguous bf16 [M, D] tensor")
        if gate is not None:
            gate = gate.reshape(-1).contiguous()
        _lib.call("fvb_fp8_ffn_residual", _lib.ptr(x8), _lib.ptr(sx), a_code,
                  _lib.ptr(lin0.weight), _lib.ptr(lin0.w_scale), _lib.ptr(lin0.bias),
                  _lib.ptr(lin2.weight), _lib.ptr(lin2.w_scale), _lib.ptr(lin2.bias), code, M, D,
                  F, _lib.ptr(residual), _lib.ptr(gate), _lib.ptr(out), _lib.ptr(workspace),
                  _lib.stream_of(x8))
        return out
    _lib.call("fvb_fp8_ffn", _lib.ptr(x8), _lib.ptr(sx), a_code, _lib.ptr(lin0.weight),
              _lib.ptr(lin0.w_scale), _lib.ptr(lin0.bias), _lib.ptr(lin2.weight),
              _lib.ptr(lin2.w_scale), _lib.ptr(lin2.bias), code, M, D, F, _lib.ptr(out),
              _lib.ptr(workspace), _lib.stream_of(x8))
    return out


class FP8FFN(nn.Module):
    """Replacement for a DiT FFN ``Sequential(Linear, GELU(tanh), Linear)`` whose
    two Linears are already FP8Linear (fp8_ffn.py:75-96)."""

    def __init__(self, lin0, lin2):
        super().__init__()
        self.lin0 = lin0
        self.lin2 = lin2

    def forward(self, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x8, s = quantize_fp8(x2, self.lin0.mode)
        out = ffn_fp8(x8, s, self.lin0, self.lin2)
        return out.reshape(*shape[:-1], out.shape[-1])


def convert_ffn_fp8(model: nn.Module) -> int:
    """Swap every ``blocks.i.ffn`` Sequential for FP8FFN; returns the count.
    Requires convert_linears_fp8(model, parts=["ffn"]) first (fp8_ffn.py:99-115)."""
    pat = re.compile(r"^blocks\.\d+\.ffn$")
    n = 0
    for name, mod in list(model.named_modules()):
        if not pat.match(name) or isinstance(mod, FP8FFN):
            continue  # already converted: re-running enable() is safe
        l0, l2 = mod[0], mod[2]
        if not (isinstance(l0, FP8Linear) and isinstance(l2, FP8Linear)):
            raise AssertionError(f"{name}: run convert_linears_fp8(parts=['ffn']) first")
        parent_name, _, leaf = name.rpartition(".")
        setattr(model.get_submodule(parent_name), leaf, FP8FFN(l0, l2))
        n += 1
    return n
