"""Fused AdaLN elementwise chains on the sm_100a library.

Drop-in for ``flashvsr_sm89_ops.fused_adaln`` (fused_adaln.py:60-85):
``fused_ln_modulate(x, scale, shift, eps)`` (note: scale BEFORE shift) and
``fused_gate_add(x, gate, residual)``, with the reference's per-op bf16 rounding
chain (gate-add is bitwise equal to eager).  ``fused_ln_modulate(...,
emit_fp8=True)`` also returns the per-token E4M3 codes and scales of its
output, so the following FP8 linear skips its own quantisation pass.
"""
from __future__ import annotations

import torch

from . import _lib


def _check(x, name):
    _lib.require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"{name}: expected bf16, got {x.dtype}")


def fused_ln_modulate(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                      eps: float = 1e-6, emit_fp8: bool = False, out: torch.Tensor | None = None,
                      want_out: bool = True):
    """LayerNorm(affine=False) + modulate. x [B, L, D] contiguous bf16; scale/shift [B, 1, D].

    emit_fp8=True also returns the output's per-token FP8 codes and scales:
    (out, q8, scale); want_out=False (with emit_fp8) skips the bf16 output (returned None).
    """
    _check(x, "fused_ln_modulate")
    B, L, D = x.shape
    assert x.is_contiguous() and scale.is_contiguous() and shift.is_contiguous()
    if scale.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16:
        raise ValueError("fused_ln_modulate: scale/shift must be bf16")
    if scale.numel() != B * D or shift.numel() != B * D:
        raise ValueError("fused_ln_modulate: scale/shift must be [B, 1, D]")
    if not want_out and not emit_fp8:
        raise ValueError("fused_ln_modulate: want_out=False needs emit_fp8=True")
    if out is None and want_out:
        out = torch.empty_like(x)
    q8 = qs = None
    if emit_fp8:
        q8 = torch.empty((B * L, D), dtype=torch.float8_e4m3fn, device=x.device)
        qs = torch.empty((B * L,), dtype=torch.float32, device=x.device)
    _lib.call("fvb_ln_modulate", _lib.ptr(x), _lib.ptr(scale), _lib.ptr(shift), B, L, D,
              float(eps), _lib.ptr(out), _lib.ptr(q8), _lib.ptr(qs), _lib.stream_of(x))
    if emit_fp8:
        return out, q8, qs
    return out


def fused_ln_modulate_adaln(x: torch.Tensor, modulation: torch.Tensor, t_mod: torch.Tensor,
                            eps: float = 1e-6, emit_fp8: bool = True, want_out: bool = True):
    """The DiT block's first norm with its modulation sum in the same launch.

    Equals ``mod = modulation + t_mod`` (bf16, [B, 6, D]) followed by
    ``fused_ln_modulate(x, mod[:, 1:2], mod[:, 0:1], eps, emit_fp8=True)`` bit for bit
    (integrate.py:154-158).  modulation [1, 6, D], t_mod [B, 6, D], both bf16.
    Returns (out, q8, scale, mod); out is None when want_out=False.
    """
    if not emit_fp8:
        raise ValueError("fused_ln_modulate_adaln: only the FP8-emitting form exists")
    _check(x, "fused_ln_modulate_adaln")
    B, L, D = x.shape
    if modulation.dtype != torch.bfloat16 or t_mod.dtype != torch.bfloat16:
        raise ValueError("fused_ln_modulate_adaln: modulation/t_mod must be bf16")
    if modulation.numel() != 6 * D or t_mod.shape != (B, 6, D):
        raise ValueError("fused_ln_modulate_adaln: modulation [1, 6, D], t_mod [B, 6, D]")
    assert x.is_contiguous() and modulation.is_contiguous() and t_mod.is_contiguous()
    out = torch.empty_like(x) if want_out else None
    mod = torch.empty((B, 6, D), dtype=torch.bfloat16, device=x.device)
    q8 = torch.empty((B * L, D), dtype=torch.float8_e4m3fn, device=x.device)
    qs = torch.empty((B * L,), dtype=torch.float32, device=x.device)
    _lib.call("fvb_ln_modulate_adaln", _lib.ptr(x), _lib.ptr(modulation), _lib.ptr(t_mod), B, L,
              D, float(eps), _lib.ptr(out), _lib.ptr(q8), _lib.ptr(qs), _lib.ptr(mod),
              _lib.stream_of(x))
    return out, q8, qs, mod


def fused_gate_add(x: torch.Tensor, gate: torch.Tensor | None, residual: torch.Tensor,
                   out: torch.Tensor | None = None):
    """x + gate * residual. x/residual [B, L, D] contiguous bf16; gate [B, 1, D] (None: x + r)."""
    _check(x, "fused_gate_add")
    B, L, D = x.shape
    assert x.is_contiguous() and residual.is_contiguous() and (gate is None or gate.is_contiguous())
    if residual.dtype != torch.bfloat16 or (gate is not None and gate.dtype != torch.bfloat16):
        raise ValueError("fused_gate_add: gate/residual must be bf16")
    if out is None:
        out = torch.empty_like(x)
    _lib.call("fvb_gate_add", _lib.ptr(x), _lib.ptr(gate), _lib.ptr(residual), B, L, D,
              _lib.ptr(out), _lib.stream_of(x))
    return out


def _fp8_bufs(rows, D, device):
    return (torch.empty((rows, D), dtype=torch.float8_e4m3fn, device=device),
            torch.empty((rows,), dtype=torch.float32, device=device))


def gate_add_ln_modulate(x, gate, residual, scale, shift, eps=1e-6, emit_fp8=False,
                         want_out=True):
    """fused_gate_add(x, gate, residual) followed by fused_ln_modulate of its result, in one
    pass over the residual stream (bitwise the two calls).  gate [B, 1, D] or None.
    Returns (x_new, out) or, with emit_fp8, (x_new, out, q8, scale); out is None when
    want_out=False."""
    _check(x, "gate_add_ln_modulate")
    B, L, D = x.shape
    for t in (x, residual, scale, shift) + ((gate,) if gate is not None else ()):
        if not t.is_contiguous() or t.dtype != torch.bfloat16:
            raise ValueError("gate_add_ln_modulate: tensors must be contiguous bf16")
    if not want_out and not emit_fp8:
        raise ValueError("gate_add_ln_modulate: want_out=False needs emit_fp8=True")
    x_new = torch.empty_like(x)
    out = torch.empty_like(x) if want_out else None
    q8, qs = _fp8_bufs(B * L, D, x.device) if emit_fp8 else (None, None)
    _lib.call("fvb_gate_add_ln_modulate", _lib.ptr(x), _lib.ptr(gate), _lib.ptr(residual),
              _lib.ptr(x_new), _lib.ptr(scale), _lib.ptr(shift), B, L, D, float(eps),
              _lib.ptr(out), _lib.ptr(q8), _lib.ptr(qs), _lib.stream_of(x))
    return (x_new, out, q8, qs) if emit_fp8 else (x_new, out)


def gate_add_layer_norm(x, gate, residual, weight, bias, eps=1e-6, emit_fp8=False, want_out=True):
    """fused_gate_add(x, gate, residual) followed by layer_norm(weight, bias) of its result,
    in one pass (bitwise the two calls).  Returns as gate_add_ln_modulate."""
    _check(x, "gate_add_layer_norm")
    B, L, D = x.shape
    for t in (x, residual) + ((gate,) if gate is not None else ()):
        if not t.is_contiguous() or t.dtype != torch.bfloat16:
            raise ValueError("gate_add_layer_norm: tensors must be contiguous bf16")
    if not want_out and not emit_fp8:
        raise ValueError("gate_add_layer_norm: want_out=False needs emit_fp8=True")
    w = weight.to(torch.bfloat16).contiguous() if weight is not None else None
    b = bias.to(torch.bfloat16).contiguous() if bias is not None else None
    x_new = torch.empty_like(x)
    out = torch.empty_like(x) if want_out else None
    q8, qs = _fp8_bufs(B * L, D, x.device) if emit_fp8 else (None, None)
    _lib.call("fvb_gate_add_layer_norm", _lib.ptr(x), _lib.ptr(gate), _lib.ptr(residual),
              _lib.ptr(x_new), _lib.ptr(w), _lib.ptr(b), B, L, D, float(eps), _lib.ptr(out),
              _lib.ptr(q8), _lib.ptr(qs), _lib.stream_of(x))
    return (x_new, out, q8, qs) if emit_fp8 else (x_new, out)


def layer_norm(x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None,
               eps: float = 1e-6, out: torch.Tensor | None = None, emit_fp8: bool = False):
    """torch.nn.LayerNorm semantics (fp32 math, one bf16 rounding) over the last dim.

    emit_fp8=True also returns the output's per-token FP8 codes [rows, D] and scales [rows]
    (what quantize_fp8(out, "token") gives), computed in the same pass:
    returns (out, q8, scale)."""
    _check(x, "layer_norm")
    D = x.shape[-1]
    x = x.contiguous()
    rows = x.numel() // D
    w = weight.to(torch.bfloat16).contiguous() if weight is not None else None
    b = bias.to(torch.bfloat16).contiguous() if bias is not None else None
    if out is None:
        out = torch.empty_like(x)
    q8 = qs = None
    if emit_fp8:
        q8 = torch.empty((rows, D), dtype=torch.float8_e4m3fn, device=x.device)
        qs = torch.empty((rows,), dtype=torch.float32, device=x.device)
    _lib.call("fvb_layer_norm", _lib.ptr(x), _lib.ptr(w), _lib.ptr(b), rows, D, float(eps),
              _lib.ptr(out), _lib.ptr(q8), _lib.ptr(qs), _lib.stream_of(x))
    if emit_fp8:
        return out, q8, qs
    return out
