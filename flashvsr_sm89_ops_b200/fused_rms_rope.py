"""Fused RMSNorm + 3-D RoPE on the sm_100a library.

Drop-in for ``flashvsr_sm89_ops.fused_rms_rope`` (fused_rms_rope.py:58-83):
same signature ``fused_rms_rope(x, weight, freqs_cis, eps, rope, head_dim)``,
same numerics (fp32 reduction, bf16 round of x*rrms before the weight,
interleaved pair rotation in fp32, one final bf16 rounding).  The complex
``freqs_cis`` -> (cos, sin) split is cached per tensor, so repeated calls with
the same freqs (30 blocks x 2 norm sites) pay it once instead of ~0.1 ms per call.
"""
from __future__ import annotations

import torch

from . import _lib

_COS_SIN_CACHE: dict = {}


def freqs_cos_sin(freqs: torch.Tensor):
    """complex [..., S, half] -> (cos, sin) fp32 [S, half], cached by tensor identity.

    The semantics of _freqs_cos_sin (fused_rms_rope.py:58-63).  A (cos, sin) tuple is
    passed through unchanged.
    """
    if isinstance(freqs, (tuple, list)):
        return freqs[0], freqs[1]
    key = (freqs.data_ptr(), freqs._version, tuple(freqs.shape), str(freqs.device))
    hit = _COS_SIN_CACHE.get(key)
    if hit is not None and hit[0] is freqs:
        return hit[1], hit[2]
    fr = torch.view_as_real(freqs.reshape(-1, freqs.shape[-1]))
    cos = fr[..., 0].float().contiguous()
    sin = fr[..., 1].float().contiguous()
    if len(_COS_SIN_CACHE) > 64:
        _COS_SIN_CACHE.clear()
    _COS_SIN_CACHE[key] = (freqs, cos, sin)
    return cos, sin


def rms_rope_rows(x2: torch.Tensor, weight: torch.Tensor, cos, sin, L: int, eps: float,
                  rope: bool, head_dim: int, out: torch.Tensor | None = None,
                  row_map: torch.Tensor | None = None) -> torch.Tensor:
    """Row-level entry: x2 [rows, D] bf16 (row pitch may exceed D), output [rows, D].

    row_map (int32 [rows]) writes input row r to output row row_map[r].
    """
    _lib.require_cuda(x2, weight)
    rows, D = x2.shape
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    ld = x2.stride(0)
    if weight.dtype != torch.bfloat16:
        weight = weight.to(torch.bfloat16)
    weight = weight.contiguous()
    if out is None:
        out = torch.empty((rows, D), dtype=torch.bfloat16, device=x2.device)
    _lib.call("fvb_rms_rope", _lib.ptr(x2), ld, _lib.ptr(weight),
              _lib.ptr(cos) if rope else None, _lib.ptr(sin) if rope else None,
              rows, L, D, head_dim, float(eps), 1 if rope else 0, _lib.ptr(row_map),
              _lib.ptr(out), _lib.stream_of(x2))
    return out


def qkv_rope_window(qkv: torch.Tensor, w_q: torch.Tensor, w_k: torch.Tensor, cos, sin, L: int,
                    eps_q: float, eps_k: float, head_dim: int, row_map: torch.Tensor | None,
                    out_q: torch.Tensor, out_k: torch.Tensor, out_v: torch.Tensor):
    """q, k and v of the self-attention from the fused projection output qkv [rows, 3D] in
    one launch: out_q / out_k = RMSNorm + RoPE of the q / k thirds (as rms_rope_rows), out_v
    = the v third, every row r written to row row_map[r] of its output (each [rows, D])."""
    _lib.require_cuda(qkv, w_q, w_k)
    rows, D3 = qkv.shape
    if qkv.stride(1) != 1 or D3 % 3:
        raise ValueError("qkv_rope_window: qkv must be [rows, 3D] with unit column stride")
    D = D3 // 3
    for o in (out_q, out_k, out_v):
        if o.shape[0] != rows or o.shape[-1] != D or not o.is_contiguous():
            raise ValueError("qkv_rope_window: outputs must be contiguous [rows, D]")
    w_q = w_q.to(torch.bfloat16).contiguous()
    w_k = w_k.to(torch.bfloat16).contiguous()
    _lib.call("fvb_qkv_rope_window", _lib.ptr(qkv), qkv.stride(0), _lib.ptr(w_q), _lib.ptr(w_k),
              _lib.ptr(cos), _lib.ptr(sin), rows, L, D, head_dim, float(eps_q), float(eps_k),
              _lib.ptr(row_map), _lib.ptr(out_q), _lib.ptr(out_k), _lib.ptr(out_v),
              _lib.stream_of(qkv))
    return out_q, out_k, out_v


def fused_rms_rope(x: torch.Tensor, weight: torch.Tensor, freqs_cis, eps: float = 1e-6,
                   rope: bool = True, head_dim: int = 128):
    """x [B, L, D] bf16 -> RMSNorm(weight) -> [x RoPE]; freqs_cis complex [L, 1, head_dim/2]."""
    B, L, D = x.shape
    if x.dtype != torch.bfloat16:
        raise ValueError(f"fused_rms_rope: expected bf16, got {x.dtype}")
    x2 = x.reshape(B * L, D)
    if rope:
        cos, sin = freqs_cos_sin(freqs_cis)
        if cos.device != x.device:
            cos, sin = cos.to(x.device), sin.to(x.device)
        if cos.shape[0] != L:
            raise ValueError(f"fused_rms_rope: freqs cover {cos.shape[0]} positions, need {L}")
    else:
        cos = sin = None
    out = rms_rope_rows(x2, weight, cos, sin, L, eps, rope, head_dim)
    return out.reshape(B, L, D)
