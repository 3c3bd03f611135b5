"""The DiT block composed from the reference's own GPU ops, for block-level comparisons (test
infrastructure, not collected by pytest).

The ops are the reference package's (flashvsr_sm89_ops, pip-installed into baseline/_ref):
its Triton kernels (quantize_fp8, fused_ln_modulate, fused_gate_add, fused_rms_rope,
fused_gelu_quant_fp8 inside FP8FFN, the LCSA block-sparse attention) and its cuBLASLt
torch._scaled_mm through FP8Linear, with per-tensor scales as the reference has them.
The glue between them is the oracle block's (oracle/wan.py: window order, KV cache, keep
mask, the stock LayerNorm for norm3, the upstream RMSNorm for the cached cross K), and the
cross-attention over the context runs on torch's fused GPU attention as upstream leaves it.
"""
from __future__ import annotations

import os
import sys

import torch
import torch.nn.functional as F

from oracle import ops as O
from oracle import wan as OW

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_reference():
    """The reference package from baseline/_ref, or None when it is not installed.  Importing
    it installs its own block_sparse_attn stand-in; the module already registered under that
    name (this pack's) is put back so other tests keep seeing it."""
    if not os.path.isdir(os.path.join(REF_DIR, "flashvsr_sm89_ops")):
        return None
    saved = sys.modules.get("block_sparse_attn")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import flashvsr_sm89_ops as R
        from flashvsr_sm89_ops.lcsa.triton_lcsa import block_sparse_attention
    except Exception:  # noqa: BLE001  (no Triton / no GPU: no reference path)
        return None
    finally:
        if saved is not None:
            sys.modules["block_sparse_attn"] = saved
    R.block_sparse_attention = block_sparse_attention
    return R


def _linear(wb, R):
    w, b = wb
    lin = torch.nn.Linear(w.shape[1], w.shape[0], device=w.device, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(b)
    return R.FP8Linear(lin)


class RefGPUBlock:
    """One DiT block on the reference's GPU ops; P: bf16 block params on the GPU
    (oracle.wan.params_from_state_dict)."""

    def __init__(self, R, P, heads=12):
        self.R, self.P, self.heads = R, P, heads
        self.lin = {(part, n): _linear(P[part][n], R) for part in ("self", "cross")
                    for n in ("q", "k", "v", "o")}
        self.ffn = R.FP8FFN(_linear(P["ffn0"], R), _linear(P["ffn2"], R))

    def cross_kv(self, ctx):
        k = OW.rmsnorm_stock(self.lin["cross", "k"](ctx), self.P["cross"]["norm_k"])
        return k.reshape(-1, k.shape[-1]), self.lin["cross", "v"](ctx).reshape(-1, k.shape[-1])

    @torch.no_grad()
    def __call__(self, x, t_mod, freqs, fhw, ctx_kv, mask_fn, cache, eps=1e-6):
        R, P, H = self.R, self.P, self.heads
        B, L, D = x.shape
        f, h, w = fhw
        mod = (P["modulation"] + t_mod).chunk(6, dim=1)
        sh1, sc1, g1, sh2, sc2, g2 = [m.contiguous() for m in mod]
        xin = R.fused_ln_modulate(x, sc1, sh1, eps=eps)
        q = R.fused_rms_rope(self.lin["self", "q"](xin), P["self"]["norm_q"], freqs, eps=eps)
        k = R.fused_rms_rope(self.lin["self", "k"](xin), P["self"]["norm_k"], freqs, eps=eps)
        v = self.lin["self", "v"](xin)
        q_w = O.window_partition(q.view(B, f, h, w, D))
        k_w = O.window_partition(k.view(B, f, h, w, D))
        v_w = O.window_partition(v.view(B, f, h, w, D))
        if cache is not None:
            k_w = torch.cat([cache[0], k_w])
            v_w = torch.cat([cache[1], v_w])
        keep = mask_fn(q_w, k_w).to(x.device)
        o_w = R.block_sparse_attention(q_w.reshape(1, -1, D), k_w.reshape(1, -1, D),
                                       v_w.reshape(1, -1, D), keep).view(q_w.shape)
        o = O.window_reverse(o_w, (2, 8, 8), fhw, B).reshape(B, L, D)
        x = R.fused_gate_add(x, g1, self.lin["self", "o"](o).contiguous())
        n3 = F.layer_norm(x, (D,), P["norm3"][0], P["norm3"][1], eps)
        cq = R.fused_rms_rope(self.lin["cross", "q"](n3), P["cross"]["norm_q"], None, eps=eps,
                              rope=False)
        qh = cq.view(B, L, H, D // H).transpose(1, 2)
        kh = ctx_kv[0].view(1, -1, H, D // H).transpose(1, 2)
        vh = ctx_kv[1].view(1, -1, H, D // H).transpose(1, 2)
        co = F.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(B, L, D)
        x = x + self.lin["cross", "o"](co)
        xin = R.fused_ln_modulate(x.contiguous(), sc2, sh2, eps=eps)
        return R.fused_gate_add(x.contiguous(), g2, self.ffn(xin).contiguous())
