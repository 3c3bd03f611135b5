"""Stand-in for upstream ``diffsynth.models.wan_video_dit`` (FlashVSR v1.1 @ cf910c6).

``enable(pipe)`` patches the DiT module of a FlashVSR checkout.  When that
checkout is not installed (this repository's tests, ``smoke()`` and the
benchmark), this module provides the same names with the same signatures and
stock semantics, restated from the upstream interface that the reference's
integrate.py relies on (integrate.py:47-184, :187-214): ``RMSNorm``,
``modulate``, ``rope_apply``, ``precompute_freqs_cis_3d``,
``WindowPartition3D``, ``build_local_block_mask_shifted_vec_normal_slide``,
``generate_draft_block_mask``, ``SelfAttention``, ``CrossAttention``,
``DiTBlock``.  Model-level helpers (``WanDiT``, ``DiTPipe``) run a streaming
chunk through N blocks with per-block KV caches, the way the FlashVSR Tiny
pipeline drives its DiT.  Weights are random-init (no checkpoints here).

Everything in this file is eager PyTorch; after ``enable()`` the hot forwards
are replaced by the sm_100a kernels of this package.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

# which keep-mask rule generate_draft_block_mask / the fused path applies:
#   "draft"  - the FlashVSR selection (window-mean scores, local mask, joint top-k)
#   "causal" - the benchmark configuration's causal top-k rule
MASK_RULE = "draft"
CAUSAL_RATIO = 0.25


def modulate(x, shift, scale):
    return x * (1 + scale) + shift


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        dtype = x.dtype
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return y.to(dtype) * self.weight


def precompute_freqs_cis(dim, end=1024, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64)[: dim // 2] / dim))
    ang = torch.outer(torch.arange(end, dtype=torch.float64), inv)
    return torch.polar(torch.ones_like(ang), ang)


def precompute_freqs_cis_3d(dim, end=1024, theta=10000.0):
    third = dim // 3
    return (precompute_freqs_cis(dim - 2 * third, end, theta),
            precompute_freqs_cis(third, end, theta), precompute_freqs_cis(third, end, theta))


def grid_freqs(freqs3d, f, h, w, f0=0):
    tf, th, tw = freqs3d
    return torch.cat([
        tf[f0:f0 + f].view(f, 1, 1, -1).expand(f, h, w, -1),
        th[:h].view(1, h, 1, -1).expand(f, h, w, -1),
        tw[:w].view(1, 1, w, -1).expand(f, h, w, -1),
    ], dim=-1).reshape(f * h * w, 1, -1)


def rope_apply(x, freqs, num_heads):
    B, S, C = x.shape
    xc = torch.view_as_complex(x.to(torch.float64).reshape(B, S, num_heads, -1, 2))
    out = torch.view_as_real(xc * freqs.to(xc.device)).flatten(2)
    return out.to(x.dtype)


class WindowPartition3D:
    @staticmethod
    def partition(x, win):
        B, Fr, H, W, C = x.shape
        wf, wh, ww = win
        t = x.view(B, Fr // wf, wf, H // wh, wh, W // ww, ww, C).permute(0, 1, 3, 5, 2, 4, 6, 7)
        return t.contiguous().view(-1, wf * wh * ww, C)

    @staticmethod
    def reverse(windows, win, orig):
        Fr, H, W = orig
        wf, wh, ww = win
        C = windows.shape[-1]
        t = windows.view(-1, Fr // wf, H // wh, W // ww, wf, wh, ww, C).permute(0, 1, 4, 2, 5, 3, 6, 7)
        return t.contiguous().view(-1, Fr, H, W, C)


def build_local_block_mask_shifted_vec_normal_slide(bh, bw, local_h, local_w, include_self=True,
                                                    device=None):
    idx = torch.arange(bh * bw, device=device)
    r, c = idx // bw, idx % bw
    r0 = r - local_h // 2
    c0 = c - local_w // 2
    in_r = (r[None, :] >= r0[:, None]) & (r[None, :] <= r0[:, None] + local_h - 1)
    in_c = (c[None, :] >= c0[:, None]) & (c[None, :] <= c0[:, None] + local_w - 1)
    m = in_r & in_c
    if not include_self:
        m &= ~torch.eye(bh * bw, dtype=torch.bool, device=device)
    return m


def generate_draft_block_mask(batch_size, nheads, seqlen, q_w, k_w, topk=10, local_attn_mask=None):
    """[B, H, NQ, NK] bool keep mask (the selection lcsa/reference.py:37-64 restates)."""
    if MASK_RULE == "causal":
        return causal_block_mask(nheads, q_w, k_w, per_row=q_w.shape[0] // seqlen)[None]
    NQ, S, C = q_w.shape
    NK = k_w.shape[0]
    d = C // nheads
    aq = q_w.mean(dim=1).view(NQ, nheads, d).transpose(0, 1)
    ak = k_w.mean(dim=1).view(NK, nheads, d).transpose(0, 1)
    scores = torch.matmul(aq, ak.transpose(1, 2)) / math.sqrt(d)
    sq, sk = local_attn_mask.shape
    lm = local_attn_mask.repeat(NQ // sq, NK // sk)
    scores = scores.masked_fill(~lm[None], float("-inf"))
    prob = torch.softmax(scores, dim=-1)
    flat = prob.reshape(nheads * seqlen, (NQ // seqlen) * NK)
    k = min(flat.shape[1] - 1, topk)
    thr = torch.topk(flat, k=k + 1, dim=1).values[:, -1:]
    return (flat > thr).reshape(nheads, NQ, NK)[None].expand(batch_size, -1, -1, -1)


def causal_block_mask(nheads, q_w, k_w, per_row, ratio=None):
    """Eager form of the benchmark's causal top-k keep rule (see lcsa.causal_topk_mask)."""
    ratio = CAUSAL_RATIO if ratio is None else ratio
    NQ, S, C = q_w.shape
    NK = k_w.shape[0]
    d = C // nheads
    aq = q_w.float().mean(1).view(NQ, nheads, d).transpose(0, 1)
    ak = k_w.float().mean(1).view(NK, nheads, d).transpose(0, 1)
    sc = torch.matmul(aq, ak.transpose(1, 2))
    cache_rows = (NK - NQ) // per_row
    keep = torch.zeros(nheads, NQ, NK, dtype=torch.bool, device=q_w.device)
    for i in range(NQ):
        row = cache_rows + i // per_row
        keep[:, i, row * per_row:(row + 1) * per_row] = True
        npast = row * per_row
        nsel = int(math.floor(ratio * npast))
        if nsel:
            top = torch.topk(sc[:, i, :npast], nsel, dim=-1).indices
            keep[:, i].scatter_(1, top, True)
    return keep


class BlockSparseAttention(nn.Module):
    """Calls block_sparse_attn_func the way FlashVSR's DiT does (varlen, batch 1)."""

    def __init__(self, num_heads):
        super().__init__()
        self.num_heads = num_heads

    def forward(self, q, k, v, attention_mask):
        from block_sparse_attn import block_sparse_attn_func
        B, Lq, C = q.shape
        n = self.num_heads
        d = C // n
        Lk = k.shape[1]
        dev = q.device
        cu_q = torch.tensor([0, Lq], dtype=torch.int32, device=dev)
        cu_k = torch.tensor([0, Lk], dtype=torch.int32, device=dev)
        head_mask_type = torch.ones(n, dtype=torch.int32, device=dev)
        out = block_sparse_attn_func(q.reshape(Lq, n, d), k.reshape(Lk, n, d), v.reshape(Lk, n, d),
                                     cu_q, cu_k, head_mask_type, None, attention_mask, Lq, Lk,
                                     0.0, False, None, False)
        return out.reshape(B, Lq, C)


class DenseAttention(nn.Module):
    def __init__(self, num_heads):
        super().__init__()
        self.num_heads = num_heads

    def forward(self, q, k, v):
        B, Lq, C = q.shape
        n = self.num_heads
        qh = q.view(B, Lq, n, -1).transpose(1, 2)
        kh = k.view(B, k.shape[1], n, -1).transpose(1, 2)
        vh = v.view(B, v.shape[1], n, -1).transpose(1, 2)
        return F.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(B, Lq, C)


class SelfAttention(nn.Module):
    def __init__(self, dim, num_heads, eps=1e-6):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = RMSNorm(dim, eps=eps)
        self.norm_k = RMSNorm(dim, eps=eps)
        self.attn = BlockSparseAttention(num_heads)
        self.local_attn_mask = None
        self.local_attn_mask_h = None
        self.local_attn_mask_w = None
        self.local_range = None

    def forward(self, x, freqs, f=None, h=None, w=None, local_num=None, topk=None,
                train_img=False, block_id=None, kv_len=None, is_full_block=False,
                is_stream=False, pre_cache_k=None, pre_cache_v=None, local_range=9):
        B, L, D = x.shape
        q = rope_apply(self.norm_q(self.q(x)), freqs, self.num_heads)
        k = rope_apply(self.norm_k(self.k(x)), freqs, self.num_heads)
        v = self.v(x)
        win = (2, 8, 8)
        q_w = WindowPartition3D.partition(q.view(B, f, h, w, D), win)
        k_w = WindowPartition3D.partition(k.view(B, f, h, w, D), win)
        v_w = WindowPartition3D.partition(v.view(B, f, h, w, D), win)
        one_len = k_w.shape[0] // B // (f // win[0])
        if pre_cache_k is not None and pre_cache_v is not None:
            k_w = torch.cat([pre_cache_k, k_w], dim=0)
            v_w = torch.cat([pre_cache_v, v_w], dim=0)
        if self.local_attn_mask is None or self.local_attn_mask_h != h // 8 \
                or self.local_attn_mask_w != w // 8 or self.local_range != local_range:
            self.local_attn_mask = build_local_block_mask_shifted_vec_normal_slide(
                h // 8, w // 8, local_range, local_range, include_self=True, device=k_w.device)
            self.local_attn_mask_h, self.local_attn_mask_w = h // 8, w // 8
            self.local_range = local_range
        mask = generate_draft_block_mask(B, self.num_heads, f // win[0], q_w, k_w, topk=topk,
                                         local_attn_mask=self.local_attn_mask)
        o = self.attn(q_w.reshape(B, -1, D), k_w.reshape(B, -1, D), v_w.reshape(B, -1, D), mask)
        if kv_len is not None and k_w.shape[0] // one_len > kv_len:
            cache_k, cache_v = k_w[one_len:], v_w[one_len:]
        else:
            cache_k, cache_v = k_w, v_w
        o = WindowPartition3D.reverse(o.reshape(-1, win[0] * win[1] * win[2], D), win, (f, h, w))
        o = self.o(o.reshape(B, L, D))
        if is_stream:
            return o, cache_k, cache_v
        return o


class CrossAttention(nn.Module):
    def __init__(self, dim, num_heads, eps=1e-6):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = RMSNorm(dim, eps=eps)
        self.norm_k = RMSNorm(dim, eps=eps)
        self.attn = DenseAttention(num_heads)
        self.cache_k = None
        self.cache_v = None

    @torch.no_grad()
    def init_cache(self, ctx):
        self.cache_k = self.norm_k(self.k(ctx))
        self.cache_v = self.v(ctx)

    def forward(self, x, y, is_stream=False):
        q = self.norm_q(self.q(x))
        return self.o(self.attn(q, self.cache_k, self.cache_v))


class GateModule(nn.Module):
    def forward(self, x, gate, residual):
        return x + gate * residual


class DiTBlock(nn.Module):
    def __init__(self, dim, num_heads, ffn_dim, eps=1e-6):
        super().__init__()
        self.self_attn = SelfAttention(dim, num_heads, eps)
        self.cross_attn = CrossAttention(dim, num_heads, eps)
        self.norm1 = nn.LayerNorm(dim, eps=eps, elementwise_affine=False)
        self.norm2 = nn.LayerNorm(dim, eps=eps, elementwise_affine=False)
        self.norm3 = nn.LayerNorm(dim, eps=eps)
        self.ffn = nn.Sequential(nn.Linear(dim, ffn_dim), nn.GELU(approximate="tanh"),
                                 nn.Linear(ffn_dim, dim))
        self.modulation = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)
        self.gate = GateModule()

    def forward(self, x, context, t_mod, freqs, f, h, w, local_num=None, topk=None,
                train_img=False, block_id=None, kv_len=None, is_full_block=False,
                is_stream=False, pre_cache_k=None, pre_cache_v=None, local_range=9):
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (
            self.modulation.to(dtype=t_mod.dtype, device=t_mod.device) + t_mod).chunk(6, dim=1)
        a, ck, cv = self.self_attn(modulate(self.norm1(x), shift_msa, scale_msa), freqs, f, h, w,
                                   local_num, topk, train_img, block_id, kv_len=kv_len,
                                   is_full_block=is_full_block, is_stream=True,
                                   pre_cache_k=pre_cache_k, pre_cache_v=pre_cache_v,
                                   local_range=local_range)
        x = self.gate(x, gate_msa, a)
        x = x + self.cross_attn(self.norm3(x), context, is_stream=is_stream)
        x = self.gate(x, gate_mlp, self.ffn(modulate(self.norm2(x), shift_mlp, scale_mlp)))
        if is_stream:
            return x, ck, cv
        return x


# ----------------------------------------------------------------------------- model level
class WanDiT(nn.Module):
    """The DiT trunk FlashVSR-Tiny streams through: N DiTBlocks + RoPE tables."""

    def __init__(self, num_layers=30, dim=1536, num_heads=12, ffn_dim=8960, eps=1e-6):
        super().__init__()
        self.dim, self.num_heads, self.ffn_dim = dim, num_heads, ffn_dim
        self.blocks = nn.ModuleList([DiTBlock(dim, num_heads, ffn_dim, eps) for _ in range(num_layers)])
        self.freqs = precompute_freqs_cis_3d(dim // num_heads)

    @torch.no_grad()
    def init_random(self, seed=0, std=0.02):
        """N(0, std) linears, N(1, 0.1) norm weights, N(0, 1) modulation (benchmark config)."""
        g = torch.Generator().manual_seed(seed)
        for name, p in self.named_parameters():
            if name.endswith("modulation"):
                t = torch.randn(p.shape, generator=g)
            elif ".norm" in name and name.endswith("weight"):
                t = 1 + 0.1 * torch.randn(p.shape, generator=g)
            elif ".norm" in name and name.endswith("bias"):
                t = 0.1 * torch.randn(p.shape, generator=g)
            else:
                t = torch.randn(p.shape, generator=g) * std
            p.copy_(t.to(p.dtype))
        return self

    @torch.no_grad()
    def init_cross_kv(self, context):
        for blk in self.blocks:
            blk.cross_attn.init_cache(context)

    def chunk_freqs(self, f, h, w, f0=0, device=None):
        fr = grid_freqs(self.freqs, f, h, w, f0)
        return fr.to(device) if device is not None else fr

    @torch.no_grad()
    def forward_chunk(self, x, t_mod, freqs, fhw, caches=None, topk=None, kv_len=3, local_range=9):
        """One streaming chunk through every block.  caches: list of (k, v) or None per block.
        Returns (x, new_caches)."""
        f, h, w = fhw
        new = []
        for i, blk in enumerate(self.blocks):
            ck = cv = None
            if caches is not None and caches[i] is not None:
                ck, cv = caches[i]
            x, k2, v2 = blk(x, None, t_mod, freqs, f, h, w, topk=topk, kv_len=kv_len,
                            is_stream=True, pre_cache_k=ck, pre_cache_v=cv, local_range=local_range)
            new.append((k2, v2))
        return x, new


class DiTPipe:
    """Minimal pipeline object with the attributes enable() touches."""

    def __init__(self, dit: WanDiT):
        self.dit = dit

    def denoising_model(self):
        return self.dit
