"""CPU restatement of a Wan2.1-style DiT block as the FlashVSR operator pack runs it
(test infrastructure only; "parity unpinned" against upstream DiffSynth, which is
not in the reference tree).

The block follows the stock branches the reference keeps beside its fused ones
(flashvsr_sm89_ops/integrate.py:47-124 self-attention, :132-143 cross-attention,
:151-182 block) with the pack's op semantics substituted (ops.ln_modulate,
ops.rms_rope, ops.gate_add, FP8 linears, block-sparse attention), which is the
computation ``enable(pipe)`` installs.
"""
from __future__ import annotations


import torch

from . import ops as O


# ----------------------------------------------------------------------------- RoPE
def rope_freqs_1d(dim: int, end: int = 1024, theta: float = 10000.0) -> torch.Tensor:
    """Complex128 [end, dim/2]: position p, pair i -> exp(1j * p * theta^(-2i/dim))
    (upstream precompute_freqs_cis, float64)."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64)[: dim // 2] / dim))
    ang = torch.arange(end, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.polar(torch.ones_like(ang), ang)


def rope_freqs_3d(head_dim: int = 128, end: int = 1024, theta: float = 10000.0):
    """(f, h, w) tables with head_dim - 2*(head_dim//3) / head_dim//3 / head_dim//3 dims
    (44/42/42 for head_dim 128; upstream precompute_freqs_cis_3d)."""
    third = head_dim // 3
    return (rope_freqs_1d(head_dim - 2 * third, end, theta), rope_freqs_1d(third, end, theta),
            rope_freqs_1d(third, end, theta))


def grid_freqs(f: int, h: int, w: int, f0: int = 0, head_dim: int = 128) -> torch.Tensor:
    """[f*h*w, 1, head_dim/2] complex128 for a (f, h, w) token grid starting at frame f0
    (the WanModel.forward construction: f, h, w tables broadcast and concatenated)."""
    tf, th, tw = rope_freqs_3d(head_dim)
    a = tf[f0:f0 + f].view(f, 1, 1, -1).expand(f, h, w, -1)
    b = th[:h].view(1, h, 1, -1).expand(f, h, w, -1)
    c = tw[:w].view(1, 1, w, -1).expand(f, h, w, -1)
    return torch.cat([a, b, c], dim=-1).reshape(f * h * w, 1, -1)


# ----------------------------------------------------------------------------- params
LINEARS_SELF = ("q", "k", "v", "o")
LINEARS_CROSS = ("q", "k", "v", "o")


def init_block_params(gen: torch.Generator, D: int = 1536, FF: int = 8960, std: float = 0.02):
    """Random-init block (N(0, std) weights and biases, fp32), RMS weights N(1, 0.1),
    modulation N(0, 1)/sqrt(D)-free N(0,1) as the benchmark configuration states."""
    def lin(n_out, n_in):
        return (torch.randn(n_out, n_in, generator=gen) * std, torch.randn(n_out, generator=gen) * std)

    P = {"modulation": torch.randn(1, 6, D, generator=gen)}
    for part in ("self", "cross"):
        P[part] = {n: lin(D, D) for n in ("q", "k", "v", "o")}
        P[part]["norm_q"] = 1 + 0.1 * torch.randn(D, generator=gen)
        P[part]["norm_k"] = 1 + 0.1 * torch.randn(D, generator=gen)
    P["norm3"] = (1 + 0.1 * torch.randn(D, generator=gen), 0.1 * torch.randn(D, generator=gen))
    P["ffn0"] = lin(FF, D)
    P["ffn2"] = lin(D, FF)
    return P


def to_bf16(P):
    if isinstance(P, dict):
        return {k: to_bf16(v) for k, v in P.items()}
    if isinstance(P, tuple):
        return tuple(to_bf16(v) for v in P)
    return P.to(torch.bfloat16)


class QLinear:
    """Oracle FP8 linear: weight codes/scales from ops.fp8_weight, forward ops.fp8_linear."""

    def __init__(self, wb, mode):
        w, b = wb
        self.q, self.s = O.fp8_weight(w.to(torch.bfloat16), "tensor" if mode == "tensor" else "channel")
        self.b = b.to(torch.bfloat16)
        self.mode = mode

    def __call__(self, x):
        return O.fp8_linear(x, self.q, self.s, self.b, self.mode)


def quantize_block(P, mode="token"):
    """bf16 params + oracle FP8 linears for every block linear (fp8_linear.py:45-67 parts)."""
    Q = to_bf16(P)
    for part in ("self", "cross"):
        for n in ("q", "k", "v", "o"):
            Q[part][n] = QLinear(P[part][n], mode)
    Q["ffn0"] = QLinear(P["ffn0"], mode)
    Q["ffn2"] = QLinear(P["ffn2"], mode)
    Q["mode"] = mode
    return Q


# ----------------------------------------------------------------------------- block
# the B200 attention kernel's lazy-rescale threshold (log2 units); 0 = the reference order
KERNEL_LAZY = 8.0
# "kernel": attention in the B200 kernel's evaluation order (parity tests of whole blocks);
# "reference": the reference's fp32 oracle (lcsa/reference.py:67-88), used when the
# reference's CPU path is timed (bench.py cpu_baseline / --impl reference)
ATTENTION = "kernel"


def rmsnorm_stock(x, weight, eps=1e-6):
    """Upstream Wan RMSNorm on bf16: bf16(x * rsqrt(mean(x^2) + eps)) * weight (a bf16 product)."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(torch.bfloat16)
    return y * weight.to(torch.bfloat16)


def cross_kv(Q, context, eps=1e-6):
    """Cached cross-attention K/V of a context (the pipeline's init_cross_kv, which runs the
    upstream norm_k, not the fused kernel)."""
    c = Q["cross"]
    k = rmsnorm_stock(c["k"](context), c["norm_k"], eps=eps)
    v = c["v"](context)
    return k.reshape(-1, k.shape[-1]), v.reshape(-1, v.shape[-1])


def self_attention(Q, x, cos, sin, fhw, mask_fn, nheads=12, cache=None, kv_len=None, eps=1e-6,
                   win=(2, 8, 8)):
    """integrate.py:47-124 (stock branch, pack ops).  Returns (out, (cache_k, cache_v))."""
    s = Q["self"]
    B, L, D = x.shape
    f, h, w = fhw
    q = O.rms_rope(s["q"](x), s["norm_q"], cos, sin, eps=eps, rope=True)
    k = O.rms_rope(s["k"](x), s["norm_k"], cos, sin, eps=eps, rope=True)
    v = s["v"](x)
    q_w = O.window_partition(q.view(B, f, h, w, D), win)
    k_w = O.window_partition(k.view(B, f, h, w, D), win)
    v_w = O.window_partition(v.view(B, f, h, w, D), win)
    one_len = k_w.shape[0] // B // (f // win[0])
    if cache is not None:
        k_w = torch.cat([cache[0], k_w], dim=0)
        v_w = torch.cat([cache[1], v_w], dim=0)
    keep = mask_fn(q_w, k_w)
    if ATTENTION == "reference":
        o_w = O.sparse_attention(q_w, k_w, v_w, keep).to(torch.bfloat16)
    else:
        o_w = O.sparse_attention_online(q_w, k_w, v_w, keep, lazy=KERNEL_LAZY).to(torch.bfloat16)
    if kv_len is not None and k_w.shape[0] // one_len > kv_len:
        new_cache = (k_w[one_len:], v_w[one_len:])
    else:
        new_cache = (k_w, v_w)
    o = O.window_reverse(o_w, win, fhw, B).reshape(B, L, D)
    return s["o"](o), new_cache


def cross_attention(Q, x, ctx_kv, nheads=12, eps=1e-6):
    """integrate.py:132-143: q = RMSNorm(q(x)) (no RoPE); dense attention over cached K/V."""
    c = Q["cross"]
    B, L, D = x.shape
    q = O.rms_rope(c["q"](x), c["norm_q"], rope=False, eps=eps)
    if ATTENTION == "reference":
        o = O.dense_attention(q.reshape(L, D), ctx_kv[0], ctx_kv[1], nheads).to(torch.bfloat16)
    else:
        o = O.dense_attention_online(q.reshape(L, D), ctx_kv[0], ctx_kv[1], nheads,
                                     lazy=KERNEL_LAZY).to(torch.bfloat16)
    return c["o"](o.reshape(B, L, D))


def block_forward(Q, x, t_mod, cos, sin, fhw, ctx_kv, mask_fn, nheads=12, cache=None, kv_len=None,
                  eps=1e-6):
    """DiTBlock.forward (integrate.py:151-182) with the pack's fused semantics."""
    mod = (Q["modulation"] + t_mod).chunk(6, dim=1)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = [m.contiguous() for m in mod]
    xin = O.ln_modulate(x, scale_msa, shift_msa, eps)
    a, new_cache = self_attention(Q, xin, cos, sin, fhw, mask_fn, nheads, cache, kv_len, eps)
    x = O.gate_add(x, gate_msa, a)
    n3 = O.layer_norm(x, Q["norm3"][0], Q["norm3"][1], eps)
    x = (x.float() + cross_attention(Q, n3, ctx_kv, nheads, eps).float()).to(torch.bfloat16)
    xin = O.ln_modulate(x, scale_mlp, shift_mlp, eps)
    h = Q["ffn0"](xin)
    qh, sh = O.gelu_quant_fp8(h.reshape(-1, h.shape[-1]), Q["mode"])
    f2 = Q["ffn2"]
    y = O.fp8_mm(qh, sh, f2.q, f2.s, f2.b).reshape(x.shape)
    x = O.gate_add(x, gate_mlp, y)
    return x, new_cache


def standin_state_dict(P):
    """Parameter names of a Wan DiTBlock (upstream layout) -> bf16 tensors of block params P."""
    sd = {"modulation": P["modulation"]}
    for part, prefix in (("self", "self_attn"), ("cross", "cross_attn")):
        for n in ("q", "k", "v", "o"):
            sd[f"{prefix}.{n}.weight"], sd[f"{prefix}.{n}.bias"] = P[part][n]
        sd[f"{prefix}.norm_q.weight"] = P[part]["norm_q"]
        sd[f"{prefix}.norm_k.weight"] = P[part]["norm_k"]
    sd["norm3.weight"], sd["norm3.bias"] = P["norm3"]
    sd["ffn.0.weight"], sd["ffn.0.bias"] = P["ffn0"]
    sd["ffn.2.weight"], sd["ffn.2.bias"] = P["ffn2"]
    return {k: v.to(torch.bfloat16) for k, v in sd.items()}


def params_from_state_dict(sd):
    """Inverse of standin_state_dict: a Wan DiTBlock state dict -> block params P (the
    tensors keep their dtype and device, so the oracle quantises the very weights the
    module holds)."""
    P = {"modulation": sd["modulation"]}
    for part, prefix in (("self", "self_attn"), ("cross", "cross_attn")):
        P[part] = {n: (sd[f"{prefix}.{n}.weight"], sd[f"{prefix}.{n}.bias"]) for n in ("q", "k", "v", "o")}
        P[part]["norm_q"] = sd[f"{prefix}.norm_q.weight"]
        P[part]["norm_k"] = sd[f"{prefix}.norm_k.weight"]
    P["norm3"] = (sd["norm3.weight"], sd["norm3.bias"])
    P["ffn0"] = (sd["ffn.0.weight"], sd["ffn.0.bias"])
    P["ffn2"] = (sd["ffn.2.weight"], sd["ffn.2.bias"])
    return P


def causal_mask_fn(nheads, per_row, ratio=0.25):
    return lambda q_w, k_w: O.causal_topk_mask(q_w, k_w, nheads, per_row, ratio)


def draft_mask_fn(nheads, fhw, topk, local_range=11):
    f, h, w = fhw
    local = O.local_block_mask(h // 8, w // 8, local_range)
    return lambda q_w, k_w: O.draft_block_mask(q_w, k_w, nheads, f // 2, local, topk)


def flops_per_token(D=1536, FF=8960):
    """Linear FLOPs per token per block: self qkvo 4*2*D^2, cross q,o 2*2*D^2, FFN 2*2*D*FF."""
    return 4 * 2 * D * D + 2 * 2 * D * D + 2 * 2 * D * FF


def attention_flops(kept_pairs, d=128, blk=128):
    return kept_pairs * 4 * blk * blk * d


def rel_l2(a, b):
    a = a.float().reshape(-1)
    b = b.float().reshape(-1)
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp(min=1e-30)).item()


def block_case(seed=0, f=2, h=16, w=24, cache_rows=3, D=1536, FF=8960, heads=12, ctx=512):
    """Seeded inputs of one streaming block step (CPU, bf16): params, x, t_mod, context, cache."""
    g = torch.Generator().manual_seed(seed)
    P = init_block_params(g, D, FF)
    x = torch.randn(1, f * h * w, D, generator=g).to(torch.bfloat16)
    t_mod = torch.randn(1, 6, D, generator=g).to(torch.bfloat16)
    context = torch.randn(1, ctx, D, generator=g).to(torch.bfloat16)
    per_row = (h // 8) * (w // 8)
    cache = None
    if cache_rows:
        cache = (torch.randn(cache_rows * per_row, 128, D, generator=g).to(torch.bfloat16),
                 torch.randn(cache_rows * per_row, 128, D, generator=g).to(torch.bfloat16))
    return P, x, t_mod, context, cache
