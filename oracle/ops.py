"""CPU restatement of the reference operator formulas (test infrastructure only).

Functions compute on the device of their inputs (CPU in the parity tests; the largest
block-level checks evaluate the same code on the GPU in fp32).  bf16 rounding points are placed
exactly where the reference kernels place them.  Citations are paths inside
aireet/flashvsr-sm89-ops.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

FP8_MAX = 448.0  # flashvsr_sm89_ops/fp8_quant.py:13
E4M3 = torch.float8_e4m3fn


def div_ieee(a, b):
    """a / b as the IEEE fp32 quotient on every device.  Evaluated in float64 and rounded to
    float32, which is exactly the correctly rounded fp32 quotient (binary64 carries more than
    2*24 + 2 bits, so the second rounding is innocuous).  A divisor given as a number is made
    a tensor first: torch's CUDA kernels turn a division by a host scalar into a multiply by
    its reciprocal, which is not the quotient (and moves exact e4m3 ties)."""
    if not torch.is_tensor(b):
        b = torch.tensor(float(b), dtype=torch.float64, device=a.device)
    return (a.double() / b.double()).float()


# ----------------------------------------------------------------------------- FP8
def quantize_fp8(x2: torch.Tensor, mode: str = "tensor"):
    """Activation quantisation of flashvsr_sm89_ops/fp8_quant.py:42-55 (kernels :16-35).

    amax = max|x| (fp32); s = max(amax, 1e-12)/448; q = e4m3(clamp(x/s, +-448)) with an
    fp32 IEEE divide and round-to-nearest-even; the returned scale is returned_scale(amax),
    i.e. amax/448 as a multiply by fl(1/448).
    mode "token" applies the same formula to each row (the per-token granularity the
    B200 pack adds; no reference counterpart beyond the formula).
    """
    xf = x2.float()
    if mode == "tensor":
        if xf.numel() == 0:
            return x2.to(E4M3), torch.zeros(1, device=xf.device)
        amax = xf.abs().amax().reshape(1)
    else:
        if xf.numel() == 0:
            return x2.to(E4M3), torch.zeros(xf.shape[0], device=xf.device)
        amax = xf.abs().amax(dim=-1)
    s = div_ieee(torch.clamp(amax, min=1e-12), FP8_MAX)
    sb = s if mode == "tensor" else s[:, None]
    q = torch.clamp(div_ieee(xf, sb), -FP8_MAX, FP8_MAX).to(E4M3)
    return q, returned_scale(amax)


# fp32 reciprocal of FP8_MAX, as torch forms it for a division of a CUDA tensor by a host scalar
INV_FP8_MAX = torch.tensor(1.0, dtype=torch.float32) / FP8_MAX


def returned_scale(amax):
    """The scale quantize_fp8 returns, `amax / FP8_MAX` (fp8_quant.py:54), as it evaluates on
    the reference's platform: torch divides a CUDA tensor by a host scalar as a multiply by
    the scalar's fp32 reciprocal, fl(amax * fl(1/448)).  Pinned by the reference's own
    quantize_fp8 run on a B200 (tests/golden/triton_b200.pt), whose returned scale differs
    from the IEEE quotient by one ulp for some amax; CPU torch divides exactly, so the
    product is spelled out."""
    return amax.float() * INV_FP8_MAX.to(amax.device)


def gelu_tanh(h: torch.Tensor) -> torch.Tensor:
    """GELU(tanh) with a bf16 result, the oracle fp8_ffn.py:7-10,24-30 targets."""
    return F.gelu(h, approximate="tanh")


def gelu_quant_fp8(h: torch.Tensor, mode: str = "tensor"):
    """fused_gelu_quant_fp8 (fp8_ffn.py:57-72) == quantize_fp8(gelu(h)) (its docstring :58-60)."""
    return quantize_fp8(gelu_tanh(h), mode)


def fp8_weight(w: torch.Tensor, mode: str = "tensor"):
    """One-time weight quantisation of FP8Linear.__init__ (fp8_linear.py:17-22).

    w_scale = (|w|.amax()/448).clamp(min=1e-12) (fp32); codes = (w / w_scale).to(e4m3),
    evaluated in the weight's own dtype exactly like the eager expression (a bf16 weight
    divides to bf16 before the e4m3 cast).  mode "channel": one scale per output row.
    """
    if mode == "tensor":
        s = (w.abs().amax() / FP8_MAX).clamp(min=1e-12).float()
        q = (w / s).to(E4M3)
        return q, s.reshape(1)
    s = (w.abs().amax(dim=1) / FP8_MAX).clamp(min=1e-12).float()
    q = (w / s[:, None]).to(E4M3)
    return q, s


def fp8_mm(qa, sa, qw, sw, bias=None):
    """FP8Linear._mm = torch._scaled_mm(x8, W.t(), scale_a, scale_b, bias, bf16) (fp8_linear.py:28-30).

    Restated as an fp32 product of the decoded codes, scaled per row of A and per row of
    W, plus bias, rounded once to bf16.
    """
    acc = qa.float() @ qw.float().t()
    sa_ = sa.reshape(-1, 1) if sa.numel() > 1 else sa.reshape(1, 1)
    sw_ = sw.reshape(1, -1) if sw.numel() > 1 else sw.reshape(1, 1)
    y = acc * (sa_ * sw_)
    if bias is not None:
        y = y + bias.float()
    return y.to(torch.bfloat16)


def fp8_linear(x, qw, sw, bias=None, act_mode="tensor"):
    """FP8Linear.forward (fp8_linear.py:32-42): quantise the activation, then _mm."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    qa, sa = quantize_fp8(x2, act_mode)
    y = fp8_mm(qa, sa, qw, sw, bias)
    return y.reshape(*shape[:-1], y.shape[-1])


def fp8_ffn(x, qw0, sw0, b0, qw2, sw2, b2, act_mode="tensor"):
    """FP8FFN.forward (fp8_ffn.py:84-96): quant -> mm0 -> GELU + quant -> mm2."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    qa, sa = quantize_fp8(x2, act_mode)
    h = fp8_mm(qa, sa, qw0, sw0, b0)
    qh, sh = gelu_quant_fp8(h, act_mode)
    out = fp8_mm(qh, sh, qw2, sw2, b2)
    return out.reshape(*shape[:-1], out.shape[-1])


# ----------------------------------------------------------------------------- norms
def freqs_cos_sin(freqs: torch.Tensor):
    """_freqs_cos_sin (fused_rms_rope.py:58-63): complex [..., S, half] -> fp32 cos, sin [S, half]."""
    fr = torch.view_as_real(freqs.reshape(-1, freqs.shape[-1]))
    return fr[..., 0].float().contiguous(), fr[..., 1].float().contiguous()


def rms_rope(x, weight, cos=None, sin=None, eps=1e-6, rope=True, head_dim=128):
    """_rms_rope_kernel (fused_rms_rope.py:21-55) for x [B, L, D] bf16.

    rrms = 1/sqrt(mean(x^2) + eps) (fp32); y = bf16(x * rrms) * w (fp32);
    pairs (2i, 2i+1) of each head: even -> y_e c - y_o s, odd -> y_o c + y_e s with
    (c, s) = cos/sin[l, i]; one bf16 rounding at the end.
    """
    B, L, D = x.shape
    xf = x.float()
    ms = div_ieee((xf * xf).sum(-1, keepdim=True), D)
    rrms = div_ieee(torch.ones_like(ms), torch.sqrt(ms + eps))
    y = (xf * rrms).to(torch.bfloat16).float() * weight.float()
    if not rope:
        return y.to(torch.bfloat16)
    half = head_dim // 2
    yp = y.view(B, L, D // head_dim, half, 2)
    c = cos.view(1, L, 1, half)
    s = sin.view(1, L, 1, half)
    ye, yo = yp[..., 0], yp[..., 1]
    oe = ye * c + yo * (-s)
    oo = yo * c + ye * s
    return torch.stack([oe, oo], dim=-1).view(B, L, D).to(torch.bfloat16)


def ln_modulate(x, scale, shift, eps=1e-6):
    """_ln_modulate_kernel (fused_adaln.py:22-42): LN without affine then modulate.

    xn = bf16((x - mean)/sqrt(var + eps)); y = bf16(bf16(xn * bf16(1 + scale)) + shift).
    x [B, L, D]; scale, shift [B, 1, D].  Note the argument order (scale before shift).
    """
    xf = x.float()
    D = x.shape[-1]
    mean = div_ieee(xf.sum(-1, keepdim=True), D)
    var = div_ieee(((xf - mean) ** 2).sum(-1, keepdim=True), D)
    xn = div_ieee(xf - mean, torch.sqrt(var + eps)).to(torch.bfloat16).float()
    one_plus = (1.0 + scale.float()).to(torch.bfloat16).float()
    y = (xn * one_plus).to(torch.bfloat16).float()
    return (y + shift.float()).to(torch.bfloat16)


def gate_add(x, gate, residual):
    """_gate_add_kernel (fused_adaln.py:45-57): bf16(x + bf16(g * r)), bitwise = eager x + g*r."""
    y = (gate.float() * residual.float()).to(torch.bfloat16).float()
    return (x.float() + y).to(torch.bfloat16)


def layer_norm(x, weight, bias, eps=1e-6):
    """torch.nn.LayerNorm on bf16 (the DiT block's norm3; eager in the reference)."""
    return F.layer_norm(x.float(), (x.shape[-1],), weight.float() if weight is not None else None,
                        bias.float() if bias is not None else None, eps).to(torch.bfloat16)


# ----------------------------------------------------------------------------- LCSA
def window_partition(x, win=(2, 8, 8)):
    """WindowPartition3D.partition (lcsa/reference.py:15-21): [B,F,H,W,C] -> [Nwin, wf*wh*ww, C]."""
    B, Fr, H, W, C = x.shape
    wf, wh, ww = win
    t = x.reshape(B, Fr // wf, wf, H // wh, wh, W // ww, ww, C)
    t = t.permute(0, 1, 3, 5, 2, 4, 6, 7)
    return t.reshape(-1, wf * wh * ww, C)


def window_reverse(xw, win, fhw, B=1):
    """Inverse of window_partition (upstream WindowPartition3D.reverse, integrate.py:117-120)."""
    Fr, H, W = fhw
    wf, wh, ww = win
    C = xw.shape[-1]
    t = xw.reshape(B, Fr // wf, H // wh, W // ww, wf, wh, ww, C)
    t = t.permute(0, 1, 4, 2, 5, 3, 6, 7)
    return t.reshape(B, Fr, H, W, C)


def local_block_mask(bh, bw, rng):
    """build_local_block_mask (lcsa/reference.py:24-34): window of side rng centred at each block."""
    idx = torch.arange(bh * bw)
    r, c = idx // bw, idx % bw
    r0 = r - rng // 2
    c0 = c - rng // 2
    in_r = (r[None, :] >= r0[:, None]) & (r[None, :] <= r0[:, None] + rng - 1)
    in_c = (c[None, :] >= c0[:, None]) & (c[None, :] <= c0[:, None] + rng - 1)
    return in_r & in_c


def draft_block_mask(q_w, k_w, nheads, q_temporal, local, topk):
    """Keep-mask selection of lcsa/reference.py:37-64 (= upstream generate_draft_block_mask).

    Window-mean pool (bf16 result) -> per-head scores / sqrt(d) (bf16) -> -inf outside the
    local mask tiled over time rows -> softmax over keys (bf16) -> per (head, query time
    row) the (k+1)-th largest probability of the flattened slab is the threshold; keep is
    strictly greater.  Returns [H, NQ, NK] bool.
    """
    NQ, _, C = q_w.shape
    NK = k_w.shape[0]
    d = C // nheads
    aq = q_w.mean(dim=1).reshape(NQ, nheads, d).permute(1, 0, 2)  # [H, NQ, d] bf16
    ak = k_w.mean(dim=1).reshape(NK, nheads, d).permute(1, 0, 2)
    scores = torch.matmul(aq, ak.transpose(1, 2)) / math.sqrt(d)
    sq, sk = local.shape
    lm = local.repeat(NQ // sq, NK // sk)
    scores = scores.masked_fill(~lm[None], float("-inf"))
    prob = torch.softmax(scores, dim=-1)
    per_row = NQ // q_temporal
    flat = prob.reshape(nheads * q_temporal, per_row * NK)
    k = min(flat.shape[1] - 1, topk)
    thr = torch.topk(flat, k=k + 1, dim=1).values[:, -1:]
    return (flat > thr).reshape(nheads, NQ, NK)


def block_mean_ordered(x_w):
    """fp32 window means [N, C] of x_w [N, 128, C] in one fixed summation order (the
    order the device pooling uses, so both give the same bits): partial sum g adds tokens
    g, g+4, ..., g+124 in turn; mean = ((p0 + p1) + (p2 + p3)) / 128."""
    xf = x_w.float()
    N, S, C = xf.shape
    g = xf.reshape(N, S // 4, 4, C)  # token 4*i + g
    p = torch.zeros(N, 4, C, dtype=torch.float32, device=xf.device)
    for i in range(S // 4):
        p = p + g[:, i]
    return ((p[:, 0] + p[:, 1]) + (p[:, 2] + p[:, 3])) / float(S)


def _dots_ordered(aq, ak):
    """[H, NQ, d] x [H, NK, d] -> [H, NQ, NK] fp32 dot products summed in ascending
    channel order, each product and each sum rounded on its own (no fused multiply-add)."""
    acc = torch.zeros(aq.shape[0], aq.shape[1], ak.shape[1], dtype=torch.float32, device=aq.device)
    for e in range(aq.shape[2]):
        acc = acc + aq[:, :, e, None] * ak[:, None, :, e]
    return acc


def draft_block_mask_ordered(q_w, k_w, nheads, q_temporal, local, topk):
    """draft_block_mask (lcsa/reference.py:37-64) with every fp32 reduction in one stated
    order, the contract the device builder meets bit for bit.  The rounding chain is the
    reference's: bf16 window means, bf16 scores, bf16 / sqrt(d) -> bf16, -inf outside the
    local mask, softmax to bf16, joint top-k per (head, query time row) with a strict `>`
    threshold.  The orders where the reference leaves them to torch: means as in
    block_mean_ordered; dots in ascending channel order; exp taken in double and rounded
    to fp32; the softmax total summed over keys in ascending order; prob = e / total."""
    NQ, _, C = q_w.shape
    NK = k_w.shape[0]
    d = C // nheads
    aq = block_mean_ordered(q_w).to(torch.bfloat16).float().reshape(NQ, nheads, d).permute(1, 0, 2)
    ak = block_mean_ordered(k_w).to(torch.bfloat16).float().reshape(NK, nheads, d).permute(1, 0, 2)
    sqrt_d = torch.tensor(math.sqrt(d), dtype=torch.float32)
    scores = (_dots_ordered(aq, ak).to(torch.bfloat16).float() / sqrt_d).to(torch.bfloat16).float()
    sq, sk = local.shape
    lm = local.to(scores.device).repeat(NQ // sq, NK // sk)
    scores = scores.masked_fill(~lm[None], float("-inf"))
    m = scores.amax(dim=-1, keepdim=True)
    e = torch.where(torch.isinf(scores), torch.zeros_like(scores),
                    torch.exp((scores - m).double()).float())
    tot = torch.zeros(nheads, NQ, dtype=torch.float32, device=scores.device)
    for j in range(NK):
        tot = tot + e[:, :, j]
    prob = (e / tot[..., None]).to(torch.bfloat16).float()
    per_row = NQ // q_temporal
    flat = prob.reshape(nheads * q_temporal, per_row * NK)
    k = min(flat.shape[1] - 1, topk)
    thr = torch.topk(flat, k=k + 1, dim=1).values[:, -1:]
    return (flat > thr).reshape(nheads, NQ, NK)


def causal_topk_mask(q_w, k_w, nheads, per_row, ratio):
    """Benchmark keep rule (synthetic causal rule of the attention configuration).

    Query block i sits in time row (NK-NQ)/per_row + i//per_row, key block j in row
    j//per_row.  Keep the query's own time row, plus the floor(ratio*#past) past blocks
    with the largest mean-pooled q.k score (ties -> lower index), never a future row.
    The rule is this pack's own (no reference counterpart), so its fp32 evaluation order
    is part of its definition: fp32 window means as block_mean_ordered, dots summed in
    ascending channel order without fused multiply-adds.
    """
    NQ, _, C = q_w.shape
    NK = k_w.shape[0]
    d = C // nheads
    aq = block_mean_ordered(q_w).reshape(NQ, nheads, d).permute(1, 0, 2)
    ak = block_mean_ordered(k_w).reshape(NK, nheads, d).permute(1, 0, 2)
    sc = _dots_ordered(aq, ak).cpu().tolist()  # [H][NQ][NK] python floats
    keep = torch.zeros(nheads, NQ, NK, dtype=torch.bool)
    cache_rows = (NK - NQ) // per_row
    for i in range(NQ):
        row = cache_rows + i // per_row
        keep[:, i, row * per_row:(row + 1) * per_row] = True
        npast = row * per_row
        nsel = int(math.floor(ratio * npast))
        if nsel > 0:
            for h in range(nheads):
                row_sc = sc[h][i]
                order = sorted(range(npast), key=lambda j: (-row_sc[j], j))
                keep[h, i, order[:nsel]] = True
    return keep


def build_csr(keep):
    """build_csr (lcsa/triton_lcsa.py:64-71) without truncation: kept block ids ascending,
    then unkept ids ascending (the stable descending argsort order); row length NK."""
    H, NQ, NK = keep.shape
    cnt = keep.sum(-1).to(torch.int32)
    order = torch.argsort(keep.to(torch.int8), dim=-1, descending=True, stable=True)
    return order.to(torch.int32), cnt


def sparse_attention(q_w, k_w, v_w, keep, pairs=None):
    """sparse_attention_ref (lcsa/reference.py:67-88): fp32, per (head, query block).

    q_w [NQ, S, H*d], k_w/v_w [NK, S, H*d]; keep [H, NQ, NK].  Rows whose selection is
    empty return 0 (the kernel's convention, triton_lcsa.py:57-59).  `pairs` (a list of
    (head, query block)) evaluates only those pairs and leaves the rest 0, for checks of a
    sample of a large problem.
    """
    NQ, S, C = q_w.shape
    H = keep.shape[0]
    d = C // H
    scale = 1.0 / math.sqrt(d)
    q = q_w.float().reshape(NQ, S, H, d).permute(2, 0, 1, 3)
    k = k_w.float().reshape(-1, S, H, d).permute(2, 0, 1, 3)
    v = v_w.float().reshape(-1, S, H, d).permute(2, 0, 1, 3)
    out = torch.zeros_like(q)
    todo = pairs if pairs is not None else [(h, i) for h in range(H) for i in range(NQ)]
    for h, i in todo:
        sel = keep[h, i].nonzero(as_tuple=True)[0]
        if sel.numel() == 0:
            continue
        kk = k[h, sel].reshape(-1, d)
        vv = v[h, sel].reshape(-1, d)
        p = torch.softmax(q[h, i] @ kk.t() * scale, dim=-1)
        out[h, i] = p @ vv
    return out.permute(1, 2, 0, 3).reshape(NQ, S, C)


def _online_pass(qi, kh, vh, blocks, c, kv_len, lazy, S, d):
    """Online softmax over the key blocks `blocks` in the given order; returns (m, l, acc)
    with m the max the exponentials were taken against (log2 units, -inf if none)."""
    m = torch.full((S,), float("-inf"), device=qi.device)
    l = torch.zeros(S, device=qi.device)
    acc = torch.zeros(S, d, device=qi.device)
    for j in blocks:
        s = (qi @ kh[j].t()) * c
        if kv_len is not None and (j + 1) * S > kv_len:
            cols = torch.arange(j * S, (j + 1) * S)
            s[:, cols >= kv_len] = float("-inf")
        mb = s.max(dim=1).values
        if lazy > 0:
            m_new = torch.where(mb > m + lazy, mb, m)
        else:
            m_new = torch.maximum(m, mb)
        safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
        alpha = torch.where(torch.isinf(m_new), torch.ones_like(m),
                            torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp2(m - safe)))
        p = torch.exp2(s - safe[:, None])
        l = l * alpha + p.sum(dim=1)
        acc = acc * alpha[:, None] + p.to(torch.bfloat16).float() @ vh[j]
        m = m_new
    return m, l, acc


def sparse_attention_online_loop(q_w, k_w, v_w, keep, kv_len=None, lazy=0.0):
    """sparse_attention_online one (head, query block) at a time (the plain statement; the
    batched form below must agree with it)."""
    NQ, S, C = q_w.shape
    H = keep.shape[0]
    d = C // H
    c = (1.0 / math.sqrt(d)) * 1.4426950408889634
    q = q_w.float().reshape(NQ, S, H, d).permute(2, 0, 1, 3)
    k = k_w.float().reshape(-1, S, H, d).permute(2, 0, 1, 3)
    v = v_w.float().reshape(-1, S, H, d).permute(2, 0, 1, 3)
    out = torch.zeros_like(q)
    for h in range(H):
        for i in range(NQ):
            blocks = keep[h, i].nonzero(as_tuple=True)[0].tolist()
            m, l, acc = _online_pass(q[h, i], k[h], v[h], blocks, c, kv_len, lazy, S, d)
            out[h, i] = torch.where(l[:, None] > 0, acc / l.clamp(min=1e-30)[:, None],
                                    torch.zeros_like(acc))
    return out.permute(1, 2, 0, 3).reshape(NQ, S, C)


def sparse_attention_online(q_w, k_w, v_w, keep, kv_len=None, lazy=0.0):
    """The reference kernel's evaluation order (lcsa/triton_lcsa.py:44-59): per (head, query
    block), kept key blocks in ascending order, online softmax in the log2 domain with fp32
    running max / sum, P rounded to bf16 before P.V (`p.to(V.dtype)`), fp32 accumulator,
    empty rows -> 0.  Keys at index >= kv_len are masked.  Returns fp32 [NQ, S, H*d].

    lazy > 0 restates the B200 kernel's variant: the max the exponentials are taken against
    is only raised when a block's max exceeds it by more than `lazy` (log2 units), and the
    accumulator / sum are rescaled only then (same softmax, P rounded at another scale).

    Evaluated for all (head, query block) pairs at once: step j takes every pair's j-th
    kept key block (ascending), and pairs with fewer kept blocks see an all -inf block,
    which leaves their running max, sum and accumulator exactly unchanged.  Runs on the
    device of q_w."""
    NQ, S, C = q_w.shape
    H = keep.shape[0]
    d = C // H
    dev = q_w.device
    c = (1.0 / math.sqrt(d)) * 1.4426950408889634
    q = q_w.float().reshape(NQ, S, H, d).permute(2, 0, 1, 3)  # [H, NQ, S, d]
    k = k_w.float().reshape(-1, S, H, d).permute(2, 0, 1, 3)  # [H, NK, S, d]
    v = v_w.float().reshape(-1, S, H, d).permute(2, 0, 1, 3)
    keep = keep.to(dev)
    cnt = keep.sum(-1)  # [H, NQ]
    maxc = int(cnt.max().item()) if cnt.numel() else 0
    order = torch.argsort((~keep).to(torch.int8), dim=-1, stable=True)  # kept ids ascending first
    hidx = torch.arange(H, device=dev)[:, None]
    cols = torch.arange(S, device=dev)
    ninf = float("-inf")
    m = torch.full((H, NQ, S), ninf, device=dev)
    l = torch.zeros(H, NQ, S, device=dev)
    acc = torch.zeros(H, NQ, S, d, device=dev)
    for j in range(maxc):
        kj = order[:, :, j]  # [H, NQ]
        s = torch.matmul(q, k[hidx, kj].transpose(-1, -2)) * c  # [H, NQ, S, S]
        valid = (j < cnt)[..., None, None]
        if kv_len is not None:
            valid = valid & ((kj[..., None] * S + cols) < kv_len)[..., None, :]
        s = torch.where(valid, s, torch.full_like(s, ninf))
        mb = s.amax(dim=-1)
        if lazy > 0:
            m_new = torch.where(mb > m + lazy, mb, m)
        else:
            m_new = torch.maximum(m, mb)
        safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
        alpha = torch.where(torch.isinf(m_new), torch.ones_like(m),
                            torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp2(m - safe)))
        p = torch.exp2(s - safe[..., None])
        l = l * alpha + p.sum(dim=-1)
        acc = acc * alpha[..., None] + torch.matmul(p.to(torch.bfloat16).float(), v[hidx, kj])
        m = m_new
    out = torch.where(l[..., None] > 0, acc / l.clamp(min=1e-30)[..., None], torch.zeros_like(acc))
    return out.permute(1, 2, 0, 3).reshape(NQ, S, C)


def dense_attention_online(q, k, v, nheads, lazy=0.0):
    """Dense attention in the kernel's order: every key block kept (cross-attention)."""
    Lq, C = q.shape
    Lk = k.shape[0]
    nq, nk = -(-Lq // 128), -(-Lk // 128)
    qp = torch.zeros(nq * 128, C, dtype=q.dtype, device=q.device)
    qp[:Lq] = q
    kp = torch.zeros(nk * 128, C, dtype=k.dtype, device=q.device)
    kp[:Lk] = k
    vp = torch.zeros(nk * 128, C, dtype=v.dtype, device=q.device)
    vp[:Lk] = v
    keep = torch.ones(nheads, nq, nk, dtype=torch.bool, device=q.device)
    o = sparse_attention_online(qp.view(nq, 128, C), kp.view(nk, 128, C), vp.view(nk, 128, C),
                                keep, kv_len=Lk, lazy=lazy)
    return o.reshape(nq * 128, C)[:Lq]


def dense_attention(q, k, v, nheads):
    """Plain softmax attention, q [Lq, H*d], k/v [Lk, H*d] (cross-attention; fp32)."""
    Lq, C = q.shape
    d = C // nheads
    qh = q.float().reshape(Lq, nheads, d).transpose(0, 1)
    kh = k.float().reshape(-1, nheads, d).transpose(0, 1)
    vh = v.float().reshape(-1, nheads, d).transpose(0, 1)
    p = torch.softmax(qh @ kh.transpose(1, 2) / math.sqrt(d), dim=-1)
    return (p @ vh).transpose(0, 1).reshape(Lq, C)


# ----------------------------------------------------------------------------- inputs
def fp8_outlier_activations(M, K, gen, frac=0.01, mult=20.0):
    """Benchmark GEMM activations: N(0,1) with `frac` of entries multiplied by `mult`."""
    x = torch.randn(M, K, generator=gen)
    mask = torch.rand(M, K, generator=gen) < frac
    return torch.where(mask, x * mult, x).to(torch.bfloat16)
