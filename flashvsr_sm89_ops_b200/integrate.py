"""One-call wiring of the B200 operator pack into a FlashVSR v1.1 Tiny pipeline.

Drop-in for ``flashvsr_sm89_ops.integrate`` (integrate.py:1-292): ``enable(pipe,
dit_module=None, parts=None, compile_memblocks=None, verbose=True) -> dict``
reads the same flags (FS89_FP8, FS89_FP8_FFNFUSED, FS89_FUSED_ROPE,
FS89_FUSED_ADALN, FS89_TCDEC_CL, FS89_TCDEC_COMPILE), converts the DiT linears
to FP8, and rebinds ``SelfAttention.forward`` / ``CrossAttention.forward`` /
``DiTBlock.forward`` of the upstream DiT module.  Each rebound forward keeps the
stock branch (flags off) and the reference-shaped fused branch, and adds the
B200 fast path taken when every op of the block is on this pack:

  LN-mod emits the per-token FP8 codes  ->  one fused q|k|v FP8 GEMM [M, 3D]
  -> RMSNorm+RoPE of q and k read straight from the GEMM output and written in
  (2,8,8)-window order, v permuted by one copy kernel -> device keep mask ->
  device CSR -> tcgen05 block-sparse attention writing raster order -> o GEMM
  -> gate-add -> affine LN -> cross-attention (same kernel, all key blocks)
  -> LN-mod with FP8 output -> FFN (GEMM-1 + GELU/amax epilogue, quant, GEMM-2)
  -> gate-add.

Extra flags of this pack: FS89_FP8_SCALE=token|tensor (activation granularity;
``tensor`` reproduces the reference's per-tensor numerics), FS89_FUSED_MASK=1
(device keep-mask builder instead of upstream generate_draft_block_mask).
"""
from __future__ import annotations

import os
import weakref

import torch

from . import lcsa
from .compat_bsa import active_backend, ensure_bsa_available
from .fp8_ffn import FP8FFN, convert_ffn_fp8, ffn_fp8
from .fp8_linear import FP8Linear, convert_linears_fp8, fp8_mm
from .fp8_quant import default_act_mode, quantize_fp8
from .fused_adaln import (fused_gate_add, fused_ln_modulate, fused_ln_modulate_adaln,
                          gate_add_layer_norm, gate_add_ln_modulate, layer_norm)
from .fused_rms_rope import freqs_cos_sin, fused_rms_rope, qkv_rope_window, rms_rope_rows


def _FLAG(name, default):
    return os.environ.get(name, default) == "1"


def _unwrap(m):
    """enable_vram_management wraps norms/linears in AutoWrappedModule."""
    return getattr(m, "module", m)


def _module_eps(m, default=1e-6):
    return getattr(_unwrap(m), "eps", default)


# ----------------------------------------------------------------------------- helpers
_ROW_MAPS: dict = {}


def _row_maps(f, h, w, device, win=(2, 8, 8)):
    """(raster->window, window->raster) int32 row maps for an (f, h, w) grid, cached."""
    key = (f, h, w, win, str(device))
    m = _ROW_MAPS.get(key)
    if m is None:
        L = f * h * w
        wf, wh, ww = win
        idx = torch.arange(L, dtype=torch.int32).view(f // wf, wf, h // wh, wh, w // ww, ww)
        w2r = idx.permute(0, 2, 4, 1, 3, 5).reshape(-1).contiguous()
        r2w = torch.empty_like(w2r)
        r2w[w2r.long()] = torch.arange(L, dtype=torch.int32)
        m = (r2w.to(device), w2r.to(device))
        _ROW_MAPS[key] = m
    return m


def _qkv_pack(attn):
    """Concatenated q|k|v FP8 weights with per-channel scales, built once per module.

    Per-tensor weight scales become constant per-channel segments, so the fused
    product is exactly the three separate ones.
    """
    q, k, v = attn.q, attn.k, attn.v
    if not all(type(l) is FP8Linear for l in (q, k, v)) or len({q.mode, k.mode, v.mode}) != 1:
        return None
    pk = getattr(attn, "_fvb_qkv", None)
    if pk is not None and pk[0] is q.weight:
        return pk
    W = torch.cat([l.weight.view(torch.uint8) for l in (q, k, v)]).view(torch.float8_e4m3fn)

    def chan(l):
        s = l.w_scale.float()
        return s.expand(l.out_features) if s.numel() == 1 else s

    S = torch.cat([chan(l) for l in (q, k, v)]).contiguous()
    Bv = torch.cat([(l.bias if l.bias is not None else torch.zeros(l.out_features, device=W.device))
                    .to(torch.bfloat16) for l in (q, k, v)]).contiguous()
    pk = (q.weight, W.contiguous(), S, Bv, q.mode)
    attn._fvb_qkv = pk
    return pk


def _take_stash(mod, x):
    st = getattr(mod, "_fvb_x8", None)
    mod._fvb_x8 = None
    if st is not None and st[0] is x:
        return st[1], st[2]
    return None


def _local_mask(self, dit, h, w, local_range, device):
    if self.local_attn_mask is None or self.local_attn_mask_h != h // 8 \
            or self.local_attn_mask_w != w // 8 or self.local_range != local_range:
        self.local_attn_mask = dit.build_local_block_mask_shifted_vec_normal_slide(
            h // 8, w // 8, local_range, local_range, include_self=True, device=device)
        self.local_attn_mask_h = h // 8
        self.local_attn_mask_w = w // 8
        self.local_range = local_range
    return self.local_attn_mask


class _KVArena:
    """Key (or value) window rows of one self-attention stream, in a buffer with spare
    time rows, so a streaming step writes its new row right after the cache it was given
    and attends to one contiguous [cache | new] view instead of concatenating them.

    ``views`` keeps a weak reference to every cache tensor handed out, with its window
    range; a range is written only while no live handed-out cache covers it, so a cache
    a caller still holds never changes underneath it.
    """

    SPARE_ROWS = 4  # time rows of headroom: one copy of the cache per 4 streaming steps

    def __init__(self, nblk, D, device):
        self.buf = torch.empty((nblk * 128, D), dtype=torch.bfloat16, device=device)
        self.cap = nblk
        self.views = []

    def covered(self, a, b):
        """Whether a live handed-out cache covers any window of [a, b)."""
        self.views = [v for v in self.views if v[0]() is not None]
        return any(x < b and a < y for _, x, y in self.views)

    def rows(self, a, b):
        return self.buf[a * 128:b * 128]

    def hand_out(self, a, b):
        t = self.rows(a, b).view(b - a, 128, -1)
        t._fvb_arena = (self, a, b)
        self.views.append((weakref.ref(t), a, b))
        return t


def _arena_slot(pre, nnew, row_blocks, D, device):
    """(arena, a, b) with the cache `pre` in windows [a, b) of an arena whose windows
    [b, b + nnew) are free for the new time row: `pre`'s own arena when it came from
    one and has room, else a new arena holding a copy of `pre`."""
    st = getattr(pre, "_fvb_arena", None) if pre is not None else None
    if st is not None:
        ar, a, b = st
        if ar.buf.shape[1] == D and ar.buf.device == device and b + nnew <= ar.cap \
                and not ar.covered(b, b + nnew):
            return ar, a, b
    npre = 0 if pre is None else pre.numel() // (128 * D)
    ar = _KVArena(npre + nnew + row_blocks * _KVArena.SPARE_ROWS, D, device)
    if npre:
        ar.rows(0, npre).copy_(pre.reshape(-1, D))
    return ar, 0, npre


def _cached_kpool(cache_k, D):
    """Pooled key means stored with a KV-cache tensor this module returned, if the tensor
    is unchanged since (same in-place version counter) and the shapes agree."""
    st = getattr(cache_k, "_fvb_kpool", None) if cache_k is not None else None
    if st is None or st[1] != cache_k._version:
        return None
    pool = st[0]
    if pool.shape[0] * 128 * D != cache_k.numel() or pool.shape[1] != D:
        return None
    return pool


def _stash_kpool(cache_k, pool):
    cache_k._fvb_kpool = (pool, cache_k._version)


def _keep_mask(self, dit, q_w, k_w, nh, seqlen, h, w, topk, local_range, pre_cache_k=None,
               csr=False):
    """Block keep mask; returns (keep, pooled keys or None).  csr (causal rule): the mask's
    CSR (sel, cnt, NK) from the rule's own launch in place of the mask."""
    D = q_w.shape[-1]
    if getattr(dit, "MASK_RULE", "draft") == "causal":
        per_row = q_w.shape[0] // 128 // seqlen
        return lcsa.causal_topk_mask(q_w, k_w, nh, per_row, getattr(dit, "CAUSAL_RATIO", 0.25),
                                     k_pool_prefix=_cached_kpool(pre_cache_k, D),
                                     return_k_pool=True, csr=csr)
    local = _local_mask(self, dit, h, w, local_range, q_w.device)
    if _FLAG("FS89_FUSED_MASK", "1"):
        return lcsa.draft_block_mask(q_w, k_w, nh, seqlen, local, topk), None
    m = dit.generate_draft_block_mask(1, nh, seqlen, q_w.view(-1, 128, D), k_w.view(-1, 128, D),
                                      topk=topk, local_attn_mask=local)
    return (m[0] if m.dim() == 4 else m), None


def _fast_self_ok(self, x):
    return x.dim() == 3 and x.shape[0] == 1 and x.dtype == torch.bfloat16 and x.is_cuda \
        and _qkv_pack(self) is not None and type(self.o) is FP8Linear


def _self_fast_path(dit, attn, x):
    """Whether attn's forward takes the B200 fast path for input shaped like x."""
    return getattr(dit, "FUSED_ROPE_FN", None) is fused_rms_rope and _fast_self_ok(attn, x)


def _cross_fast_path(dit, ca, x):
    """Whether the cross-attention forward takes the B200 fast path for input like x."""
    return getattr(dit, "FUSED_ROPE_FN", None) is fused_rms_rope and x.dim() == 3 \
        and x.shape[0] == 1 and x.is_cuda and type(ca.q) is FP8Linear and type(ca.o) is FP8Linear


# ----------------------------------------------------------------------------- forwards
def _fast_self_attn(self, dit, x, freqs, f, h, w, topk, kv_len, pre_cache_k, pre_cache_v,
                    local_range):
    _, L, D = x.shape
    nh = self.num_heads
    hd = D // nh
    _, W, S, Bv, mode = _qkv_pack(self)
    pre = _take_stash(self, x)
    if pre is None:
        x8, s8 = quantize_fp8(x.reshape(L, D), mode)
    else:
        x8, s8 = pre
    qkv = fp8_mm(x8, s8, W, S, Bv)  # [L, 3D]
    cos, sin = freqs_cos_sin(freqs)
    if cos.device != x.device:
        cos, sin = cos.to(x.device), sin.to(x.device)
    r2w, w2r = _row_maps(f, h, w, x.device)
    nq, nk = _unwrap(self.norm_q), _unwrap(self.norm_k)
    seqlen = f // 2
    one_len = (L // 128) // seqlen
    nnew = L // 128
    pk = pre_cache_k if (pre_cache_k is not None and pre_cache_v is not None) else None
    pv = pre_cache_v if pk is not None else None
    ark, ak0, ak1 = _arena_slot(pk, nnew, one_len, D, x.device)
    arv, av0, av1 = _arena_slot(pv, nnew, one_len, D, x.device)
    # q, and the new keys / values right after the cache ([cache | new] is one contiguous
    # view), in window order from one launch over the fused projection
    q_w = torch.empty((L, D), dtype=torch.bfloat16, device=x.device)
    qkv_rope_window(qkv, nq.weight, nk.weight, cos, sin, L, _module_eps(self.norm_q),
                    _module_eps(self.norm_k), hd, r2w, q_w, ark.rows(ak1, ak1 + nnew),
                    arv.rows(av1, av1 + nnew))
    k_w, v_w = ark.rows(ak0, ak1 + nnew), arv.rows(av0, av1 + nnew)
    if getattr(dit, "MASK_RULE", "draft") == "causal":
        (sel, cnt, _), kpool = _keep_mask(self, dit, q_w, k_w, nh, seqlen, h, w, topk,
                                          local_range, pre_cache_k, csr=True)
    else:
        keep, kpool = _keep_mask(self, dit, q_w, k_w, nh, seqlen, h, w, topk, local_range,
                                 pre_cache_k)
        sel, cnt, _ = lcsa.build_csr(keep)
    o = lcsa.attention_csr(q_w, k_w, v_w, sel, cnt, nh, row_map=w2r)  # raster order
    nkb = k_w.shape[0] // 128
    drop = one_len if (kv_len is not None and nkb // one_len > kv_len) else 0
    cache_k = ark.hand_out(ak0 + drop, ak1 + nnew)
    cache_v = arv.hand_out(av0 + drop, av1 + nnew)
    if kpool is not None:
        _stash_kpool(cache_k, kpool[drop:])
    return self.o(o.view(1, L, D)), cache_k, cache_v


def _make_self_attn_forward(dit):
    from einops import rearrange

    def forward(self, x, freqs, f=None, h=None, w=None, local_num=None, topk=None,
                train_img=False, block_id=None, kv_len=None, is_full_block=False,
                is_stream=False, pre_cache_k=None, pre_cache_v=None, local_range=9):
        B, L, D = x.shape
        if is_stream and pre_cache_k is not None and pre_cache_v is not None:
            assert f == 2, "f must be 2"
        if is_stream and (pre_cache_k is None or pre_cache_v is None):
            assert f == 6, " start f must be 6"
        assert L == f * h * w, "Sequence length mismatch with provided (f,h,w)."

        rope_fn = getattr(dit, "FUSED_ROPE_FN", None)
        if _self_fast_path(dit, self, x):
            out, ck, cv = _fast_self_attn(self, dit, x, freqs, f, h, w, topk, kv_len,
                                          pre_cache_k, pre_cache_v, local_range)
            return (out, ck, cv) if is_stream else out

        if rope_fn is not None:
            q = rope_fn(self.q(x), _unwrap(self.norm_q).weight, freqs,
                        eps=_module_eps(self.norm_q), rope=True, head_dim=self.head_dim)
            k = rope_fn(self.k(x), _unwrap(self.norm_k).weight, freqs,
                        eps=_module_eps(self.norm_k), rope=True, head_dim=self.head_dim)
        else:
            q = dit.rope_apply(self.norm_q(self.q(x)), freqs, self.num_heads)
            k = dit.rope_apply(self.norm_k(self.k(x)), freqs, self.num_heads)
        v = self.v(x)
        win = (2, 8, 8)
        q_w = dit.WindowPartition3D.partition(q.view(B, f, h, w, D), win)
        k_w = dit.WindowPartition3D.partition(k.view(B, f, h, w, D), win)
        v_w = dit.WindowPartition3D.partition(v.view(B, f, h, w, D), win)
        seqlen = f // win[0]
        one_len = k_w.shape[0] // B // seqlen
        if pre_cache_k is not None and pre_cache_v is not None:
            k_w = torch.cat([pre_cache_k, k_w], dim=0)
            v_w = torch.cat([pre_cache_v, v_w], dim=0)
        block_n = q_w.shape[0] // B
        block_s = q_w.shape[1]
        block_n_kv = k_w.shape[0] // B
        reorder_q = rearrange(q_w, "(b n) s d -> b (n s) d", n=block_n, s=block_s)
        reorder_k = rearrange(k_w, "(b n) s d -> b (n s) d", n=block_n_kv, s=block_s)
        reorder_v = rearrange(v_w, "(b n) s d -> b (n s) d", n=block_n_kv, s=block_s)
        local = _local_mask(self, dit, h, w, local_range, k_w.device)
        mask = dit.generate_draft_block_mask(B, self.num_heads, seqlen, q_w, k_w, topk=topk,
                                             local_attn_mask=local)
        x = self.attn(reorder_q, reorder_k, reorder_v, mask)
        cur_n = k_w.shape[0]
        if kv_len is not None and cur_n // one_len > kv_len:
            cache_k, cache_v = k_w[one_len:], v_w[one_len:]
        else:
            cache_k, cache_v = k_w, v_w
        x = rearrange(x, "b (n s) d -> (b n) s d", n=block_n, s=block_s)
        x = dit.WindowPartition3D.reverse(x, win, (f, h, w)).reshape(B, f * h * w, D)
        if is_stream:
            return self.o(x), cache_k, cache_v
        return self.o(x)

    return forward


def _make_cross_attn_forward(dit):
    def forward(self, x, y, is_stream=False):
        rope_fn = getattr(dit, "FUSED_ROPE_FN", None)
        assert self.cache_k is not None and self.cache_v is not None
        if _cross_fast_path(dit, self, x):
            _, L, D = x.shape
            pre = _take_stash(self, x)
            if pre is None:
                q = self.q(x).view(L, D)
            else:
                q = self.q._mm(pre[0], pre[1])
            qn = rms_rope_rows(q, _unwrap(self.norm_q).weight, None, None, L,
                               _module_eps(self.norm_q), False, D // self.num_heads)
            o = lcsa.dense_attention(qn, self.cache_k.reshape(-1, D), self.cache_v.reshape(-1, D),
                                     self.num_heads)
            return self.o(o.view(1, L, D))
        if rope_fn is not None:
            q = rope_fn(self.q(x), _unwrap(self.norm_q).weight, None,
                        eps=_module_eps(self.norm_q), rope=False)
        else:
            q = self.norm_q(self.q(x))
        return self.o(self.attn(q, self.cache_k, self.cache_v))

    return torch.no_grad()(forward)


def _make_dit_block_forward(dit):
    def forward(self, x, context, t_mod, freqs, f, h, w, local_num=None, topk=None,
                train_img=False, block_id=None, kv_len=None, is_full_block=False,
                is_stream=False, pre_cache_k=None, pre_cache_v=None, local_range=9):
        fa = getattr(dit, "FUSED_ADALN", None)
        fast = fa is not None and fa[0] is fused_ln_modulate and x.shape[0] == 1 and x.is_cuda
        token = fast and default_act_mode() == "token"
        fp8_norm1 = token and _qkv_pack(self.self_attn) is not None \
            and self.self_attn.q.mode == "token"
        mod_p = self.modulation
        # norm1 forms the modulation sum in its own launch when both operands are the bf16
        # device tensors the kernel takes
        fused_mod = fp8_norm1 and mod_p.dtype == t_mod.dtype == torch.bfloat16 and mod_p.is_cuda \
            and t_mod.is_cuda and t_mod.dim() == 3 and t_mod.shape[1] == 6 \
            and mod_p.is_contiguous() and t_mod.is_contiguous()
        if not fused_mod:
            shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (
                mod_p.to(dtype=t_mod.dtype, device=t_mod.device) + t_mod).chunk(6, dim=1)
        if fa is not None:
            ln_mod, gate_add = fa
            if fp8_norm1:
                # the fast self-attention path reads only the FP8 codes: no bf16 output then
                # (the block input stands in for it as the stash key)
                skip = _self_fast_path(dit, self.self_attn, x)
                eps1 = _module_eps(self.norm1)
                if fused_mod:
                    input_x, x8, s8, mod = fused_ln_modulate_adaln(
                        x, mod_p, t_mod, eps=eps1, emit_fp8=True, want_out=not skip)
                    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = \
                        mod.chunk(6, dim=1)
                else:
                    input_x, x8, s8 = fused_ln_modulate(x, scale_msa, shift_msa, eps=eps1,
                                                        emit_fp8=True, want_out=not skip)
                input_x = x if input_x is None else input_x
                self.self_attn._fvb_x8 = (input_x, x8.view(-1, x.shape[-1]), s8)
            else:
                input_x = ln_mod(x, scale_msa, shift_msa, eps=_module_eps(self.norm1))
        else:
            input_x = dit.modulate(self.norm1(x), shift_msa, scale_msa)
        self_attn_output, self_attn_cache_k, self_attn_cache_v = self.self_attn(
            input_x, freqs, f, h, w, local_num, topk, train_img, block_id,
            kv_len=kv_len, is_full_block=is_full_block, is_stream=True,
            pre_cache_k=pre_cache_k, pre_cache_v=pre_cache_v, local_range=local_range)
        ca_out = None  # fast path: cross-attention output not yet added to x
        if fast:
            n3 = _unwrap(self.norm3)
            ca = self.cross_attn
            if token and type(getattr(ca, "q", None)) is FP8Linear and ca.q.mode == "token":
                # gate-add and norm3 in one pass; norm3 also emits the per-token FP8 codes of
                # its output, which the cross-attention q projection takes directly (its bf16
                # output only when the cross-attention would read it)
                skip = _cross_fast_path(dit, ca, x)
                x, xn, x8, s8 = gate_add_layer_norm(x, gate_msa, self_attn_output, n3.weight,
                                                    n3.bias, eps=getattr(n3, "eps", 1e-6),
                                                    emit_fp8=True, want_out=not skip)
                xn = x if xn is None else xn
                ca._fvb_x8 = (xn, x8, s8)
            else:
                x = gate_add(x, gate_msa, self_attn_output)
                xn = layer_norm(x, n3.weight, n3.bias, eps=getattr(n3, "eps", 1e-6))
            ca_out = ca(xn, context, is_stream=is_stream)
        else:
            if fa is not None:
                x = gate_add(x, gate_msa, self_attn_output)
            else:
                x = self.gate(x, gate_msa, self_attn_output)
            x = x + self.cross_attn(self.norm3(x), context, is_stream=is_stream)
        if fa is not None:
            ffn = self.ffn
            if ca_out is not None and token and isinstance(ffn, FP8FFN) \
                    and ffn.lin0.mode == "token":
                # cross-attention add and norm2 in one pass; the FFN reads only the FP8 codes
                x, _, x8, s8 = gate_add_ln_modulate(x, None, ca_out, scale_mlp, shift_mlp,
                                                    eps=_module_eps(self.norm2), emit_fp8=True,
                                                    want_out=False)
                # FFN and the block's closing gated residual add in one call (the add runs in
                # the down-projection's epilogue; bit for bit gate_add(x, gate_mlp, FFN(.)))
                x = ffn_fp8(x8.view(-1, x.shape[-1]), s8, ffn.lin0, ffn.lin2, residual=x,
                            gate=gate_mlp).view(x.shape)
                y = None
            else:
                if ca_out is not None:
                    x = fused_gate_add(x, None, ca_out)
                input_x = ln_mod(x, scale_mlp, shift_mlp, eps=_module_eps(self.norm2))
                y = self.ffn(input_x)
            if y is not None:
                x = gate_add(x, gate_mlp, y)
        else:
            input_x = dit.modulate(self.norm2(x), shift_mlp, scale_mlp)
            x = self.gate(x, gate_mlp, self.ffn(input_x))
        if is_stream:
            return x, self_attn_cache_k, self_attn_cache_v
        return x

    return forward


# ----------------------------------------------------------------------------- patching
_EXPECTED_SIGS = {
    "SelfAttention": ("x", "freqs", "f", "h", "w", "local_num", "topk", "train_img",
                      "block_id", "kv_len", "is_full_block", "is_stream",
                      "pre_cache_k", "pre_cache_v", "local_range"),
    "DiTBlock": ("x", "context", "t_mod", "freqs", "f", "h", "w", "local_num", "topk",
                 "train_img", "block_id", "kv_len", "is_full_block", "is_stream",
                 "pre_cache_k", "pre_cache_v", "local_range"),
}


def _check_dit_structure(dit):
    """Guard against upstream drift (integrate.py:197-214): same classes and argument names."""
    import inspect
    for cls, expected in _EXPECTED_SIGS.items():
        c = getattr(dit, cls, None)
        if c is None:
            raise RuntimeError(f"upstream wan_video_dit has no {cls}; this pack "
                               f"targets FlashVSR v1.1 - got {dit}")
        fwd = getattr(c, "_fvb_stock_forward", c.forward)
        params = tuple(inspect.signature(fwd).parameters)
        missing = [p for p in expected if p not in params]
        if missing:
            raise RuntimeError(f"upstream {cls}.forward lacks args {missing} - upstream signature "
                               f"changed since the tested revision (cf910c6).")
    if not hasattr(dit, "WindowPartition3D") or not hasattr(dit, "generate_draft_block_mask"):
        raise RuntimeError("upstream wan_video_dit lacks WindowPartition3D / "
                           "generate_draft_block_mask - unsupported revision.")


def _patch_dit(dit, fused_rope, fused_adaln):
    _check_dit_structure(dit)
    dit.FUSED_ROPE_FN = fused_rms_rope if fused_rope else None
    dit.FUSED_ADALN = (fused_ln_modulate, fused_gate_add) if fused_adaln else None
    if getattr(dit, "_FS89_PATCHED", False):
        return
    for cls in ("SelfAttention", "CrossAttention", "DiTBlock"):
        c = getattr(dit, cls)
        c._fvb_stock_forward = c.forward
    dit.SelfAttention.forward = _make_self_attn_forward(dit)
    dit.CrossAttention.forward = _make_cross_attn_forward(dit)
    dit.DiTBlock.forward = _make_dit_block_forward(dit)
    dit._FS89_PATCHED = True


def enable(pipe, dit_module=None, parts=None, compile_memblocks=None, verbose=True):
    """Apply the B200 operator pack to a FlashVSR Tiny pipeline (integrate.py:229-292).

    Call once after ``pipe.enable_vram_management(...)`` and before
    ``pipe.init_cross_kv()``.  Returns a dict of what was enabled.  Re-running it on
    an already patched pipeline is safe.
    """
    if parts is None:
        parts = [p for p in os.environ.get("FS89_FP8", "ffn,self,cross").split(",") if p]
    if compile_memblocks is None:
        compile_memblocks = _FLAG("FS89_TCDEC_COMPILE", "0")
    applied = {}
    if dit_module is None:
        try:
            import diffsynth.models.wan_video_dit as dit_module
        except ImportError as e:
            raise ImportError(
                "enable() could not import diffsynth.models.wan_video_dit. Run from a "
                "FlashVSR checkout (or pass dit_module=).") from e

    if hasattr(pipe, "TCDecoder") and _FLAG("FS89_TCDEC_CL", "1"):
        pipe.TCDecoder.to(memory_format=torch.channels_last)
        applied["tcdec_channels_last"] = True
    if compile_memblocks and hasattr(pipe, "TCDecoder"):
        try:
            from utils.TCDecoder import MemBlock
        except ImportError:
            raise ImportError(
                "compile_memblocks=True needs the FlashVSR example utils package "
                "(examples/WanVSR) on sys.path, or leave FS89_TCDEC_COMPILE=0.")
        n = 0
        for m in pipe.TCDecoder.modules():
            if isinstance(m, MemBlock):
                m.forward = torch.compile(m.forward, mode="max-autotune-no-cudagraphs", dynamic=False)
                n += 1
        applied["tcdec_compiled_memblocks"] = n

    if parts:
        mode = default_act_mode()
        model = pipe.denoising_model()
        applied["fp8_linears"] = convert_linears_fp8(model, parts=parts, mode=mode)
        applied["fp8_scales"] = mode
        if "ffn" in parts and _FLAG("FS89_FP8_FFNFUSED", "1"):
            applied["fp8_ffn_blocks"] = convert_ffn_fp8(model)

    _patch_dit(dit_module, fused_rope=_FLAG("FS89_FUSED_ROPE", "1"),
               fused_adaln=_FLAG("FS89_FUSED_ADALN", "1"))
    applied["fused_rope"] = _FLAG("FS89_FUSED_ROPE", "1")
    applied["fused_adaln"] = _FLAG("FS89_FUSED_ADALN", "1")
    ensure_bsa_available()
    applied["lcsa_backend"] = active_backend()
    if verbose:
        print(f"[flashvsr-sm89-ops-b200] enabled: {', '.join(f'{k}={v}' for k, v in applied.items())}")
    return applied
