"""Block-sparse attention (LCSA) on a tcgen05 flash-attention kernel, plus the
window layout and keep-mask builders around it.

Drop-in for ``flashvsr_sm89_ops.lcsa.triton_lcsa`` (triton_lcsa.py:64-94) and
the selection of ``lcsa/reference.py:37-64``:
  * ``build_csr(keep)`` -> (sel, cnt, maxk) computed on the device, with no
    host synchronisation (maxk is NK; rows are padded with the unkept ids in the
    same stable order as the reference).
  * ``block_sparse_attention(q, k, v, keep, sm_scale)`` with the window-order
    layout contract [1, N*128, H*D].
  * ``draft_block_mask`` (reference semantics) and ``causal_topk_mask`` (the
    benchmark's synthetic causal rule), both device kernels.
  * ``window_partition`` / ``window_reverse`` for the (2, 8, 8) windows.
"""
from __future__ import annotations

import math

import torch

from . import _lib

BLOCK = 128


def build_csr(keep: torch.Tensor):
    """keep [H, NQ, NK] bool -> (sel [H, NQ, NK] int32, cnt [H, NQ] int32, maxk = NK)."""
    _lib.require_cuda(keep)
    H, NQ, NK = keep.shape
    k8 = keep.contiguous().view(torch.uint8) if keep.dtype == torch.bool else keep.to(torch.uint8).contiguous()
    sel = torch.empty((H, NQ, NK), dtype=torch.int32, device=keep.device)
    cnt = torch.empty((H, NQ), dtype=torch.int32, device=keep.device)
    _lib.call("fvb_mask_to_csr", _lib.ptr(k8), H, NQ, NK, _lib.ptr(sel), _lib.ptr(cnt),
              _lib.stream_of(keep))
    return sel, cnt, NK


def attention_csr(q2: torch.Tensor, k2: torch.Tensor, v2: torch.Tensor, sel: torch.Tensor,
                  cnt: torch.Tensor, nheads: int, sm_scale: float | None = None,
                  kv_len: int | None = None, out: torch.Tensor | None = None,
                  row_map: torch.Tensor | None = None) -> torch.Tensor:
    """q2 [Lq, H*d], k2/v2 [Lk, H*d] bf16, sel [H, NQ, S] / cnt [H, NQ] int32 -> [Lq, H*d].

    row_map (int32 [Lq]) writes query row r to output row row_map[r]."""
    _lib.require_cuda(q2, k2, v2, sel, cnt)
    Lq, C = q2.shape
    Lk = k2.shape[0]
    d = C // nheads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(d)
    q2, k2, v2 = q2.contiguous(), k2.contiguous(), v2.contiguous()
    if out is None:
        out = torch.empty((Lq, C), dtype=torch.bfloat16, device=q2.device)
    _lib.call("fvb_bsa_fwd", _lib.ptr(q2), _lib.ptr(k2), _lib.ptr(v2), _lib.ptr(sel),
              _lib.ptr(cnt), sel.shape[-1], nheads, Lq, Lk, Lk if kv_len is None else kv_len, d,
              float(sm_scale), _lib.ptr(row_map), _lib.ptr(out), _lib.stream_of(q2))
    return out


def block_sparse_attention(q, k, v, keep, sm_scale=None):
    """q/k/v: [1, L, H*D] bf16 in window order; keep: [H, L//128, K//128] bool.
    Returns [1, L, H*D] bf16.  Rows with no selected key blocks output 0."""
    L, HD = q.shape[-2], q.shape[-1]
    H, NQ, NK = keep.shape
    if L != NQ * BLOCK or k.shape[-2] != NK * BLOCK:
        raise AssertionError(f"block_sparse_attention: L={L}, K={k.shape[-2]} do not match keep "
                             f"{tuple(keep.shape)} x 128")
    sel, cnt, _ = build_csr(keep)
    out = attention_csr(q.reshape(L, HD), k.reshape(-1, HD), v.reshape(-1, HD), sel, cnt, H,
                        sm_scale)
    return out.reshape(1, L, HD)


def dense_attention(q2, k2, v2, nheads, sm_scale=None, out=None):
    """Plain attention of every query over all keys (cross-attention) on the same kernel:
    every query block keeps every key block; keys past Lk are masked."""
    Lq = q2.shape[0]
    Lk = k2.shape[0]
    NQ = (Lq + BLOCK - 1) // BLOCK
    NK = (Lk + BLOCK - 1) // BLOCK
    dev = q2.device
    key = (NQ, NK, nheads, dev)
    cached = _DENSE_CSR.get(key)
    if cached is None:
        sel = torch.arange(NK, dtype=torch.int32, device=dev).repeat(nheads, NQ, 1).contiguous()
        cnt = torch.full((nheads, NQ), NK, dtype=torch.int32, device=dev)
        cached = (sel, cnt)
        _DENSE_CSR[key] = cached
    if Lk % BLOCK != 0:
        pad = NK * BLOCK - Lk
        k2 = torch.cat([k2, k2.new_zeros(pad, k2.shape[1])])
        v2 = torch.cat([v2, v2.new_zeros(pad, v2.shape[1])])
    return attention_csr(q2, k2, v2, cached[0], cached[1], nheads, sm_scale, kv_len=Lk, out=out)


_DENSE_CSR: dict = {}


def window_partition(x: torch.Tensor, fhw, win=(2, 8, 8), out=None) -> torch.Tensor:
    """[B, F*H*W, C] (or a strided [B*F*H*W, C] view) raster -> [B*Nwin*128, C] window order."""
    f, h, w = fhw
    C = x.shape[-1]
    x2 = x.reshape(-1, C) if x.dim() != 2 else x
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    B = rows // (f * h * w)
    if out is None:
        out = torch.empty((rows, C), dtype=x2.dtype, device=x2.device)
    _lib.call("fvb_window_partition", _lib.ptr(x2), x2.stride(0), B, f, h, w, C, win[0], win[1],
              win[2], 0, _lib.ptr(out), _lib.stream_of(x2))
    return out


def window_reverse(xw: torch.Tensor, fhw, win=(2, 8, 8), out=None) -> torch.Tensor:
    """[B*Nwin*128, C] window order -> [B*F*H*W, C] raster."""
    f, h, w = fhw
    C = xw.shape[-1]
    x2 = xw.reshape(-1, C).contiguous()
    rows = x2.shape[0]
    B = rows // (f * h * w)
    if out is None:
        out = torch.empty((rows, C), dtype=x2.dtype, device=x2.device)
    _lib.call("fvb_window_partition", _lib.ptr(x2), C, B, f, h, w, C, win[0], win[1], win[2], 1,
              _lib.ptr(out), _lib.stream_of(x2))
    return out


def build_local_block_mask(bh: int, bw: int, rng: int, device) -> torch.Tensor:
    """Local window mask [bh*bw, bh*bw] (lcsa/reference.py:24-34); tiny, built once per shape."""
    idx = torch.arange(bh * bw, device=device)
    r, c = idx // bw, idx % bw
    r0 = r - rng // 2
    c0 = c - rng // 2
    in_r = (r[None, :] >= r0[:, None]) & (r[None, :] <= r0[:, None] + rng - 1)
    in_c = (c[None, :] >= c0[:, None]) & (c[None, :] <= c0[:, None] + rng - 1)
    return in_r & in_c


def _workspace(nbytes, device, ws):
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
    return ws


def draft_block_mask(q_w, k_w, nheads, q_temporal, local, topk, workspace=None):
    """Device keep-mask selection with the semantics of lcsa/reference.py:37-64.

    q_w [NQ, 128, H*d] (or [NQ*128, H*d]) window order, k_w [NK, 128, H*d]; local [sq, sk]
    bool.  Returns keep [H, NQ, NK] bool.
    """
    _lib.require_cuda(q_w, k_w)
    C = q_w.shape[-1]
    NQ = q_w.numel() // (BLOCK * C)
    NK = k_w.numel() // (BLOCK * C)
    d = C // nheads
    keep = torch.empty((nheads, NQ, NK), dtype=torch.bool, device=q_w.device)
    lm = local.to(device=q_w.device, dtype=torch.bool).contiguous().view(torch.uint8)
    ws = _workspace(_lib.load().fvb_draft_mask_workspace_bytes(nheads, NQ, NK, d), q_w.device, workspace)
    _lib.call("fvb_draft_block_mask", _lib.ptr(q_w.contiguous()), _lib.ptr(k_w.contiguous()),
              nheads, NQ, NK, d, _lib.ptr(lm), lm.shape[0], lm.shape[1], q_temporal, int(topk),
              _lib.ptr(keep.view(torch.uint8)), _lib.ptr(ws), _lib.stream_of(q_w))
    return keep


def block_mean_pool(x_w, out=None):
    """fp32 mean over each 128-token window (avg_q / avg_k of lcsa/reference.py:41-42):
    x_w holds nblk windows of 128 rows x C bf16 -> [nblk, C] fp32."""
    _lib.require_cuda(x_w)
    C = x_w.shape[-1]
    nblk = x_w.numel() // (BLOCK * C)
    if out is None:
        out = torch.empty((nblk, C), dtype=torch.float32, device=x_w.device)
    _lib.call("fvb_block_mean_pool", _lib.ptr(x_w.contiguous()), nblk, C, _lib.ptr(out),
              _lib.stream_of(x_w))
    return out


def causal_topk_mask(q_w, k_w, nheads, per_row, ratio=0.25, workspace=None, k_pool_prefix=None,
                     return_k_pool=False, csr=False):
    """Benchmark keep rule on the device: own time row + top floor(ratio*#past) past blocks.

    k_pool_prefix: pooled fp32 means of the first key blocks (a streaming caller keeps
    them with its KV cache, since a cached block's mean never changes); only the other
    key blocks are pooled.  return_k_pool: also return the pooled keys [NK, C].
    csr: return the rule's CSR (sel, cnt, NK), exactly build_csr of the mask, written by
    the same launch, instead of the mask.
    """
    _lib.require_cuda(q_w, k_w)
    C = q_w.shape[-1]
    NQ = q_w.numel() // (BLOCK * C)
    NK = k_w.numel() // (BLOCK * C)
    d = C // nheads
    keep = None if csr else torch.empty((nheads, NQ, NK), dtype=torch.bool, device=q_w.device)
    if k_pool_prefix is None and not return_k_pool and not csr:
        ws = _workspace(_lib.load().fvb_draft_mask_workspace_bytes(nheads, NQ, NK, d), q_w.device,
                        workspace)
        _lib.call("fvb_causal_topk_mask", _lib.ptr(q_w.contiguous()), _lib.ptr(k_w.contiguous()),
                  nheads, NQ, NK, d, per_row, float(ratio), _lib.ptr(keep.view(torch.uint8)),
                  _lib.ptr(ws), _lib.stream_of(q_w))
        return keep
    n0 = 0 if k_pool_prefix is None else k_pool_prefix.shape[0]
    if n0 > NK or (n0 and tuple(k_pool_prefix.shape) != (n0, C)):
        raise ValueError(f"causal_topk_mask: k_pool_prefix {tuple(k_pool_prefix.shape)} does not "
                         f"fit {NK} key blocks of {C} channels")
    aq = torch.empty((NQ, C), dtype=torch.float32, device=q_w.device)
    ak = torch.empty((NK, C), dtype=torch.float32, device=q_w.device)
    if n0:
        ak[:n0].copy_(k_pool_prefix)
    # the query windows and the new key windows pooled in one launch
    qc = q_w.contiguous()
    kn = k_w.reshape(-1, C)[n0 * BLOCK:]
    kn = kn if kn.is_contiguous() else kn.contiguous()
    _lib.call("fvb_block_mean_pool2", _lib.ptr(qc), NQ, _lib.ptr(kn), NK - n0, C, _lib.ptr(aq),
              _lib.ptr(ak[n0:]), _lib.stream_of(q_w))
    if csr:
        sel = torch.empty((nheads, NQ, NK), dtype=torch.int32, device=q_w.device)
        cnt = torch.empty((nheads, NQ), dtype=torch.int32, device=q_w.device)
        _lib.call("fvb_causal_topk_pooled_csr", _lib.ptr(aq), _lib.ptr(ak), nheads, NQ, NK, d,
                  per_row, float(ratio), None, _lib.ptr(sel), _lib.ptr(cnt), _lib.stream_of(q_w))
        res = (sel, cnt, NK)
    else:
        _lib.call("fvb_causal_topk_pooled", _lib.ptr(aq), _lib.ptr(ak), nheads, NQ, NK, d,
                  per_row, float(ratio), _lib.ptr(keep.view(torch.uint8)), _lib.stream_of(q_w))
        res = keep
    return (res, ak) if return_k_pool else res
