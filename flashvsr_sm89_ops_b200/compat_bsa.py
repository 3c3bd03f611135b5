"""``block_sparse_attn`` stand-in backed by the sm_100a block-sparse kernel.

Drop-in for ``flashvsr_sm89_ops.compat_bsa`` (compat_bsa.py:31-98): upstream
FlashVSR imports ``block_sparse_attn_func`` from the mit-han-lab package at
module load time; importing this pack installs a module of that name whose
function serves the FlashVSR call shape with the tcgen05 kernel.

``FS89_LCSA`` (read at import): ``auto`` (default) installs the stand-in only
when the real package is absent, ``b200`` (alias ``triton``) always installs
it, ``bsa`` never does.
"""
from __future__ import annotations

import os
import sys
import types

STUB_VERSION = "flashvsr-sm89-ops-b200/tcgen05-stub"


def _b200_block_sparse_attn_func(
    q, k, v,
    cu_seqlens_q, cu_seqlens_k,
    head_mask_type,
    streaming_info,
    attn_mask,
    max_seqlen_q, max_seqlen_k,
    dropout_p=0.0,
    deterministic=False,
    softmax_scale=None,
    is_causal=False,
    exact_streaming=False,
    return_attn_probs=False,
):
    """The one call shape FlashVSR uses (compat_bsa.py:31-67).

    q/k/v: [S, H, D] bf16 varlen batch 1 in window order; attn_mask: [1, H, Nq, Nk] or
    [H, Nq, Nk] bool block mask.  Returns [S, H, D].
    """
    if streaming_info is not None or is_causal or dropout_p != 0.0 or return_attn_probs:
        raise NotImplementedError(
            "block_sparse_attn_func stand-in (B200 pack): this call asks for streaming_info, "
            "is_causal, dropout or returned probabilities, which the tcgen05 kernel does not "
            "implement; it serves FlashVSR's one call shape (batch 1, a block keep mask). Use "
            "the mit-han-lab block_sparse_attn package for other modes.")
    from .lcsa import block_sparse_attention

    sq, heads, dim = q.shape
    keep = attn_mask[0] if attn_mask.dim() == 4 else attn_mask
    out = block_sparse_attention(q.reshape(1, sq, heads * dim), k.reshape(1, k.shape[0], heads * dim),
                                 v.reshape(1, v.shape[0], heads * dim), keep, sm_scale=softmax_scale)
    return out.reshape(sq, heads, dim)


def ensure_bsa_available():
    """Install the stand-in unless the real package should win; returns the backend."""
    mode = os.environ.get("FS89_LCSA", "auto").lower()
    present = "block_sparse_attn" in sys.modules and getattr(
        sys.modules["block_sparse_attn"], "__version__", "") != STUB_VERSION
    if not present and "block_sparse_attn" not in sys.modules:
        try:
            import block_sparse_attn  # noqa: F401
            present = True
        except ImportError:
            present = False
    if mode == "bsa":
        return "bsa"
    if present and mode == "auto":
        return "bsa"
    stub = types.ModuleType("block_sparse_attn")
    stub.block_sparse_attn_func = _b200_block_sparse_attn_func
    stub.__version__ = STUB_VERSION
    sys.modules["block_sparse_attn"] = stub
    return "b200"


def active_backend():
    """Report which backend ``import block_sparse_attn`` resolves to."""
    mod = sys.modules.get("block_sparse_attn")
    if mod is None:
        return "bsa" if os.environ.get("FS89_LCSA", "auto").lower() == "bsa" else "unresolved"
    return "b200" if getattr(mod, "__version__", "") == STUB_VERSION else "bsa"
