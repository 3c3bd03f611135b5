"""flashvsr-sm89-ops-b200 — the FlashVSR v1.1 operator pack, rebuilt for NVIDIA B200 (sm_100a).

Same public surface as ``flashvsr_sm89_ops`` (its __init__.py:23-39): importing
the package installs the ``block_sparse_attn`` stand-in (``FS89_LCSA``), and
``enable(pipe)`` wires every operator into a FlashVSR (Wan-style DiT) pipeline.
Every op runs on hand-written sm_100a CUDA kernels behind the C ABI declared in
``include/flashvsr_b200.h`` (``libflashvsr_b200.so``); there is no CPU or Triton
fallback.
"""
from .compat_bsa import active_backend, ensure_bsa_available

ensure_bsa_available()

from .fused_rms_rope import fused_rms_rope  # noqa: E402
from .fused_adaln import fused_ln_modulate, fused_gate_add  # noqa: E402
from .fp8_quant import quantize_fp8, FP8_MAX  # noqa: E402
from .fp8_linear import FP8Linear, convert_linears_fp8  # noqa: E402
from .fp8_ffn import FP8FFN, convert_ffn_fp8  # noqa: E402
from .integrate import enable  # noqa: E402
from .tiling import auto_tile_limits, plan_tiles, render_tiled, tile_weight  # noqa: E402

__all__ = [
    "enable",
    "fused_rms_rope",
    "fused_ln_modulate",
    "fused_gate_add",
    "quantize_fp8",
    "FP8_MAX",
    "FP8Linear",
    "convert_linears_fp8",
    "FP8FFN",
    "convert_ffn_fp8",
    "plan_tiles",
    "render_tiled",
    "auto_tile_limits",
    "tile_weight",
    "active_backend",
]
