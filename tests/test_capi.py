"""The C-ABI library loads and exports every entry point declared in include/*.h;
argument validation runs on the host and returns FVB_ERR_INVALID without any GPU
work (CPU only: no compute call is made)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            names |= set(re.findall(r"^FVB_API\s+[\w\s\*]+?\b(fvb_\w+)\s*\(", src, flags=re.M))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("fvb_quant_fp8", "fvb_fp8_gemm", "fvb_fp8_ffn", "fvb_rms_rope", "fvb_ln_modulate",
                 "fvb_gate_add", "fvb_mask_to_csr", "fvb_bsa_fwd", "fvb_window_partition",
                 "fvb_draft_block_mask", "fvb_gelu_quant_fp8"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from flashvsr_sm89_ops_b200 import _lib
    lib = _lib.load()
    raw = ctypes.CDLL(_lib.lib_path())
    for name in declared_symbols():
        assert hasattr(raw, name), f"{name} declared in include/ but not exported"
    assert set(declared_symbols()) == set(_lib.exported_symbols())
    assert lib.fvb_abi_version() >= 1


def test_built_for_sm100a():
    from flashvsr_sm89_ops_b200 import _build
    cmd = " ".join(_build.nvcc_command())
    assert "arch=compute_100a,code=sm_100a" in cmd


def test_host_validation_without_gpu():
    from flashvsr_sm89_ops_b200 import _lib
    lib = _lib.load()
    assert lib.fvb_quant_fp8(None, -1, 4, None, None, 0, None, None) == _lib.FVB_ERR_INVALID
    assert "negative" in lib.fvb_last_error().decode()
    assert lib.fvb_quant_fp8(None, 4, 4, None, None, 7, None, None) == _lib.FVB_ERR_INVALID
    assert lib.fvb_fp8_gemm(None, None, 0, None, None, 0, None, 8, 8, 10, None, 0, None, None) \
        == _lib.FVB_ERR_INVALID  # K % 16 != 0
    assert lib.fvb_bsa_fwd(None, None, None, None, None, 1, 12, 128, 128, 128, 64, 0.1, None, None,
                           None) == _lib.FVB_ERR_INVALID  # head_dim != 128
    assert lib.fvb_window_partition(None, 0, 1, 3, 8, 8, 8, 2, 8, 8, 0, None, None) == \
        _lib.FVB_ERR_INVALID  # F=3 not divisible by 2
    assert lib.fvb_ln_modulate(None, None, None, 1, 4, 3000, 1e-6, None, None, None, None) == \
        _lib.FVB_ERR_INVALID  # D > 2048
    # a crop window that leaves the plane is refused before any copy is queued
    assert lib.fvb_copy_window_h2d(1, 7680, 2048, 255, 2 * 3000, 0, 1792, 768, 1, None) == \
        _lib.FVB_ERR_INVALID  # x_bytes + width_bytes > pitch
    assert "outside" in lib.fvb_last_error().decode()
    assert lib.fvb_copy_window_h2d(1, 7680, 2048, 255, 0, 1500, 1792, 768, 1, None) == \
        _lib.FVB_ERR_INVALID  # y + height > rows
    # empty problems are valid no-ops that need no device
    assert lib.fvb_gate_add(None, None, None, 0, 4, 8, None, None) == _lib.FVB_OK
    assert lib.fvb_fp8_gemm(None, None, 0, None, None, 0, None, 0, 8, 16, None, 0, None, None) == _lib.FVB_OK


def test_workspace_queries():
    from flashvsr_sm89_ops_b200 import _lib
    lib = _lib.load()
    assert lib.fvb_quant_fp8_workspace_bytes(8, 8, 0) >= 4
    assert lib.fvb_quant_fp8_workspace_bytes(8, 8, 1) == 0
    M, F = 8448, 8960
    assert lib.fvb_fp8_ffn_workspace_bytes(M, F) >= M * F * 3 + 8 * M
    assert lib.fvb_draft_mask_workspace_bytes(12, 66, 264, 128) >= (66 + 264) * 1536 * 4


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: a CPU tensor is rejected loudly."""
    import torch
    from flashvsr_sm89_ops_b200 import quantize_fp8, fused_gate_add
    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        quantize_fp8(x)
    with pytest.raises(ValueError, match="CUDA"):
        fused_gate_add(x.view(1, 4, 16), x[:1].view(1, 1, 16), x.view(1, 4, 16))
