"""Op-level parity of the sm_100a kernels (through the C ABI) against the CPU oracle.

Bars: FP8 codes and scales bit-exact; gate-add bitwise;
LN-mod / RMS-RoPE within 1 bf16 ulp on a tiny fraction of elements; GEMM / FFN /
attention within 1e-2 max relative error (attention: the reference test's
atol = rtol = 1e-2, lcsa/test_correctness.py:59).
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle import ops as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def gen(seed=0):
    return torch.Generator().manual_seed(seed)


def bf16_ulp(t):
    """bf16 unit in the last place at |t| (8 significant bits)."""
    mag = t.float().abs().clamp(min=2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(mag)) - 7)


def within_ulps(out, ref, operand_mag, n=1.0, extra=None):
    """|out-ref| <= n ulp of the output + n ulp of the operand magnitude feeding the last
    add/rotation (an fp32-last-bit difference upstream of a cancelling add moves the
    bf16 result by one ulp of the operands, not of the small result) + `extra` (an
    upstream one-ulp difference carried through a multiply)."""
    out = out.float().cpu()
    ref = ref.float().cpu()
    tol = n * (bf16_ulp(torch.maximum(out.abs(), ref.abs())) + bf16_ulp(operand_mag.float().cpu()))
    if extra is not None:
        tol = tol + extra.float().cpu()
    d = (out - ref).abs()
    return bool((d <= tol).all()), (d > 0).float().mean().item(), d.max().item()


def max_rel(out, ref):
    out = out.float().cpu()
    ref = ref.float().cpu()
    return ((out - ref).abs().max() / ref.abs().max().clamp(min=1e-12)).item()


# ----------------------------------------------------------------------------- quant
@pytest.mark.parametrize("M,K", [(257, 1536), (64, 8960), (33, 24), (1, 1536), (128, 4608)])
@pytest.mark.parametrize("mode", ["tensor", "token"])
def test_quantize_fp8_bitexact(M, K, mode):
    from flashvsr_sm89_ops_b200 import quantize_fp8
    x = O.fp8_outlier_activations(M, K, gen(M + K))
    q, s = quantize_fp8(x.to(DEV), mode)
    qr, sr = O.quantize_fp8(x, mode)
    assert torch.equal(q.view(torch.uint8).cpu(), qr.view(torch.uint8))
    assert torch.equal(s.cpu(), sr.float())


@pytest.mark.parametrize("M,K", [(8448, 1536), (16896, 1536), (8448, 8960)])
@pytest.mark.parametrize("mode", ["tensor", "token"])
def test_quantize_fp8_bitexact_step_shapes(M, K, mode):
    """The step's row counts: every warp of the per-token kernel carries several rows (its
    two-row pipeline), which the small shapes above never reach."""
    from flashvsr_sm89_ops_b200 import quantize_fp8
    x = O.fp8_outlier_activations(M, K, gen(M + 2 * K))
    q, s = quantize_fp8(x.to(DEV), mode)
    qr, sr = O.quantize_fp8(x, mode)
    assert torch.equal(q.view(torch.uint8).cpu(), qr.view(torch.uint8))
    assert torch.equal(s.cpu(), sr.float())


@pytest.mark.parametrize("mode", ["tensor", "token"])
def test_oracle_on_gpu_quantizes_like_oracle_on_cpu(mode):
    """The block-level checks evaluate the oracle's torch code on the GPU; its quantisation
    must give the CPU oracle's codes and scales bit for bit (a division by a host scalar on
    a CUDA tensor is a reciprocal multiply, which div_ieee keeps out)."""
    g = gen(77)
    x = (torch.randn(8448, 1536, generator=g) * 3).to(torch.bfloat16)
    x[::5, 0] = 7.0 * 2.0 ** torch.randint(-2, 4, (x[::5].shape[0],), generator=g).float()  # ties
    qg, sg = O.quantize_fp8(x.to(DEV), mode)
    qc, sc = O.quantize_fp8(x, mode)
    assert torch.equal(qg.view(torch.uint8).cpu(), qc.view(torch.uint8))
    assert torch.equal(sg.cpu(), sc)


def _near_midpoint_rows(rows, K, seed):
    """bf16 rows whose quotients x / s (s = row amax / 448, the reference's fp32 IEEE
    divide) sit on or next to e4m3 rounding midpoints or in the e4m3 subnormal range.
    Even rows: s with few mantissa bits, so x / s is exactly a midpoint m (a tie).  Odd
    rows: an amax found by search for which some bf16 x round to a different e4m3 code
    through x * fl(1/s) than through x / s; the row holds those x (both signs)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    mids = [(1 + (2 * i + 1) / 16) * 2.0 ** k for k in range(-6, 9) for i in range(8)]
    mids = [m for m in mids if m < 448] + [(2 * i + 1) * 2.0 ** -10 for i in range(8)]
    mids = np.array(mids + [1.0, 1.125, 2.0 ** -7, 448.0], np.float64)
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.int16)
    allx = torch.from_numpy(bits).view(torch.bfloat16).float().numpy()
    allx = allx[np.isfinite(allx)]

    def codes(v):
        return torch.from_numpy(np.clip(v, -448, 448).astype(np.float32)).to(
            torch.float8_e4m3fn).view(torch.uint8).numpy()

    out = np.zeros((rows, K), np.float32)
    for r in range(rows):
        if r % 2 == 0:
            s = (1.0, 1.5, 1.25)[r // 2 % 3] * 2.0 ** int(rng.integers(-8, 2))
            amax = 448 * s
            pick = np.resize(mids * s * rng.choice([-1.0, 1.0], size=mids.size), K - 1)
        else:
            while True:
                amax = float(torch.tensor(rng.uniform(0.01, 100)).to(torch.bfloat16).float())
                sf = np.float32(amax) / np.float32(448.0)
                xs = allx[np.abs(allx) <= amax]
                diff = xs[codes(xs / sf) != codes(xs * (np.float32(1.0) / sf))]
                if diff.size:
                    break
            pick = np.resize(np.concatenate([diff, -diff]), K - 1)
        out[r, :K - 1] = pick
        out[r, K - 1] = amax
    x = torch.from_numpy(out).to(torch.bfloat16)
    assert torch.equal(x.float(), torch.from_numpy(out))  # every value exact in bf16
    return x


def test_quantize_fp8_near_midpoints():
    """Quotients next to e4m3 rounding midpoints and in the subnormal range: the codes must
    still equal the reference's IEEE divide (token mode, row kernels and the FFN path's
    quantisation with a given amax)."""
    from flashvsr_sm89_ops_b200 import _lib, quantize_fp8
    x = _near_midpoint_rows(16, 1536, 5)
    q, s = quantize_fp8(x.to(DEV), "token")
    qr, sr = O.quantize_fp8(x, "token")
    assert torch.equal(q.view(torch.uint8).cpu(), qr.view(torch.uint8))
    assert torch.equal(s.cpu(), sr.float())
    xd = x.to(DEV)
    amax = xd.float().abs().amax(dim=1).contiguous()
    q2 = torch.empty_like(q)
    s2 = torch.empty_like(s)
    _lib.call("fvb_quant_fp8_with_amax", _lib.ptr(xd), x.shape[0], x.shape[1], _lib.ptr(amax),
              _lib.FVB_SCALE_ROW, _lib.ptr(q2), _lib.ptr(s2), _lib.stream_of(xd))
    assert torch.equal(q2.view(torch.uint8).cpu(), qr.view(torch.uint8))


@pytest.mark.parametrize("M,K", [(1, 8), (5, 8960), (1000, 8960), (297, 1536), (6000, 1536),
                                 (8448, 8960), (3, 12288), (7, 12296)])
@pytest.mark.parametrize("mode", ["token", "tensor"])
def test_quant_with_amax_shapes_bitexact(M, K, mode):
    """The quantiser given the amax (the FFN's hidden quantisation): fewer rows than warps,
    a few rows per warp and the step's 8448 x 8960, row lengths from one vector to 12296
    (a ragged last round of a lane's four loads), both scale modes, against the oracle."""
    from flashvsr_sm89_ops_b200 import _lib
    x = (torch.randn(M, K, generator=gen(M + K)) * 2).to(torch.bfloat16)
    qr, sr = O.quantize_fp8(x, mode)
    xd = x.to(DEV)
    a = xd.float().abs()
    amax = (a.amax(dim=1) if mode == "token" else a.amax().reshape(1)).contiguous()
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=DEV)
    s = torch.empty(M if mode == "token" else 1, dtype=torch.float32, device=DEV)
    code = _lib.FVB_SCALE_ROW if mode == "token" else _lib.FVB_SCALE_TENSOR
    _lib.call("fvb_quant_fp8_with_amax", _lib.ptr(xd), M, K, _lib.ptr(amax), code, _lib.ptr(q),
              _lib.ptr(s), _lib.stream_of(xd))
    assert torch.equal(q.view(torch.uint8).cpu(), qr.view(torch.uint8))
    assert torch.equal(s.cpu().reshape(-1), sr.float().reshape(-1))
    assert _lib.device_error() == 0


def test_quantize_fp8_tensor_ragged_and_empty():
    from flashvsr_sm89_ops_b200 import quantize_fp8
    x = torch.randn(7, 13, generator=gen(3)).to(torch.bfloat16)
    q, s = quantize_fp8(x.to(DEV), "tensor")
    qr, sr = O.quantize_fp8(x, "tensor")
    assert torch.equal(q.view(torch.uint8).cpu(), qr.view(torch.uint8))
    assert torch.equal(s.cpu(), sr)
    q0, s0 = quantize_fp8(torch.empty(0, 1536, dtype=torch.bfloat16, device=DEV))
    assert q0.shape == (0, 1536) and s0.item() == 0.0
    z = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    qz, sz = quantize_fp8(z, "token")
    assert qz.view(torch.uint8).eq(0).all() and sz.eq(0).all()


@pytest.mark.parametrize("mode", ["tensor", "token"])
def test_gelu_quant_matches_gpu_eager_bitexact(mode):
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_quant import fused_gelu_quant_fp8
    h = (torch.randn(96, 8960, generator=gen(5)) * 3).to(torch.bfloat16).to(DEV)
    q, s = fused_gelu_quant_fp8(h, mode)
    g = F.gelu(h, approximate="tanh")  # torch eager on the same GPU
    qe, se = quantize_fp8(g, mode)
    assert torch.equal(s, se)
    neq = (q.view(torch.uint8) != qe.view(torch.uint8)).sum().item()
    assert neq == 0, f"{neq} codes differ from quantize_fp8(F.gelu(h)) on the GPU"
    # against the CPU oracle: CPU and CUDA tanh may differ by an fp32 ulp (rare bf16 flips)
    qr, sr = O.gelu_quant_fp8(h.cpu(), mode)
    d = (q.view(torch.uint8).cpu().to(torch.int16) - qr.view(torch.uint8).to(torch.int16)).abs()
    assert d.max().item() <= 1 and (d > 0).float().mean().item() < 1e-3


@pytest.mark.parametrize("rows", ["every_bf16", "step", "small_max"])
def test_gelu_quant_long_rows_bitexact(rows):
    """Per-token GELU -> FP8 on rows longer than 2048 (the FFN hidden, 8960 wide): one warp
    per row, GELU from a shared table, the row amax taken as GELU(row max) when that is at
    least every negative input's |GELU|, else from GELU of every element.  Codes and scales
    must equal quantize_fp8(F.gelu(h)) on the GPU bit for bit: for every bf16 input value
    (NaN patterns zeroed; rows holding +-inf included), at the step's 8448 rows (each warp
    takes several rows in turn), and on rows whose maximum is too small for the shortcut
    (values in [-4, 0.25], an all-negative row, a row peaking near the bound)."""
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_quant import fused_gelu_quant_fp8
    K = 8960
    if rows == "every_bf16":
        x = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
        x = torch.where(torch.isnan(x), torch.zeros_like(x), x)
        x = torch.cat([x, torch.zeros(8 * K - x.numel(), dtype=torch.bfloat16)]).view(8, K)
        h = x[torch.randperm(8, generator=gen(8))].contiguous().to(DEV)
    elif rows == "step":
        h = (torch.randn(8448, K, generator=gen(9)) * 2).to(torch.bfloat16).to(DEV)
    else:
        g = gen(10)
        h = torch.rand(16, K, generator=g) * 4.25 - 4.0       # max 0.25: GELU 0.149 < ~0.17
        h[1] = -torch.rand(K, generator=g) * 3 - 0.01         # all negative
        h[2, :] = -0.75                                       # |GELU| at its negative peak,
        h[2, 7] = 0.279296875                                 # tied by GELU of this peak
        h[3, :] = -0.75
        h[3, 7] = 0.27734375                                  # one bf16 step below: the
        #                                                       negative inputs set the amax
        h = h.to(torch.bfloat16).to(DEV)
    q, s = fused_gelu_quant_fp8(h, "token")
    qe, se = quantize_fp8(F.gelu(h, approximate="tanh"), "token")
    assert torch.equal(s, se)
    neq = (q.view(torch.uint8) != qe.view(torch.uint8)).sum().item()
    assert neq == 0, f"{neq} codes differ from quantize_fp8(F.gelu(h))"


@pytest.mark.parametrize("case", ["every_bf16", "small_max", "all_negative", "tie", "below_tie",
                                  "ragged"])
def test_gelu_quant_tensor_mode_bitexact(case):
    """Per-tensor GELU -> FP8 (the reference's default mode) takes the amax as GELU(max h) when
    that bounds every negative input's |GELU|, else from GELU of every element; both paths
    and a ragged tail must give quantize_fp8(F.gelu(h), "tensor") on the GPU bit for bit."""
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_quant import fused_gelu_quant_fp8
    g = gen(11)
    if case == "every_bf16":
        h = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
        h = torch.where(torch.isnan(h), torch.zeros_like(h), h)
        h = h[torch.isfinite(h)]  # the finite values: GELU(+inf) would make the amax inf
        h = torch.cat([h, torch.zeros(-h.numel() % 64, dtype=h.dtype)]).view(-1, 64)
    elif case == "small_max":
        h = torch.rand(64, 1024, generator=g) * 4.25 - 4.0
    elif case == "all_negative":
        h = -torch.rand(64, 1024, generator=g) * 3 - 0.01
    elif case in ("tie", "below_tie"):
        h = torch.full((64, 1024), -0.75)
        h[5, 9] = 0.279296875 if case == "tie" else 0.27734375
    else:
        h = torch.randn(7, 13, generator=g) * 3
    h = h.to(torch.bfloat16).to(DEV)
    q, s = fused_gelu_quant_fp8(h, "tensor")
    qe, se = quantize_fp8(F.gelu(h, approximate="tanh"), "tensor")
    assert torch.equal(s, se)
    assert torch.equal(q.view(torch.uint8), qe.view(torch.uint8))


# ----------------------------------------------------------------------------- AdaLN
def test_gate_add_bitwise():
    from flashvsr_sm89_ops_b200 import fused_gate_add
    B, L, D = 2, 528, 1536
    x = torch.randn(B, L, D, generator=gen(1)).to(torch.bfloat16)
    r = torch.randn(B, L, D, generator=gen(2)).to(torch.bfloat16)
    g = torch.randn(B, 1, D, generator=gen(3)).to(torch.bfloat16)
    out = fused_gate_add(x.to(DEV), g.to(DEV), r.to(DEV)).cpu()
    assert torch.equal(out, O.gate_add(x, g, r))
    assert torch.equal(out, x + g * r)  # eager bf16 (fused_adaln.py:8-12 "bitwise")


@pytest.mark.parametrize("B,L,D", [(1, 16896, 1536), (2, 37, 256)])
def test_ln_modulate(B, L, D):
    from flashvsr_sm89_ops_b200 import fused_ln_modulate, quantize_fp8
    x = (torch.randn(B, L, D, generator=gen(4)) * 2 + 0.5).to(torch.bfloat16)
    mod = torch.randn(B, 6, D, generator=gen(5)).to(torch.bfloat16)
    shift, scale = mod[:, 0:1].contiguous(), mod[:, 1:2].contiguous()
    out, q8, qs = fused_ln_modulate(x.to(DEV), scale.to(DEV), shift.to(DEV), emit_fp8=True)
    ref = O.ln_modulate(x, scale, shift)
    # operand of the final add: bf16(xn * bf16(1 + scale))
    xf = x.float()
    xn = (xf - xf.mean(-1, keepdim=True)) / torch.sqrt(xf.var(-1, unbiased=False, keepdim=True) + 1e-6)
    y1 = xn * (1 + scale.float())
    # xn itself may differ by one bf16 ulp (fp32 mean/var summation order), scaled by (1+s)
    ok, frac, dmax = within_ulps(out, ref, y1, extra=(1 + scale.float()).abs() * bf16_ulp(xn))
    assert ok and frac < 1e-3, (frac, dmax)
    qq, ss = quantize_fp8(out.reshape(-1, D), "token")
    assert torch.equal(q8.view(torch.uint8), qq.view(torch.uint8)) and torch.equal(qs, ss)


@pytest.mark.parametrize("L,D,with_bias", [(4224, 1536, True), (37, 256, False)])
def test_layer_norm_affine(L, D, with_bias):
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200.fused_adaln import layer_norm
    x = torch.randn(1, L, D, generator=gen(6)).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(D, generator=gen(7))).to(torch.bfloat16)
    b = (0.1 * torch.randn(D, generator=gen(8))).to(torch.bfloat16) if with_bias else None
    out = layer_norm(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV))
    xf = x.float()
    xn = (xf - xf.mean(-1, keepdim=True)) / torch.sqrt(xf.var(-1, unbiased=False, keepdim=True) + 1e-6)
    ok, frac, dmax = within_ulps(out, O.layer_norm(x, w, b), xn * w.float())
    assert ok and frac < 1e-2, (frac, dmax)
    # the FP8 emission equals quantising the bf16 output per token
    out2, q8, qs = layer_norm(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), emit_fp8=True)
    assert torch.equal(out2, out)
    qq, ss = quantize_fp8(out.reshape(-1, D), "token")
    assert torch.equal(q8.view(torch.uint8), qq.view(torch.uint8)) and torch.equal(qs, ss)


@pytest.mark.parametrize("B,L,D,gated", [(1, 4224, 1536, True), (2, 37, 256, False)])
def test_gate_add_fused_norms(B, L, D, gated):
    """The gated residual add fused into LN-modulate / affine LayerNorm equals the two
    separate kernels bit for bit (residual, bf16 output and FP8 codes), with and without
    the bf16 output."""
    from flashvsr_sm89_ops_b200.fused_adaln import (fused_gate_add, fused_ln_modulate,
                                                    gate_add_layer_norm, gate_add_ln_modulate,
                                                    layer_norm)
    x = torch.randn(B, L, D, generator=gen(11)).to(torch.bfloat16).to(DEV)
    r = torch.randn(B, L, D, generator=gen(12)).to(torch.bfloat16).to(DEV)
    g = torch.randn(B, 1, D, generator=gen(13)).to(torch.bfloat16).to(DEV) if gated else None
    mod = torch.randn(B, 2, D, generator=gen(14)).to(torch.bfloat16).to(DEV)
    shift, scale = mod[:, 0:1].contiguous(), mod[:, 1:2].contiguous()
    w = (1 + 0.1 * torch.randn(D, generator=gen(15))).to(torch.bfloat16).to(DEV)
    b = (0.1 * torch.randn(D, generator=gen(16))).to(torch.bfloat16).to(DEV)
    xs = fused_gate_add(x, g, r)
    o1, q1, s1 = fused_ln_modulate(xs, scale, shift, emit_fp8=True)
    xn, o, q, qs = gate_add_ln_modulate(x, g, r, scale, shift, emit_fp8=True)
    assert torch.equal(xn, xs) and torch.equal(o, o1)
    assert torch.equal(q.view(torch.uint8), q1.view(torch.uint8)) and torch.equal(qs, s1)
    xn, o, q, qs = gate_add_ln_modulate(x, g, r, scale, shift, emit_fp8=True, want_out=False)
    assert o is None and torch.equal(xn, xs)
    assert torch.equal(q.view(torch.uint8), q1.view(torch.uint8)) and torch.equal(qs, s1)
    o2, q2, s2 = layer_norm(xs, w, b, emit_fp8=True)
    xn, o, q, qs = gate_add_layer_norm(x, g, r, w, b, emit_fp8=True)
    assert torch.equal(xn, xs) and torch.equal(o, o2)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(qs, s2)
    xn, o, q, qs = gate_add_layer_norm(x, g, r, w, b, emit_fp8=True, want_out=False)
    assert o is None and torch.equal(xn, xs) and torch.equal(q.view(torch.uint8), q2.view(torch.uint8))
    xn, o = gate_add_layer_norm(x, g, r, w, None)
    assert torch.equal(xn, xs) and torch.equal(o, layer_norm(xs, w, None))


# ----------------------------------------------------------------------------- RMS+RoPE
def _wan_freqs(L):
    from oracle.wan import grid_freqs
    f, h, w = 4, 48, 88
    assert f * h * w == L
    return grid_freqs(f, h, w)


@pytest.mark.parametrize("rope", [True, False])
def test_rms_rope(rope):
    from flashvsr_sm89_ops_b200 import fused_rms_rope
    L, D = 16896, 1536
    x = torch.randn(1, L, D, generator=gen(9)).to(torch.bfloat16)
    wgt = (1 + 0.1 * torch.randn(D, generator=gen(10))).to(torch.bfloat16)
    freqs = _wan_freqs(L)
    out = fused_rms_rope(x.to(DEV), wgt.to(DEV), freqs.to(DEV), eps=1e-6, rope=rope)
    cos, sin = O.freqs_cos_sin(freqs)
    ref = O.rms_rope(x, wgt, cos, sin, eps=1e-6, rope=rope)
    # operands of the rotation: the normalised pair (y_e, y_o); without RoPE the result itself
    y = O.rms_rope(x, wgt, rope=False).float()
    pair = y.view(1, L, D // 2, 2).abs().amax(-1, keepdim=True).expand(1, L, D // 2, 2).reshape(1, L, D)
    ok, frac, dmax = within_ulps(out, ref, pair if rope else ref.float())
    assert ok and frac < 1e-3, (frac, dmax)


# ----------------------------------------------------------------------------- layout
def test_window_partition_roundtrip():
    from flashvsr_sm89_ops_b200.lcsa import window_partition, window_reverse
    f, h, w, C = 4, 48, 88, 1536
    x = torch.randn(1, f * h * w, C, generator=gen(11)).to(torch.bfloat16)
    xw = window_partition(x.to(DEV), (f, h, w))
    ref = O.window_partition(x.view(1, f, h, w, C)).reshape(-1, C)
    assert torch.equal(xw.cpu(), ref)
    back = window_reverse(xw, (f, h, w))
    assert torch.equal(back.cpu(), x.view(-1, C))


def test_mask_to_csr_exact():
    from flashvsr_sm89_ops_b200.lcsa import build_csr
    keep = torch.rand(12, 66, 264, generator=gen(12)) < 0.3
    keep[0, 0] = False
    keep[1, 1] = True
    sel, cnt, maxk = build_csr(keep.to(DEV))
    sr, cr = O.build_csr(keep)
    assert maxk == 264
    assert torch.equal(cnt.cpu(), cr) and torch.equal(sel.cpu(), sr)


# ----------------------------------------------------------------------------- GEMM
GEMM_CASES = [
    (4224, 1536, 1536), (4224, 4608, 1536), (512, 8960, 1536), (512, 1536, 8960),
    (300, 200, 80), (129, 264, 48), (1, 1536, 1536),
]


@pytest.mark.parametrize("M,N,K", GEMM_CASES)
@pytest.mark.parametrize("mode", ["tensor", "token"])
def test_fp8_gemm(M, N, K, mode):
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm, quantize_weight
    g = gen(M * 7 + N + K)
    x = O.fp8_outlier_activations(M, K, g)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    qw, sw = quantize_weight(w.to(DEV), mode)
    qx, sx = quantize_fp8(x.to(DEV), mode)
    out = fp8_mm(qx, sx, qw, sw, b.to(DEV))
    qwr, swr = O.fp8_weight(w, mode)
    assert torch.equal(qw.view(torch.uint8).cpu(), qwr.view(torch.uint8))
    ref = O.fp8_mm(qx.cpu(), sx.cpu(), qwr, swr, b)
    assert max_rel(out, ref) < 1e-2


@pytest.mark.parametrize("epilogue", [0])
def test_fp8_gemm_cta_pair_rows_equal_single_cta(epilogue):
    """Wide GEMMs (N >= 4096, plain epilogue) with more than 128 rows run on CTA pairs
    (cta_group::2, 256-row tiles: the even CTA's TMEM holds rows 0-127 of a tile, the odd
    CTA's rows 128-255).
    Every row must be bit for bit what the single-CTA kernel (M <= 128) gives for that row
    alone: rows 0-127 from the even CTA, 128-255 from the odd one, 256-299 from a pair whose
    odd CTA has no valid row.  N = 4104 also leaves a ragged last column tile."""
    from flashvsr_sm89_ops_b200 import _lib, quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm, quantize_weight
    M, N, K = 300, 4104, 1536
    g = gen(77)
    x = O.fp8_outlier_activations(M, K, g)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    qw, sw = quantize_weight(w.to(DEV), "token")
    qx, sx = quantize_fp8(x.to(DEV), "token")

    def run(lo, hi):
        amax = torch.zeros(hi - lo, device=DEV)
        kw = dict(epilogue=_lib.FVB_EPI_GELU_AMAX, amax_out=amax) if epilogue else {}
        y = fp8_mm(qx[lo:hi].contiguous(), sx[lo:hi].contiguous(), qw, sw, b, **kw)
        return y, amax

    whole, amax_whole = run(0, M)
    for lo, hi in ((0, 128), (128, 256), (256, M)):
        part, amax_part = run(lo, hi)
        assert torch.equal(whole[lo:hi], part), (lo, hi)
        if epilogue:
            assert torch.equal(amax_whole[lo:hi], amax_part), (lo, hi)


# every (K -> N) pair at the two large token counts.  The GEMM
# runs in full on the GPU; the oracle (fp32 product of the decoded codes, CPU) checks two
# rows of every 128-row tile (rows are independent, so a tile's rows share its code path).
BIG_GEMM = [(M, N, K) for M in (16896, 33792)
            for (K, N) in ((1536, 1536), (1536, 4608), (1536, 8960), (8960, 1536))]


@pytest.mark.parametrize("M,N,K", BIG_GEMM)
@pytest.mark.parametrize("mode", ["token", "tensor"])
def test_fp8_gemm_bench_shapes(M, N, K, mode):
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm, quantize_weight
    gd = torch.Generator(device=DEV).manual_seed(M + 3 * N + 7 * K)
    x = torch.randn(M, K, generator=gd, device=DEV)
    x = torch.where(torch.rand(M, K, generator=gd, device=DEV) < 0.01, x * 20, x).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, generator=gd, device=DEV)).to(torch.bfloat16)
    b = (0.02 * torch.randn(N, generator=gd, device=DEV)).to(torch.bfloat16)
    qw, sw = quantize_weight(w, mode)
    qx, sx = quantize_fp8(x, mode)
    out = fp8_mm(qx, sx, qw, sw, b)
    torch.cuda.synchronize()
    qwr, swr = O.fp8_weight(w.cpu(), mode)
    assert torch.equal(qw.view(torch.uint8).cpu(), qwr.view(torch.uint8))
    g = gen(M + N + K)
    tiles = torch.arange(0, M, 128)
    rows = torch.cat([tiles + torch.randint(0, 128, tiles.shape, generator=g),
                      tiles + torch.randint(0, 128, tiles.shape, generator=g)]).clamp(max=M - 1)
    rows = torch.unique(torch.cat([rows, torch.tensor([0, M - 1])]))
    sxr = sx.cpu()[rows] if mode == "token" else sx.cpu()
    ref = O.fp8_mm(qx[rows.to(DEV)].cpu(), sxr, qwr, swr, b.cpu())
    got = out[rows.to(DEV)]
    assert max_rel(got, ref) < 1e-2
    # same codes on both sides: only fp32 summation order and the final bf16 rounding differ
    assert (got.float().cpu() - ref.float()).norm().item() / ref.float().norm().item() < 1e-4
    assert torch.isfinite(out.float()).all()


def test_fp8_gemm_gelu_epilogue_amax():
    from flashvsr_sm89_ops_b200 import quantize_fp8
    from flashvsr_sm89_ops_b200 import _lib
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm, quantize_weight
    M, N, K = 1000, 8960, 1536
    g = gen(21)
    x = O.fp8_outlier_activations(M, K, g)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    qw, sw = quantize_weight(w.to(DEV), "token")
    qx, sx = quantize_fp8(x.to(DEV), "token")
    amax = torch.zeros(M, device=DEV)
    h = fp8_mm(qx, sx, qw, sw, b.to(DEV), epilogue=_lib.FVB_EPI_GELU_AMAX, amax_out=amax)
    plain = fp8_mm(qx, sx, qw, sw, b.to(DEV))
    ge = F.gelu(plain, approximate="tanh")
    assert torch.equal(h, ge), "GELU epilogue differs from eager GELU of the plain GEMM output"
    assert torch.equal(amax, ge.float().abs().amax(dim=1))


def test_gelu_epilogue_every_bf16_input():
    """Every bf16 value (finite and infinite) through the GELU epilogue: A is zero, so the
    bias column carries x, and each output must equal eager GELU of the plain GEMM output
    bit for bit (the table's range and the rules outside it are checked exhaustively)."""
    from flashvsr_sm89_ops_b200 import _lib
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm
    x = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    x = torch.where(torch.isnan(x), torch.zeros_like(x), x).to(DEV)
    M, K, N = 32, 16, x.numel()
    qa = torch.zeros(M, K, dtype=torch.float8_e4m3fn, device=DEV)
    qw = torch.zeros(N, K, dtype=torch.float8_e4m3fn, device=DEV)
    one = torch.ones(1, device=DEV)
    amax = torch.zeros(1, device=DEV)
    h = fp8_mm(qa, one, qw, one, x, epilogue=_lib.FVB_EPI_GELU_AMAX, amax_out=amax)
    plain = fp8_mm(qa, one, qw, one, x)
    ge = F.gelu(plain, approximate="tanh")
    nan = torch.isnan(ge)
    assert torch.equal(torch.isnan(h), nan)
    hv, gv = h.view(torch.int16)[~nan], ge.view(torch.int16)[~nan]
    bad = (hv != gv).sum().item()
    assert bad == 0, f"{bad} of {hv.numel()} GELU outputs differ from eager"


@pytest.mark.parametrize("mode", ["tensor", "token"])
def test_fp8_ffn(mode):
    from flashvsr_sm89_ops_b200.fp8_ffn import FP8FFN
    from flashvsr_sm89_ops_b200.fp8_linear import FP8Linear
    D, Fh, M = 1536, 8960, 777
    g = gen(31)
    l0 = torch.nn.Linear(D, Fh)
    l2 = torch.nn.Linear(Fh, D)
    with torch.no_grad():
        for lin in (l0, l2):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.02)
    l0 = l0.to(torch.bfloat16)
    l2 = l2.to(torch.bfloat16)
    import copy
    ffn = FP8FFN(FP8Linear(copy.deepcopy(l0).to(DEV), mode), FP8Linear(copy.deepcopy(l2).to(DEV), mode))
    x = torch.randn(1, M, D, generator=g).to(torch.bfloat16)
    out = ffn(x.to(DEV))
    q0, s0 = O.fp8_weight(l0.weight.detach(), mode)
    q2, s2 = O.fp8_weight(l2.weight.detach(), mode)
    ref = O.fp8_ffn(x, q0, s0, l0.bias.detach(), q2, s2, l2.bias.detach(), mode)
    assert max_rel(out, ref) < 1e-2


@pytest.mark.parametrize("mode", ["tensor", "token"])
@pytest.mark.parametrize("gated", [True, False])
def test_fp8_ffn_residual_equals_ffn_then_gate_add(mode, gated):
    """fvb_fp8_ffn_residual (the gated residual add in the down-projection's epilogue) is bit
    for bit fused_gate_add(x, gate, FFN(x_in)) -- the DiT block's closing update."""
    from flashvsr_sm89_ops_b200 import fused_gate_add, quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_ffn import ffn_fp8
    from flashvsr_sm89_ops_b200.fp8_linear import FP8Linear
    D, Fh, M = 1536, 8960, 1000
    g = gen(33)
    l0 = torch.nn.Linear(D, Fh).to(torch.bfloat16)
    l2 = torch.nn.Linear(Fh, D).to(torch.bfloat16)
    with torch.no_grad():
        for lin in (l0, l2):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.02)
    f0, f2 = FP8Linear(l0.to(DEV), mode), FP8Linear(l2.to(DEV), mode)
    xin = torch.randn(M, D, generator=g).to(torch.bfloat16).to(DEV)
    res = (torch.randn(1, M, D, generator=g) * 3).to(torch.bfloat16).to(DEV)
    gate = torch.randn(1, 1, D, generator=g).to(torch.bfloat16).to(DEV) if gated else None
    x8, sx = quantize_fp8(xin, mode)
    y = ffn_fp8(x8, sx, f0, f2)
    ref = fused_gate_add(res, gate, y.view(1, M, D))
    got = ffn_fp8(x8, sx, f0, f2, residual=res, gate=gate)
    assert torch.equal(got.view(1, M, D), ref)


# ----------------------------------------------------------------------------- attention
ATTN_CASES = [(16, 24, 0, 0.4), (32, 48, 0, 0.3), (48, 88, 198, 0.46)]  # lcsa/test_correctness.py:46-50


@pytest.mark.parametrize("h_lat,w_lat,nk_extra,ratio", ATTN_CASES)
def test_block_sparse_attention(h_lat, w_lat, nk_extra, ratio):
    from flashvsr_sm89_ops_b200.lcsa import block_sparse_attention
    H, Dh, S, f = 12, 128, 128, 2
    g = gen(0)
    L = f * h_lat * w_lat
    bh, bw = h_lat // 8, w_lat // 8
    Nq = (f // 2) * bh * bw
    Nk = Nq + nk_extra
    q = torch.randn(1, L, H * Dh, generator=g).to(torch.bfloat16)
    k = torch.randn(1, Nk * S, H * Dh, generator=g).to(torch.bfloat16)
    v = torch.randn(1, Nk * S, H * Dh, generator=g).to(torch.bfloat16)
    q_w = O.window_partition(q.view(1, f, h_lat, w_lat, H * Dh))
    local = O.local_block_mask(bh, bw, 11)
    keep = O.draft_block_mask(q_w, k.view(Nk, S, H * Dh), H, f // 2, local, int(Nq * Nk * ratio))
    keep[0, 0] = False  # an empty row must come back as zeros
    out = block_sparse_attention(q_w.reshape(1, -1, H * Dh).to(DEV), k.to(DEV), v.to(DEV), keep.to(DEV))
    ref = O.sparse_attention(q_w, k.view(Nk, S, H * Dh), v.view(Nk, S, H * Dh), keep).reshape(1, -1, H * Dh)
    assert torch.allclose(out.float().cpu(), ref, atol=1e-2, rtol=1e-2), \
        (out.float().cpu() - ref).abs().max().item()
    assert out[0, :S, :Dh].abs().max().item() == 0.0


def test_block_sparse_attention_cfg4():
    """q/k/v [1, 12, 16896, 128] N(0,1) in (2,8,8) windows, Nq = 132
    in two time rows of 66, the causal top-25% rule (117,216 kept pairs).  Whole output vs
    the kernel-order restatement evaluated on the GPU in fp32; a sample of (head, query
    window) pairs vs the reference's fp32 oracle (lcsa/reference.py:67-88) on the CPU at the
    reference test's atol = rtol = 1e-2 (lcsa/test_correctness.py:59)."""
    from flashvsr_sm89_ops_b200.lcsa import attention_csr, build_csr, causal_topk_mask
    H, Dh, S, NQ = 12, 128, 128, 132
    gd = torch.Generator(device=DEV).manual_seed(4)
    q_w = torch.randn(NQ, S, H * Dh, generator=gd, device=DEV).to(torch.bfloat16)
    k_w = torch.randn(NQ, S, H * Dh, generator=gd, device=DEV).to(torch.bfloat16)
    v_w = torch.randn(NQ, S, H * Dh, generator=gd, device=DEV).to(torch.bfloat16)
    keep = causal_topk_mask(q_w, k_w, H, 66, 0.25)
    assert keep.sum().item() == 117_216
    sel, cnt, _ = build_csr(keep)
    out = attention_csr(q_w.view(-1, H * Dh), k_w.view(-1, H * Dh), v_w.view(-1, H * Dh), sel, cnt, H)
    out = out.view(NQ, S, H * Dh).float()
    torch.cuda.synchronize()
    full = O.sparse_attention_online(q_w, k_w, v_w, keep, lazy=8.0)
    assert (out - full).abs().max().item() < 2e-2
    assert (out - full).norm().item() / full.norm().item() < 3e-3
    g = gen(44)
    pairs = [(0, i) for i in range(NQ)] + [(int(h), int(i)) for h, i in zip(
        torch.randint(1, H, (48,), generator=g), torch.randint(0, NQ, (48,), generator=g))]
    keep_c = keep.cpu()
    ref = O.sparse_attention(q_w.cpu(), k_w.cpu(), v_w.cpu(), keep_c, pairs=pairs)
    oc = out.cpu().view(NQ, S, H, Dh)
    rc = ref.view(NQ, S, H, Dh)
    for h, i in pairs:
        assert torch.allclose(oc[i, :, h], rc[i, :, h], atol=1e-2, rtol=1e-2), (h, i)


def test_long_list_attention_kernel_order():
    """Key lists of >= 16 blocks take the two-window kernel (two query windows per CTA sharing
    one score buffer).  An odd number of query windows (the last CTA has one), rows with 0, 1,
    2, 3 kept blocks, a ragged key tail (kv_len) and a row map; checked against the oracle's
    restatement of the kernel's evaluation order (tight) and the reference order (loose)."""
    from flashvsr_sm89_ops_b200.lcsa import attention_csr, build_csr
    H, Dh, S, NQ, NK = 4, 128, 128, 7, 20
    g = gen(17)
    q_w = torch.randn(NQ, S, H * Dh, generator=g).to(torch.bfloat16)
    k_w = torch.randn(NK, S, H * Dh, generator=g).to(torch.bfloat16)
    v_w = torch.randn(NK, S, H * Dh, generator=g).to(torch.bfloat16)
    keep = torch.rand(H, NQ, NK, generator=g) < 0.5
    for i, n in enumerate([0, 1, 2, 3]):
        keep[i % H, i] = False
        keep[i % H, i, torch.randperm(NK, generator=g)[:n]] = True
    keep[:, 5, NK - 1] = True  # the tail block (partly past kv_len)
    kv_len = NK * S - 37
    sel, cnt, _ = build_csr(keep.to(DEV))
    row_map = torch.randperm(NQ * S, generator=g).to(torch.int32)
    out = attention_csr(q_w.reshape(-1, H * Dh).to(DEV), k_w.reshape(-1, H * Dh).to(DEV),
                        v_w.reshape(-1, H * Dh).to(DEV), sel, cnt, H, kv_len=kv_len,
                        row_map=row_map.to(DEV))
    got = torch.empty_like(out)
    got[torch.arange(NQ * S, device=DEV)] = out[row_map.long().to(DEV)]
    got = got.float().cpu().view(NQ, S, H * Dh)
    ref = O.sparse_attention_online(q_w, k_w, v_w, keep, kv_len=kv_len, lazy=8.0)
    assert (got - ref).abs().max().item() < 2e-2
    assert (got - ref).norm().item() / ref.norm().item() < 3e-3
    ref32 = O.sparse_attention_online(q_w, k_w, v_w, keep, kv_len=kv_len)  # reference order
    assert torch.allclose(got, ref32, atol=1e-2, rtol=1e-2)
    assert got[0].view(S, H, Dh)[:, 0].abs().max().item() == 0.0  # row with no kept block


def test_dense_attention_cross():
    from flashvsr_sm89_ops_b200.lcsa import dense_attention
    H, Dh = 12, 128
    g = gen(41)
    q = torch.randn(1000, H * Dh, generator=g).to(torch.bfloat16)
    k = torch.randn(512, H * Dh, generator=g).to(torch.bfloat16)
    v = torch.randn(512, H * Dh, generator=g).to(torch.bfloat16)
    out = dense_attention(q.to(DEV), k.to(DEV), v.to(DEV), H)
    ref = O.dense_attention(q, k, v, H)
    assert torch.allclose(out.float().cpu(), ref, atol=1e-2, rtol=1e-2)
    k2 = torch.randn(300, H * Dh, generator=g).to(torch.bfloat16)  # ragged key count
    v2 = torch.randn(300, H * Dh, generator=g).to(torch.bfloat16)
    out2 = dense_attention(q.to(DEV), k2.to(DEV), v2.to(DEV), H)
    assert torch.allclose(out2.float().cpu(), O.dense_attention(q, k2, v2, H), atol=1e-2, rtol=1e-2)


# ----------------------------------------------------------------------------- masks
# Keep masks are index output: the device builders must equal the oracle bit for bit.
# Both rules state their fp32 evaluation order (oracle.ops.block_mean_ordered, ascending
# dot products, double-precision exp), which the kernels follow.
MASK_SHAPES = [(66, 264), (132, 132)]  # the 1408x768 step (3 cached rows) and cfg 4


@pytest.mark.parametrize("nq,nk", MASK_SHAPES)
def test_draft_block_mask_device(nq, nk):
    from flashvsr_sm89_ops_b200.lcsa import draft_block_mask
    H, C, S = 12, 1536, 128
    g = gen(51 + nq)
    q_w = torch.randn(nq, S, C, generator=g).to(torch.bfloat16)
    k_w = torch.randn(nk, S, C, generator=g).to(torch.bfloat16)
    local = O.local_block_mask(6, 11, 11)
    qt = nq // 66
    topk = int(66 * nk * 0.46)
    keep = draft_block_mask(q_w.to(DEV), k_w.to(DEV), H, qt, local, topk).cpu()
    ref = O.draft_block_mask_ordered(q_w, k_w, H, qt, local, topk)
    assert torch.equal(keep, ref), (keep != ref).sum().item()
    # the ordered restatement against the torch-native one (pinned to the reference's own
    # draft_block_mask): they differ only where fp32 summation order moves a bf16 value
    native = O.draft_block_mask(q_w, k_w, H, qt, local, topk)
    assert (native != ref).float().mean().item() < 1e-4


def test_draft_block_mask_ties_at_threshold():
    """Equal probabilities at the threshold: the strict '>' keeps none of the tied entries
    (lcsa/reference.py:62-64), on the device as in the oracle."""
    from flashvsr_sm89_ops_b200.lcsa import draft_block_mask
    H, C, S, nq, nk = 12, 1536, 128, 66, 132
    g = gen(61)
    q_w = torch.randn(nq, S, C, generator=g).to(torch.bfloat16)
    base = torch.randn(nk // 4, S, C, generator=g).to(torch.bfloat16)
    k_w = base.repeat(4, 1, 1)  # every key window four times: scores tie in groups of 4
    local = torch.ones(66, 66, dtype=torch.bool)  # no local restriction: every key competes
    topk = 66 * 7 + 1  # a rank inside a tie group
    keep = draft_block_mask(q_w.to(DEV), k_w.to(DEV), H, 1, local, topk).cpu()
    ref = O.draft_block_mask_ordered(q_w, k_w, H, 1, local, topk)
    assert torch.equal(keep, ref)
    assert (keep.view(H, -1).sum(-1) <= topk).all()  # tied entries at the threshold dropped


@pytest.mark.parametrize("nq,nk", MASK_SHAPES)
def test_causal_topk_mask_device(nq, nk):
    from flashvsr_sm89_ops_b200.lcsa import causal_topk_mask
    H, C, S = 12, 1536, 128
    g = gen(52 + nq)
    q_w = torch.randn(nq, S, C, generator=g).to(torch.bfloat16)
    k_w = torch.randn(nk, S, C, generator=g).to(torch.bfloat16)
    keep = causal_topk_mask(q_w.to(DEV), k_w.to(DEV), H, 66, 0.25).cpu()
    ref = O.causal_topk_mask(q_w, k_w, H, 66, 0.25)
    assert torch.equal(keep, ref), (keep != ref).sum().item()
    if (nq, nk) == (132, 132):
        assert keep.sum().item() == 12 * (66 * 66 + 66 * 82)  # the configuration's kept pairs
    else:
        assert keep.sum().item() == 12 * 66 * (66 + 49)  # 91,080: the benchmark step
    # the streaming split: pooled means of the cached key blocks passed in, the rest pooled
    keep2, ak = causal_topk_mask(q_w.to(DEV), k_w.to(DEV), H, 66, 0.25, return_k_pool=True)
    assert torch.equal(keep2.cpu(), keep)
    assert torch.equal(ak.cpu(), O.block_mean_ordered(k_w))
    npre = nk - nq
    if npre:
        keep3 = causal_topk_mask(q_w.to(DEV), k_w.to(DEV), H, 66, 0.25,
                                 k_pool_prefix=ak[:npre].clone())
        assert torch.equal(keep3.cpu(), keep)
    # the CSR written by the rule's own launch (the block path) equals build_csr of the mask
    from flashvsr_sm89_ops_b200.lcsa import build_csr
    sel_r, cnt_r, _ = build_csr(keep.to(DEV))
    (sel, cnt, maxk), _ = causal_topk_mask(q_w.to(DEV), k_w.to(DEV), H, 66, 0.25,
                                           k_pool_prefix=ak[:npre].clone() if npre else None,
                                           return_k_pool=True, csr=True)
    assert maxk == nk and torch.equal(cnt, cnt_r) and torch.equal(sel, sel_r)


def test_causal_topk_mask_ties_take_lower_index():
    """Past key windows with identical content score equally; the rule keeps the lower
    indices of a tie group that straddles the selection boundary."""
    from flashvsr_sm89_ops_b200.lcsa import causal_topk_mask
    H, C, S, per_row = 12, 1536, 128, 66
    g = gen(62)
    q_w = torch.randn(per_row, S, C, generator=g).to(torch.bfloat16)
    past = torch.randn(per_row, S, C, generator=g).to(torch.bfloat16)
    past[10:40] = past[10]  # 30 equal past windows
    k_w = torch.cat([past, torch.randn(per_row, S, C, generator=g).to(torch.bfloat16)])
    keep = causal_topk_mask(q_w.to(DEV), k_w.to(DEV), H, per_row, 0.25).cpu()
    ref = O.causal_topk_mask(q_w, k_w, H, per_row, 0.25)
    assert torch.equal(keep, ref)
    kp = keep[:, :, 10:40]  # within the tie group, a kept window has every lower one kept
    taken = kp.sum(-1)
    for h in range(H):
        for i in range(per_row):
            n = int(taken[h, i])
            assert kp[h, i, :n].all() and not kp[h, i, n:].any()
    # the CSR path resolves the ties the same way
    from flashvsr_sm89_ops_b200.lcsa import build_csr
    sel, cnt, _ = causal_topk_mask(q_w.to(DEV), k_w.to(DEV), H, per_row, 0.25, csr=True)
    sel_r, cnt_r, _ = build_csr(keep.to(DEV))
    assert torch.equal(sel, sel_r) and torch.equal(cnt, cnt_r)


@pytest.mark.parametrize("B,L,D", [(1, 8448, 1536), (2, 37, 256)])
@pytest.mark.parametrize("want_out", [True, False])
def test_ln_modulate_adaln_equals_add_then_ln_modulate(B, L, D, want_out):
    """norm1 with the block's modulation sum in the same launch equals the eager
    `modulation + t_mod` followed by fused_ln_modulate on chunks 1 (scale) and 0 (shift), bit
    for bit: the six summed chunks, the bf16 output and the FP8 codes and scales."""
    from flashvsr_sm89_ops_b200 import fused_ln_modulate
    from flashvsr_sm89_ops_b200.fused_adaln import fused_ln_modulate_adaln
    g = gen(41)
    x = (torch.randn(B, L, D, generator=g) * 2).to(torch.bfloat16).to(DEV)
    modulation = (torch.randn(1, 6, D, generator=g) / D ** 0.5).to(torch.bfloat16).to(DEV)
    t_mod = torch.randn(B, 6, D, generator=g).to(torch.bfloat16).to(DEV)
    out, q8, qs, mod = fused_ln_modulate_adaln(x, modulation, t_mod, emit_fp8=True,
                                               want_out=want_out)
    ref_mod = modulation + t_mod
    assert torch.equal(mod, ref_mod)
    shift, scale = ref_mod[:, 0:1].contiguous(), ref_mod[:, 1:2].contiguous()
    ro, rq, rs = fused_ln_modulate(x, scale, shift, emit_fp8=True)
    if want_out:
        assert torch.equal(out, ro)
    else:
        assert out is None
    assert torch.equal(q8.view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(qs, rs)


@pytest.mark.parametrize("fhw", [(2, 48, 88), (2, 16, 24)])
def test_qkv_rope_window_equals_three_launches(fhw):
    """q / k RMSNorm + RoPE and the v window permute of the fused qkv projection in one
    launch equal the separate rms_rope_rows (q, k) and window_partition (v) launches bit for
    bit, rows in window order (the 1408x768 step's grid and a small one)."""
    from flashvsr_sm89_ops_b200 import lcsa
    from flashvsr_sm89_ops_b200.fused_rms_rope import qkv_rope_window, rms_rope_rows
    from flashvsr_sm89_ops_b200.integrate import _row_maps
    f, h, w = fhw
    L, D, hd = f * h * w, 1536, 128
    g = gen(61)
    qkv = (torch.randn(L, 3 * D, generator=g) * 3).to(torch.bfloat16).to(DEV)
    wq = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(DEV)
    wk = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(DEV)
    ang = torch.rand(L, hd // 2, generator=g) * 6.3
    cos, sin = torch.cos(ang).to(DEV), torch.sin(ang).to(DEV)
    r2w, _ = _row_maps(f, h, w, torch.device(DEV))
    oq, ok, ov = (torch.empty(L, D, dtype=torch.bfloat16, device=DEV) for _ in range(3))
    qkv_rope_window(qkv, wq, wk, cos, sin, L, 1e-6, 2e-6, hd, r2w, oq, ok, ov)
    rq = rms_rope_rows(qkv[:, :D], wq, cos, sin, L, 1e-6, True, hd, row_map=r2w)
    rk = rms_rope_rows(qkv[:, D:2 * D], wk, cos, sin, L, 2e-6, True, hd, row_map=r2w)
    rv = lcsa.window_partition(qkv[:, 2 * D:], (f, h, w))
    assert torch.equal(oq, rq)
    assert torch.equal(ok, rk)
    assert torch.equal(ov, rv)
