"""Run the reference's own GPU kernels (its Triton kernels and its torch._scaled_mm / cuBLASLt
call) on a B200, save their outputs as fixtures, and time them beside this pack's kernels.

    python tests/golden/make_golden_triton.py --reference <dir holding flashvsr_sm89_ops> \
        --out tests/golden/triton_b200.pt --timing <file.json>

<dir> is a checkout of aireet/flashvsr-sm89-ops or a pip --target install of it (the
reference is not vendored here).  Needs a CUDA GPU; the fixtures are committed so the
tests never need the reference at run time:
  * tests/test_oracle_golden.py pins the CPU oracle (oracle/ops.py) against them: the
    rows that had only a restated formula before (RMSNorm + RoPE fused_rms_rope.py:21-55,
    LN-modulate / gate-add fused_adaln.py:22-57, Triton quantisation fp8_quant.py:16-35,
    GELU -> FP8 fp8_ffn.py:24-72, the LCSA kernel lcsa/triton_lcsa.py:19-61);
  * tests/test_ref_triton_gpu.py compares this pack's kernels with them on the GPU.
Inputs are stored with the outputs (small shapes, D = 1536 as in the DiT).

--timing also times, at the benchmark step's shapes (1408x768, f=2: 8448 tokens), each
reference GPU op and this pack's replacement on the same GPU (CUDA events, warm, median of
5 runs of 20 launches) and writes a JSON summary.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _outliers(M, K, g):
    x = torch.randn(M, K, generator=g)
    return torch.where(torch.rand(M, K, generator=g) < 0.01, x * 20, x).to(torch.bfloat16)


def _freqs(L, seed):
    """complex64 [L, 1, 64] of unit modulus (a RoPE table over arbitrary positions)."""
    ang = torch.rand(L, 64, generator=_gen(seed)) * 2 * math.pi * 8
    return torch.polar(torch.ones_like(ang), ang).reshape(L, 1, 64)


def _near_tie_tensor(amax, rows, K):
    """bf16 [rows, K] whose max |x| is `amax` and whose other entries x have fp32 quotients
    x / s (s = fl(amax / 448), the kernel's scale) within two fp32 ulps of an e4m3 rounding
    midpoint: where an approximate divide and the IEEE divide could round to different
    codes."""
    import numpy as np
    allx = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float().numpy()
    allx = allx[np.isfinite(allx) & (np.abs(allx) <= amax) & (allx != 0)]
    s = np.float32(np.float32(amax) / np.float32(448.0))
    q = allx.astype(np.float64) / np.float64(s)
    vals = torch.arange(127, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy().astype(np.float64)
    mids = (vals[:-1] + vals[1:]) / 2
    aq = np.abs(q)
    idx = np.clip(np.searchsorted(mids, aq), 1, len(mids) - 1)
    near = np.minimum(np.abs(aq - mids[idx - 1]), np.abs(aq - mids[idx]))
    ulp = np.spacing(np.abs(q).astype(np.float32)).astype(np.float64)
    pick = allx[near <= 2 * ulp]
    out = np.resize(pick if pick.size else allx, rows * K).reshape(rows, K)
    out[0, 0] = amax
    return torch.from_numpy(out.astype(np.float32)).to(torch.bfloat16)


def make_fixtures(R, dev):
    """R: the reference package.  Returns {case: {inputs..., outputs...}} on the CPU."""
    out = {}
    # a1: quantize_fp8 (Triton absmax + quant kernels, per tensor)
    x = _outliers(64, 1536, _gen(1))
    q, s = R.quantize_fp8(x.to(dev))
    out["quant"] = {"x": x, "q": q.view(torch.uint8).cpu(), "scale": s.cpu()}
    # near e4m3 rounding midpoints: x / s lands on or next to a tie for many elements
    xm = (torch.randint(-448 * 4, 448 * 4 + 1, (64, 1536), generator=_gen(2)).float() / 4)
    xm[0, 0] = 448.0  # amax 448 -> s = 1: quotients are the quarter-step values themselves
    xm = xm.to(torch.bfloat16)
    q, s = R.quantize_fp8(xm.to(dev))
    out["quant_mid"] = {"x": xm, "q": q.view(torch.uint8).cpu(), "scale": s.cpu()}
    # quotients within two fp32 ulps of an e4m3 midpoint for three scales
    for i, amax in enumerate((3.71875, 0.0537109375, 96.5)):
        xe = _near_tie_tensor(amax, 16, 1536)
        q, s = R.quantize_fp8(xe.to(dev))
        out[f"quant_edge{i}"] = {"x": xe, "q": q.view(torch.uint8).cpu(), "scale": s.cpu()}
    # a5: fused_gelu_quant_fp8 (Triton GELU via the exp identity, bf16 round-trip, quant)
    h = (torch.randn(32, 8960, generator=_gen(3)) * 3).to(torch.bfloat16)
    q, s = R.fused_gelu_quant_fp8(h.to(dev))
    out["gelu_quant"] = {"h": h, "q": q.view(torch.uint8).cpu(), "scale": s.cpu()}
    # a7: fused_rms_rope, rope on and off
    x = torch.randn(1, 64, 1536, generator=_gen(4)).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(1536, generator=_gen(5))).to(torch.bfloat16)
    fr = _freqs(64, 6)
    y = R.fused_rms_rope(x.to(dev), w.to(dev), fr.to(dev), eps=1e-6, rope=True, head_dim=128)
    y0 = R.fused_rms_rope(x.to(dev), w.to(dev), None, eps=1e-6, rope=False, head_dim=128)
    out["rms_rope"] = {"x": x, "w": w, "freqs": fr, "y": y.cpu(), "y_norope": y0.cpu()}
    # a8 / a9: fused_ln_modulate (scale before shift) and fused_gate_add
    x = (torch.randn(1, 64, 1536, generator=_gen(7)) * 2 + 0.5).to(torch.bfloat16)
    sc = torch.randn(1, 1, 1536, generator=_gen(8)).to(torch.bfloat16)
    sh = torch.randn(1, 1, 1536, generator=_gen(9)).to(torch.bfloat16)
    y = R.fused_ln_modulate(x.to(dev), sc.to(dev), sh.to(dev), eps=1e-6)
    r = torch.randn(1, 64, 1536, generator=_gen(10)).to(torch.bfloat16)
    gt = torch.randn(1, 1, 1536, generator=_gen(11)).to(torch.bfloat16)
    ga = R.fused_gate_add(x.to(dev), gt.to(dev), r.to(dev))
    out["adaln"] = {"x": x, "scale": sc, "shift": sh, "y": y.cpu(), "r": r, "gate": gt,
                    "gate_add": ga.cpu()}
    # a12: block_sparse_attention (Triton LCSA), 2 heads, 4 query / 6 key windows
    H, NQ, NK = 2, 4, 6
    g = _gen(12)
    qa = torch.randn(1, NQ * 128, H * 128, generator=g).to(torch.bfloat16)
    ka = torch.randn(1, NK * 128, H * 128, generator=g).to(torch.bfloat16)
    va = torch.randn(1, NK * 128, H * 128, generator=g).to(torch.bfloat16)
    keep = torch.rand(H, NQ, NK, generator=g) < 0.5
    keep[0, 0] = False  # an empty row
    keep[1, 1] = True
    o = R.block_sparse_attention(qa.to(dev), ka.to(dev), va.to(dev), keep.to(dev))
    out["attention"] = {"q": qa, "k": ka, "v": va, "keep": keep, "out": o.cpu()}
    # a3: FP8Linear._mm = torch._scaled_mm (cuBLASLt) on the GPU, per-tensor scales
    lin = torch.nn.Linear(1536, 256).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(0.02 * torch.randn(256, 1536, generator=_gen(13)))
        lin.bias.copy_(0.02 * torch.randn(256, generator=_gen(14)))
    fl = R.FP8Linear(lin.to(dev))
    xa = _outliers(128, 1536, _gen(15))
    x8, s = R.quantize_fp8(xa.to(dev))
    y = fl._mm(x8, s)
    out["scaled_mm"] = {"x": xa, "w": lin.weight.detach().cpu(), "b": lin.bias.detach().cpu(),
                        "w8": fl.weight.detach().view(torch.uint8).cpu(),
                        "w_scale": fl.w_scale.detach().cpu(), "x8": x8.view(torch.uint8).cpu(),
                        "x_scale": s.cpu(), "y": y.cpu()}
    return out


def _time(fn, dev, reps=20, rounds=5):
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    ts = []
    for _ in range(rounds):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        torch.cuda.synchronize(dev)
        ts.append(e0.elapsed_time(e1) / reps)
    return statistics.median(ts)


def timing(R, dev):
    """Reference GPU ops vs this pack's at the benchmark step's shapes (8448 tokens)."""
    from flashvsr_sm89_ops_b200 import fused_gate_add, fused_ln_modulate, fused_rms_rope, lcsa
    from flashvsr_sm89_ops_b200 import quantize_fp8 as b_quant
    from flashvsr_sm89_ops_b200.fp8_ffn import ffn_fp8
    from flashvsr_sm89_ops_b200.fp8_linear import FP8Linear as BLinear
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm
    L, D, FF, H = 8448, 1536, 8960, 12
    gd = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *s: torch.randn(*s, generator=gd, device=dev).to(torch.bfloat16)  # noqa: E731
    rows = []

    def add(op, shape, ref_fn, b200_fn, note=""):
        tr, tb = _time(ref_fn, dev), _time(b200_fn, dev)
        rows.append({"op": op, "shape": shape, "reference_ms": tr, "b200_ms": tb,
                     "speedup": tr / tb, "note": note})

    x = rnd(L, D)
    add("quantize_fp8 (per tensor)", f"[{L},{D}]", lambda: R.quantize_fp8(x),
        lambda: b_quant(x, "tensor"))
    add("quantize_fp8 (reference per tensor vs pack per token)", f"[{L},{D}]",
        lambda: R.quantize_fp8(x), lambda: b_quant(x, "token"), "the pack's benchmark mode")
    hdn = rnd(L, FF)
    from flashvsr_sm89_ops_b200 import _lib
    amax = hdn.float().abs().amax(dim=1).contiguous()
    q8 = torch.empty(L, FF, dtype=torch.float8_e4m3fn, device=dev)
    s8 = torch.empty(L, device=dev)
    add("GELU->FP8 mid-section of the FFN", f"[{L},{FF}]", lambda: R.fused_gelu_quant_fp8(hdn),
        lambda: _lib.call("fvb_quant_fp8_with_amax", _lib.ptr(hdn), L, FF, _lib.ptr(amax),
                          _lib.FVB_SCALE_ROW, _lib.ptr(q8), _lib.ptr(s8), _lib.stream_of(hdn)),
        "reference: 2 passes (GELU+amax, GELU+quant); pack: GELU and amax are in the GEMM-1 "
        "epilogue, this is the one remaining pass")
    from flashvsr_sm89_ops_b200.fp8_quant import fused_gelu_quant_fp8 as b_gelu_quant
    add("fused_gelu_quant_fp8 (standalone, per tensor)", f"[{L},{FF}]",
        lambda: R.fused_gelu_quant_fp8(hdn), lambda: b_gelu_quant(hdn, "tensor"),
        "both sides apply GELU, reduce the amax and quantise")
    add("fused_gelu_quant_fp8 (standalone, pack per token)", f"[{L},{FF}]",
        lambda: R.fused_gelu_quant_fp8(hdn), lambda: b_gelu_quant(hdn, "token"),
        "the reference per tensor")
    w = (1 + 0.1 * torch.randn(D, generator=gd, device=dev)).to(torch.bfloat16)
    fr = _freqs(L, 3).to(dev)
    x3 = x.view(1, L, D)
    add("fused_rms_rope", f"[1,{L},{D}]", lambda: R.fused_rms_rope(x3, w, fr),
        lambda: fused_rms_rope(x3, w, fr))
    sc, sh, gt = rnd(1, 1, D), rnd(1, 1, D), rnd(1, 1, D)
    add("fused_ln_modulate", f"[1,{L},{D}]", lambda: R.fused_ln_modulate(x3, sc, sh),
        lambda: fused_ln_modulate(x3, sc, sh))
    r3 = rnd(1, L, D)
    add("fused_gate_add", f"[1,{L},{D}]", lambda: R.fused_gate_add(x3, gt, r3),
        lambda: fused_gate_add(x3, gt, r3))
    for K, N in ((1536, 1536), (1536, 4608), (1536, 8960), (8960, 1536)):
        lin = torch.nn.Linear(K, N).to(torch.bfloat16).to(dev)
        rl, bl = R.FP8Linear(lin), BLinear(lin, "tensor")
        xk = rnd(L, K)
        rx8, rs = R.quantize_fp8(xk)
        bx8, bs = b_quant(xk, "tensor")
        add(f"FP8 GEMM {K}->{N} (per tensor)", f"M={L}", lambda: rl._mm(rx8, rs),
            lambda: fp8_mm(bx8, bs, bl.weight, bl.w_scale, bl.bias),
            "reference: torch._scaled_mm (cuBLASLt)")
    l0 = torch.nn.Linear(D, FF).to(torch.bfloat16).to(dev)
    l2 = torch.nn.Linear(FF, D).to(torch.bfloat16).to(dev)
    rffn = R.FP8FFN(R.FP8Linear(l0), R.FP8Linear(l2))
    b0, b2 = BLinear(l0, "tensor"), BLinear(l2, "tensor")
    x3c = x3.contiguous()
    add("FP8FFN.forward", f"[1,{L},{D}]", lambda: rffn(x3c),
        lambda: ffn_fp8(*b_quant(x, "tensor"), b0, b2), "whole FFN incl. input quantisation")
    per_row = 66
    q, k, v = rnd(1, L, D), rnd(1, 4 * per_row * 128, D), rnd(1, 4 * per_row * 128, D)
    keep = lcsa.causal_topk_mask(q.view(-1, 128, D), k.view(-1, 128, D), H, per_row, 0.25)
    sel, cnt, _ = lcsa.build_csr(keep)
    out = torch.empty_like(q[0])
    add("block_sparse_attention (Triton LCSA, incl. build_csr)", "66 x 264 windows, 91,080 pairs",
        lambda: R.block_sparse_attention(q, k, v, keep),
        lambda: lcsa.block_sparse_attention(q, k, v, keep),
        "both calls include their mask -> CSR step (the reference's has a host sync)")
    rsel, rcnt, rmaxk = R.lcsa_build_csr(keep)

    def ref_kernel():
        o = torch.empty_like(q)
        R.bsa_kernel[(H * per_row,)](q, k, v, o, rsel, rcnt, 1.0 / math.sqrt(128), per_row, rmaxk,
                                    NUM_HEADS=H, D=128, BLOCK_S=128, num_warps=8, num_stages=2)
    add("block-sparse attention kernel only", "66 x 264 windows, 91,080 pairs", ref_kernel,
        lambda: lcsa.attention_csr(q[0], k[0], v[0], sel, cnt, H, out=out))
    return rows


def load_reference(path):
    sys.path.insert(0, os.path.abspath(path))
    import flashvsr_sm89_ops as R
    from flashvsr_sm89_ops.fp8_ffn import fused_gelu_quant_fp8
    from flashvsr_sm89_ops.lcsa.triton_lcsa import _bsa_fwd_kernel, block_sparse_attention, build_csr
    R.fused_gelu_quant_fp8 = fused_gelu_quant_fp8
    R.block_sparse_attention = block_sparse_attention
    R.lcsa_build_csr = build_csr
    R.bsa_kernel = _bsa_fwd_kernel
    return R


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FVB_REFERENCE", ""))
    ap.add_argument("--out", default=os.path.join(ROOT, "tests", "golden", "triton_b200.pt"))
    ap.add_argument("--timing", default="")
    a = ap.parse_args()
    if not a.reference:
        raise SystemExit("give --reference <dir holding flashvsr_sm89_ops> (or FVB_REFERENCE)")
    sys.path.insert(0, ROOT)
    R = load_reference(a.reference)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    import triton
    fx = make_fixtures(R, dev)
    fx["_meta"] = {"gpu": torch.cuda.get_device_name(dev), "torch": torch.__version__,
                   "triton": triton.__version__, "cap": list(torch.cuda.get_device_capability(dev))}
    torch.save(fx, a.out)
    print(f"wrote {a.out}: {sorted(k for k in fx if not k.startswith('_'))}", flush=True)
    if a.timing:
        rows = timing(R, dev)
        with open(a.timing, "w") as f:
            json.dump({"meta": fx["_meta"], "rows": rows}, f, indent=1)
        for r in rows:
            print(f"{r['op']:58s} ref {r['reference_ms'] * 1e3:9.1f} us  b200 {r['b200_ms'] * 1e3:9.1f} us"
                  f"  x{r['speedup']:.2f}", flush=True)


if __name__ == "__main__":
    main()
