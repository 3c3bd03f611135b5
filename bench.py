#!/usr/bin/env python3
"""Benchmark of the FlashVSR B200 operator pack (one JSON line on rank 0).

Metric: DiT tokens/s @1408x768 on B200.  A step is one steady-
state FlashVSR streaming chunk through the 30-block FlashVSR-Tiny-shaped DiT
(dim 1536, 12 heads x 128, FFN 8960; f=2 latent frames x 48 x 88 = 8448 tokens
= 8 output frames; KV cache of 3 time rows, so attention sees 264 key windows;
keep rule: own time row + top 25% of past windows by mean-pooled q.k), every op
on this pack's sm_100a kernels, the step replayed as one CUDA graph.  Random-init
weights (N(0, 0.02)), synthetic N(0,1) inputs.

  python bench.py [--gpus N --steps K --warmup W]          # this pack
  python bench.py --impl reference [...]                    # the reference path on CPU

With N > 1 (torchrun) every rank renders its own tile stream of the same shape
(tiles are independent; "scaling": "weak") and value = all tokens / max-over-
ranks time.  The reference arm times the reference's torch-eager formulas (the
CPU oracle restated from the reference, since the reference's own kernels are
Triton and need a GPU) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

H_PX, W_PX = 768, 1408
BLOCKS = 30
D, HEADS, FFN = 1536, 12, 8960
CTX = 512
KV_LEN = 3
RATIO = 0.25
METRIC = "DiT tokens/s @1408x768 (30-block FlashVSR-Tiny DiT, streaming f=2 step)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--blocks", type=int, default=BLOCKS)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--only", default=None,
                   help="time kernels of the step in isolation at the step's shape "
                        "(profiling / per-kernel roofline): one name of ONLY_KERNELS or a "
                        "comma-separated list; prints one JSON line per kernel")
    p.add_argument("--graph", action="store_true",
                   help="with --only: capture the timed calls in one CUDA graph and time its "
                        "replay, so host-side call overhead is not in the per-launch time")
    a = p.parse_args()
    if a.only is not None:
        bad = [k for k in a.only.split(",") if k not in ONLY_KERNELS]
        if bad:
            p.error(f"--only: unknown kernel(s) {bad}; choose from {sorted(ONLY_KERNELS)}")
    return a


# kernels of one block at the step's shape, runnable in isolation (--only)
ONLY_KERNELS = ("attention", "cross_attention", "gemm_qkv", "gemm_o", "gemm_up", "gemm_up_gelu",
                "gemm_down",
                "ffn", "gelu_quant_hidden", "quant_hidden", "quant_token", "ln_mod_fp8", "gate_add_ln_mod_fp8",
                "gate_add_norm3_fp8", "rms_rope", "gate_add", "pool", "window", "causal_mask",
                "mask_csr", "cublaslt_qkv", "cublaslt_o", "cublaslt_up", "cublaslt_down")
L2_BYTES = 126 << 20


def run_only(args, local_rank):
    """Run each kernel named by --only (comma-separated) in turn, in this process."""
    import copy
    for name in args.only.split(","):
        one = copy.copy(args)
        one.only = name
        _run_only_one(one, local_rank)


def _time_graph(fn, steps, dev):
    """Per-launch ms of `steps` calls of fn captured in one CUDA graph, replayed once to warm
    and once timed with CUDA events on the launching stream."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            fn()
    graph.replay()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    del graph
    return ms


def _run_only_one(args, local_rank):
    """Run one kernel class K times at the workload's shapes; report time and roofline.

    Memory-bound kernels cycle through enough independent input sets to cover three times
    the L2, so every call reads its operands from HBM as in the step."""
    from flashvsr_sm89_ops_b200 import _lib, fused_gate_add, fused_ln_modulate, lcsa, quantize_fp8
    from flashvsr_sm89_ops_b200.fp8_linear import fp8_mm
    from flashvsr_sm89_ops_b200.fused_adaln import gate_add_layer_norm, gate_add_ln_modulate
    from flashvsr_sm89_ops_b200.fused_rms_rope import rms_rope_rows
    from flashvsr_sm89_ops_b200.fp8_ffn import ffn_fp8
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    lat_h, lat_w = H_PX // 16, W_PX // 16
    L = 2 * lat_h * lat_w
    per_row = (lat_h // 8) * (lat_w // 8)
    peaks, kind = load_peaks()
    rnd = lambda *s: torch.randn(*s, generator=g, device=dev).to(torch.bfloat16)  # noqa: E731
    st = _lib.stream_of(rnd(1))

    def wq(n, k):
        from flashvsr_sm89_ops_b200.fp8_linear import quantize_weight
        return quantize_weight(0.02 * torch.randn(n, k, generator=g, device=dev).to(torch.bfloat16), "token")

    def rotating(make, set_bytes):
        """Callable cycling over independent input sets (3x L2 in total) built by make()."""
        n = max(1, min(16, -(-3 * L2_BYTES // max(set_bytes, 1))))
        fns = [make() for _ in range(n)]
        i = [0]

        def fn():
            fns[i[0] % n]()
            i[0] += 1
        return fn

    x8, sx = quantize_fp8(rnd(L, D), "token")
    work, bound = None, "hbm"
    k_rows = (KV_LEN + 1) * per_row * 128
    if args.only == "attention":
        q, k, v = rnd(L, D), rnd(k_rows, D), rnd(k_rows, D)
        keep = lcsa.causal_topk_mask(q, k, HEADS, per_row, RATIO)
        sel, cnt, _ = lcsa.build_csr(keep)
        out = torch.empty_like(q)
        fn = lambda: lcsa.attention_csr(q, k, v, sel, cnt, HEADS, out=out)  # noqa: E731
        work, bound = int(keep.sum().item()) * 4 * 128 ** 3, "tensor"
    elif args.only == "cross_attention":
        q, k, v = rnd(L, D), rnd(CTX, D), rnd(CTX, D)
        out = torch.empty_like(q)
        fn = lambda: lcsa.dense_attention(q, k, v, HEADS, out=out)  # noqa: E731
        work, bound = L * CTX * 4 * D, "tensor"
    elif args.only in ("gemm_qkv", "gemm_o", "gemm_up", "gemm_down"):
        n, kk = {"gemm_qkv": (3 * D, D), "gemm_o": (D, D), "gemm_up": (FFN, D),
                 "gemm_down": (D, FFN)}[args.only]
        a8, sa = (x8, sx) if kk == D else quantize_fp8(rnd(L, kk), "token")
        w8, sw = wq(n, kk)
        b = rnd(n)
        out = torch.empty(L, n, dtype=torch.bfloat16, device=dev)
        fn = lambda: fp8_mm(a8, sa, w8, sw, b, out=out)  # noqa: E731
        work, bound = 2 * L * n * kk, "tensor"
    elif args.only.startswith("cublaslt_"):
        # the reference's own GEMM path on this box: torch._scaled_mm (cuBLASLt) with the
        # per-tensor scales of its FP8Linear, bias in the call, bf16 out, same shapes
        n, kk = {"cublaslt_qkv": (3 * D, D), "cublaslt_o": (D, D), "cublaslt_up": (FFN, D),
                 "cublaslt_down": (D, FFN)}[args.only]
        a8 = torch.randn(L, kk, generator=g, device=dev).to(torch.float8_e4m3fn)
        w8 = (torch.randn(n, kk, generator=g, device=dev) * 0.02).to(torch.float8_e4m3fn)
        one = torch.ones((), device=dev)
        b = rnd(n)
        fn = lambda: torch._scaled_mm(a8, w8.t(), scale_a=one, scale_b=one, bias=b,  # noqa: E731
                                      out_dtype=torch.bfloat16)
        work, bound = 2 * L * n * kk, "tensor"
    elif args.only == "gemm_up_gelu":
        w8, sw = wq(FFN, D)
        b = rnd(FFN)
        h = torch.empty(L, FFN, dtype=torch.bfloat16, device=dev)
        amax = torch.zeros(L, device=dev)
        fn = lambda: fp8_mm(x8, sx, w8, sw, b, out=h, epilogue=_lib.FVB_EPI_GELU_AMAX,  # noqa: E731
                            amax_out=amax)
        work, bound = 2 * L * FFN * D, "tensor"
    elif args.only == "ffn":
        from flashvsr_sm89_ops_b200.fp8_linear import FP8Linear
        l0 = torch.nn.Linear(D, FFN).to(torch.bfloat16).to(dev)
        l2 = torch.nn.Linear(FFN, D).to(torch.bfloat16).to(dev)
        f0, f2 = FP8Linear(l0, "token"), FP8Linear(l2, "token")
        res, gate = rnd(1, L, D), rnd(1, 1, D)
        out = torch.empty(L, D, dtype=torch.bfloat16, device=dev)
        ws = torch.empty(2 * L * FFN * 3, dtype=torch.uint8, device=dev)
        # the block's call: FFN with the closing gated residual add in its epilogue
        fn = lambda: ffn_fp8(x8, sx, f0, f2, out=out, workspace=ws, residual=res, gate=gate)  # noqa: E731
        work, bound = 4 * L * D * FFN, "tensor"
    elif args.only == "gelu_quant_hidden":
        from flashvsr_sm89_ops_b200.fp8_quant import fused_gelu_quant_fp8

        def make():
            h = rnd(L, FFN)
            return lambda: fused_gelu_quant_fp8(h, "token")
        work = L * FFN * 3 + L * 4
        fn = rotating(make, work)
    elif args.only == "quant_hidden":
        def make():
            h = rnd(L, FFN)
            amax = h.float().abs().amax(dim=1).contiguous()
            q = torch.empty(L, FFN, dtype=torch.float8_e4m3fn, device=dev)
            sc = torch.empty(L, device=dev)
            return lambda: _lib.call("fvb_quant_fp8_with_amax", _lib.ptr(h), L, FFN, _lib.ptr(amax),
                                     _lib.FVB_SCALE_ROW, _lib.ptr(q), _lib.ptr(sc),
                                     _lib.stream_of(h))
        work = L * FFN * 3 + L * 8
        fn = rotating(make, work)
    elif args.only == "quant_token":
        def make():
            xx = rnd(L, D)
            return lambda: quantize_fp8(xx, "token")
        work = L * D * 3 + L * 4
        fn = rotating(make, work)
    elif args.only == "ln_mod_fp8":
        sc, sh = rnd(1, 1, D), rnd(1, 1, D)

        def make():
            x3 = rnd(1, L, D)
            return lambda: fused_ln_modulate(x3, sc, sh, emit_fp8=True, want_out=False)
        work = L * D * (2 + 1) + L * 4
        fn = rotating(make, work)
    elif args.only == "gate_add_ln_mod_fp8":
        sc, sh = rnd(1, 1, D), rnd(1, 1, D)

        def make():
            x3, r3 = rnd(1, L, D), rnd(1, L, D)
            return lambda: gate_add_ln_modulate(x3, None, r3, sc, sh, emit_fp8=True, want_out=False)
        work = L * D * 7 + L * 4
        fn = rotating(make, work)
    elif args.only == "gate_add_norm3_fp8":
        gt, w, b = rnd(1, 1, D), rnd(D), rnd(D)

        def make():
            x3, r3 = rnd(1, L, D), rnd(1, L, D)
            return lambda: gate_add_layer_norm(x3, gt, r3, w, b, emit_fp8=True, want_out=False)
        work = L * D * 7 + L * 4
        fn = rotating(make, work)
    elif args.only == "rms_rope":
        cos = torch.rand(L, 64, generator=g, device=dev)
        sin = torch.rand(L, 64, generator=g, device=dev)
        w = rnd(D)

        def make():
            xx, out = rnd(L, D), torch.empty(L, D, dtype=torch.bfloat16, device=dev)
            return lambda: rms_rope_rows(xx, w, cos, sin, L, 1e-6, True, 128, out=out)
        work = L * D * 4 + L * 64 * 8
        fn = rotating(make, work)
    elif args.only == "gate_add":
        gt = rnd(1, 1, D)

        def make():
            x3, r3 = rnd(1, L, D), rnd(1, L, D)
            out = torch.empty_like(x3)
            return lambda: fused_gate_add(x3, gt, r3, out=out)
        work = L * D * 6
        fn = rotating(make, work)
    elif args.only == "pool":
        def make():
            xw = rnd(L // 128, 128, D)
            out = torch.empty(L // 128, D, dtype=torch.float32, device=dev)
            return lambda: lcsa.block_mean_pool(xw, out=out)
        work = L * D * 2 + (L // 128) * D * 4
        fn = rotating(make, work)
    elif args.only == "window":
        def make():
            xx = rnd(L, D)
            out = torch.empty(L // 128, 128, D, dtype=torch.bfloat16, device=dev)
            return lambda: lcsa.window_partition(xx, (2, lat_h, lat_w), out=out)
        work = L * D * 4
        fn = rotating(make, work)
    elif args.only == "causal_mask":
        q, k = rnd(L, D), rnd(k_rows, D)
        fn = lambda: lcsa.causal_topk_mask(q, k, HEADS, per_row, RATIO)  # noqa: E731
        work = (L + k.shape[0]) * D * 2
    elif args.only == "mask_csr":
        keep = torch.rand(HEADS, L // 128, k_rows // 128, generator=g, device=dev) < 0.4
        fn = lambda: lcsa.build_csr(keep)  # noqa: E731
        work = keep.numel() * (1 + 4) + HEADS * (L // 128) * 4  # mask in, sel + cnt out
    for _ in range(max(args.warmup, 1)):
        fn()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("fvb_only")
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    ms_eager = ms
    if args.graph:
        ms = _time_graph(fn, args.steps, dev)
    fp8 = args.only in ("gemm_qkv", "gemm_o", "gemm_up", "gemm_up_gelu", "gemm_down", "ffn") or \
        args.only.startswith("cublaslt_")
    if bound == "tensor" and fp8:
        ach, peak, unit = work / (ms / 1e3) / 1e12, measure_fp8_peak(dev), "TFLOP/s"
        kind = "measured here: cuBLASLt FP8 8192^3 best-of-10"
    elif bound == "tensor":
        ach, peak, unit = work / (ms / 1e3) / 1e12, float(peaks.get("bf16_tflops", 1590.0)), "TFLOP/s"
    else:
        ach, peak, unit = work / (ms / 1e3) / 1e9, float(peaks.get("hbm_gbs", 6650.0)), "GB/s"
    print(json.dumps({"only": args.only, "ms_per_launch": ms, "work_per_launch": work, "bound": bound,
                      "achieved": ach, "peak": peak, "unit": unit, "frac": ach / peak,
                      "peak_kind": kind, "timing": "cuda_graph" if args.graph else "eager",
                      "ms_per_launch_eager": ms_eager}))


def measure_fp8_peak(dev):
    """Dense FP8 denominator: cuBLASLt torch._scaled_mm at 8192^3, best of 10 (TFLOP/s).
    MEASURED_PEAKS.json holds bf16 only; this is the same style of measurement for FP8."""
    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones(1, device=dev)
    best = 1e9
    for _ in range(12):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1))
    return 2 * n ** 3 / (best / 1e3) / 1e12


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def config(args, world):
    lat_h, lat_w = H_PX // 16, W_PX // 16
    return {
        "workload": "dit30_1408x768_stream_f2",
        "tokens_per_step": 2 * lat_h * lat_w,
        "frames_per_step": 8,
        "blocks": args.blocks,
        "dim": D, "heads": HEADS, "ffn": FFN, "context_tokens": CTX,
        "kv_cache_rows": KV_LEN, "query_windows": lat_h // 8 * (lat_w // 8),
        "key_windows": (KV_LEN + 1) * (lat_h // 8) * (lat_w // 8),
        "keep_rule": f"own time row + top {int(RATIO * 100)}% past windows (mean-pooled q.k)",
        "fp8_scales": "per-token activations x per-channel weights",
        "parallelism": f"tile-replica x{world}",
        "global_batch": world,
        "seq_len": 2 * lat_h * lat_w,
        "l2_policy": "inputs larger than L2: 1.39 GB of FP8 weights stream through each step",
        "cuda_graph": not args.no_graph,
    }


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        loaded = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_block_sample(steps=1, warm=True):
    """Reference formulas on the host: one DiT block at the step's exact shape.

    Returns (seconds per block, threads)."""
    from oracle import ops as O
    from oracle import wan
    wan.ATTENTION = "reference"  # the reference's own fp32 attention formula
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    lat_h, lat_w = H_PX // 16, W_PX // 16
    P = wan.init_block_params(g, D, FFN)
    Q = wan.quantize_block(P, "token")
    L = 2 * lat_h * lat_w
    x = torch.randn(1, L, D, generator=g).to(torch.bfloat16)
    t_mod = torch.randn(1, 6, D, generator=g).to(torch.bfloat16)
    ctx = torch.randn(1, CTX, D, generator=g).to(torch.bfloat16)
    kv = wan.cross_kv(Q, ctx)
    per_row = (lat_h // 8) * (lat_w // 8)
    cache = (torch.randn(KV_LEN * per_row, 128, D, generator=g).to(torch.bfloat16),
             torch.randn(KV_LEN * per_row, 128, D, generator=g).to(torch.bfloat16))
    cos, sin = O.freqs_cos_sin(wan.grid_freqs(2, lat_h, lat_w, f0=6))
    mask_fn = wan.causal_mask_fn(HEADS, per_row, RATIO)
    run = lambda: wan.block_forward(Q, x, t_mod, cos, sin, (2, lat_h, lat_w), kv, mask_fn,  # noqa: E731
                                    HEADS, cache, KV_LEN)
    if warm:
        run()
    t0 = time.perf_counter()
    for _ in range(steps):
        run()
    return (time.perf_counter() - t0) / steps, torch.get_num_threads()


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, world, rank):
    if rank != 0:
        return
    cfg = config(args, world)
    tokens = cfg["tokens_per_step"]
    for _ in range(max(args.warmup, 0) and 1):
        cpu_block_sample(steps=1, warm=False)
    times = []
    budget = 240.0
    t_start = time.perf_counter()
    for i in range(args.steps):
        t, threads = cpu_block_sample(steps=1, warm=False)
        times.append(t)
        if time.perf_counter() - t_start > budget:
            break
    per_block = statistics.mean(times)
    step_s = per_block * args.blocks
    value = tokens / step_s
    sample = (f"each timed step is a bounded sample of the workload: one DiT block forward of "
              f"the step shape ({tokens} tokens, 264 key windows) of the {args.blocks}; value "
              f"scales the mean block time by {args.blocks}; torch-eager reference formulas on "
              f"{cpu_model()}")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        # steps x ms_per_step is the wall time of the timed samples; the full 30-block step
        # this value describes takes ms_per_full_step (extrapolated from the samples)
        "steps": len(times), "warmup": args.warmup, "ms_per_step": per_block * 1e3,
        "ms_per_full_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (fp8 fake-quant linears)", "data": "synthetic", "config": cfg,
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- B200 arm
def tiled_4k(runner, world, rank, dev, dist_mod):
    """4K tiled frames/s: the 3840x2048 canvas in 24 tiles of 896x768 (the survey's scaling
    plan, plan_tiles(target=threshold=700_000)), tile i on rank i % world, each tile through
    the DiT streaming schedule (one f=6 chunk + seven f=2 chunks = 20 latent frames -> 80
    output frames) by TiledDiTPipe, blended on the rank's GPU and reduced to rank 0 by the
    pack's own render_tiled.  Strong scaling: the canvas is fixed, ranks split the tiles.
    The LQ video (85 frames) lives in pinned host memory and each tile's crop is copied in,
    as the reference's render_tiled does.  Timed on the device (events around the whole
    render, max over ranks) after a one-tile warm-up that also makes the one-time allocations
    (pinned crop staging, the canvas block)."""
    from flashvsr_sm89_ops_b200.runner import TiledDiTPipe
    from flashvsr_sm89_ops_b200.tiling import plan_tiles, render_tiled, reserve_staging
    W4, H4 = 3840, 2048
    pipe = TiledDiTPipe(runner)
    frames_in = 4 * pipe.latent_frames() + 5  # 85
    g = torch.Generator(device=dev).manual_seed(13)
    lq = torch.empty((3, frames_in, H4, W4), dtype=torch.bfloat16, pin_memory=True)
    for fi in range(frames_in):  # per frame, to keep the device staging buffer small
        lq[:, fi].copy_((torch.rand(3, H4, W4, generator=g, device=dev) * 2 - 1).to(torch.bfloat16))
    tiles = plan_tiles(W4, H4, target=700_000, threshold=700_000)
    x, y, w, h = tiles[0]
    warm = pipe(LQ_video=lq[:, :, y:y + h, x:x + w].to(dev), num_frames=frames_in, height=h, width=w)
    pipe.tokens = 0
    # warm-up of the one-time allocations outside the timed region: this rank's pinned crop
    # staging (kept by render_tiled across calls) and the caching allocator's block for the
    # fp32 canvas
    reserve_staging(lq, tile_target=700_000, tile_threshold=700_000, device=dev)
    del warm
    canvas_warm = torch.empty((3, 4 * pipe.latent_frames(), H4, W4), dtype=torch.float32, device=dev)
    del canvas_warm
    torch.cuda.synchronize(dev)
    if world > 1:
        dist_mod.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    tm = {}
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    e0.record(stream)
    out = render_tiled(pipe, lq, tile_target=700_000, tile_threshold=700_000, device=dev,
                       timings=tm)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ev = tm["events"]
    # this rank's split: its tiles (render + blend), the cross-rank reduce, crop-packing waits
    part = torch.tensor([ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), tm["load_wait_s"] * 1e3,
                         float(tm["tiles"])], device=dev, dtype=torch.float64)
    t = torch.tensor([e0.elapsed_time(e1), float(pipe.tokens)], device=dev, dtype=torch.float64)
    parts = [part]
    if world > 1:
        tok = t[1:2].clone()
        dist_mod.all_reduce(t[0:1], op=dist_mod.ReduceOp.MAX)
        dist_mod.all_reduce(tok, op=dist_mod.ReduceOp.SUM)
        t[1] = tok[0]
        parts = [torch.empty_like(part) for _ in range(world)]
        dist_mod.all_gather(parts, part)
    ms, tokens = float(t[0].item()), float(t[1].item())
    # the same canvas on one GPU in the same job (rank 0 alone, the others wait): the
    # single-GPU time the strong-scaling efficiency is measured against
    solo = None
    if world > 1 and os.environ.get("FVB_SKIP_TILED_N1") != "1":
        g0 = dist_mod.new_group([0])
        if rank == 0:
            pipe.tokens = 0
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            solo_sampler = ClockSampler(dev.index if dev.index is not None else 0)
            solo_sampler.start()
            s0.record(stream)
            ref = render_tiled(pipe, lq, tile_target=700_000, tile_threshold=700_000, device=dev,
                               group=g0)
            s1.record(stream)
            torch.cuda.synchronize(dev)
            solo = {"ms": s0.elapsed_time(s1), "clocks": solo_sampler.stop(),
                    "max_abs_diff_vs_sharded": float((ref.float() - out.float()).abs().max().item())}
            del ref
        dist_mod.barrier()
    if rank != 0:
        return None
    n_out = int(out.shape[1])
    per_rank = [[float(v) for v in p.tolist()] for p in parts]
    breakdown = {
        "per_rank_tiles_ms": [round(p[0], 1) for p in per_rank],
        "per_rank_reduce_ms": [round(p[1], 1) for p in per_rank],
        "per_rank_crop_wait_ms": [round(p[2], 1) for p in per_rank],
        "per_rank_tiles": [int(p[3]) for p in per_rank],
        "canvas_reduce_bytes": int(out.numel()) * 4,
    }
    extra = {}
    if solo is not None:
        extra = {"n1_same_job_ms": solo["ms"], "n1_same_job_fps": n_out / (solo["ms"] / 1e3),
                 "n1_same_job_clocks_rank0": solo["clocks"],
                 "efficiency_vs_n1_same_job": solo["ms"] / (world * ms),
                 "n1_max_abs_diff_vs_sharded": solo["max_abs_diff_vs_sharded"]}
    return {
        "fps": n_out / (ms / 1e3), "unit": "frames/s", "frames": n_out, "ms": ms,
        "canvas": f"{W4}x{H4}", "input_frames": frames_in, "tiles": len(tiles),
        "tile": f"{w}x{h}", "tiles_per_rank": -(-len(tiles) // world),
        "dit_tokens_per_s": tokens / (ms / 1e3), "scaling": "strong",
        "checksum": float(out.float().abs().sum().item()),
        "schedule": "per tile: f=6 chunk + 7 f=2 chunks (KV cache of 3 time rows), 30 blocks; "
                    "patch-embed / unpatchify are bf16 linears standing in for the LQ "
                    "projection and VAE",
        "breakdown": breakdown, "clocks_rank0": clocks, **extra,
    }


def attention_roofline(runner, iters, stream):
    """Time the dominant kernel (block-sparse attention at the step's shape) with CUDA events."""
    from flashvsr_sm89_ops_b200 import lcsa
    dev = runner.device
    g = torch.Generator(device=dev).manual_seed(11)
    per_row = runner.h // 8 * (runner.w // 8)
    nq, nk = per_row, (KV_LEN + 1) * per_row
    q = torch.randn(nq * 128, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(nk * 128, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(nk * 128, D, generator=g, device=dev).to(torch.bfloat16)
    keep = lcsa.causal_topk_mask(q, k, HEADS, per_row, RATIO)
    sel, cnt, _ = lcsa.build_csr(keep)
    pairs = int(keep.sum().item())
    out = torch.empty_like(q)
    for _ in range(3):
        lcsa.attention_csr(q, k, v, sel, cnt, HEADS, out=out)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        lcsa.attention_csr(q, k, v, sel, cnt, HEADS, out=out)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / iters
    flops = pairs * 4 * 128 * 128 * 128
    return ms, flops, pairs


def traffic_from_profiles(kernel):
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            d = json.load(f)
        return d.get(kernel, {}).get("bytes_per_launch")
    except Exception:
        return None


def run_b200(args, world, rank, local_rank):
    import torch.distributed as dist
    from flashvsr_sm89_ops_b200 import _lib
    from flashvsr_sm89_ops_b200.runner import HostStream, StreamingDiT

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    runner = StreamingDiT(num_layers=args.blocks, dim=D, heads=HEADS, ffn=FFN, height=H_PX,
                          width=W_PX, ctx_len=CTX, kv_len=KV_LEN, mask_rule="causal",
                          seed=0, device=dev)  # one model, replicated on every rank
    runner.prime()
    tokens = runner.tokens(2)
    x_static = runner.make_input(2)
    stream = torch.cuda.current_stream(dev)

    # launches of this pack's kernels per step (counted on one eager step)
    _lib.start_launch_count()
    runner.step(x_static)
    launches = _lib.stop_launch_count()
    torch.cuda.synchronize(dev)

    if args.no_graph:
        step = lambda: runner.step(x_static)  # noqa: E731
        y = runner.step(x_static)
    else:
        graph, y = runner.capture(x_static)
        step = graph.replay
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("fvb_timed")
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * tokens * args.steps / (ms_max / 1e3)

    # end to end through the public API: pinned host input -> step -> pinned host output for
    # every step, the transfers overlapped with the neighbouring steps' compute (HostStream)
    x_host = torch.empty(x_static.shape, dtype=x_static.dtype, pin_memory=True)
    x_host.copy_(x_static.cpu())
    y_hosts = [torch.empty(y.shape, dtype=y.dtype, pin_memory=True) for _ in range(2)]
    hs = HostStream(step, x_static, y)
    hs.run([x_host] * 2, y_hosts)
    torch.cuda.synchronize(dev)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    hs.run([x_host] * args.steps, [y_hosts[i & 1] for i in range(args.steps)])
    e3.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    t2 = torch.tensor([e2.elapsed_time(e3)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e = world * tokens * args.steps / (float(t2.item()) / 1e3)

    # roofline of the dominant kernel, timed live with CUDA events on the launching stream
    att_ms, att_flops, pairs = attention_roofline(runner, max(args.steps, 10), stream)
    peaks, peak_kind = load_peaks()
    achieved = att_flops / (att_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tiled = None
    if os.environ.get("FVB_SKIP_TILED") != "1":
        import torch.distributed as dist_mod
        try:  # the secondary 4K workload must not cost the step's line
            tiled = tiled_4k(runner, world, rank, dev, dist_mod)
        except Exception as e:  # noqa: BLE001
            tiled = {"error": f"{type(e).__name__}: {e}"[:300]}
            print(f"tiled_4k failed: {tiled['error']}", file=sys.stderr, flush=True)
    devs = _lib.device_error()
    if devs:
        raise RuntimeError(f"device error word set: {devs:#x}")

    if rank != 0:
        return
    cfg = config(args, world)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8_e4m3 GEMMs + bf16 attention/norms", "data": "synthetic (random-init weights, N(0,1) inputs)",
        "config": cfg,
        "fps": world * 8 * args.steps / (ms_max / 1e3),
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": x_static.numel() * 2,
                "d2h_bytes_per_step": y.numel() * 2},
        "gpu_launches": launches * args.steps,
        "roofline": {"kernel": "bsa6::bsa_fwd_v6_kernel (block-sparse self-attention, 91,080 kept "
                               "window pairs)",
                     "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_kind": f"{peak_kind} bf16 dense (burst)",
                     "traffic": traffic_from_profiles("bsa_fwd_kernel"),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this "
                                       "kernel at this shape, from the committed capture "
                                       "profiles/traffic.json (not re-measured in this run)",
                     "launch_ms": att_ms, "flops_per_launch": att_flops},
        "clocks": clocks,
    }
    if tiled is not None:
        line["tiled_4k"] = tiled
    if world == 1 and os.environ.get("FVB_SKIP_CPU_BASELINE") != "1":
        t_block, threads = cpu_block_sample(steps=1, warm=False)
        cpu_value = tokens / (t_block * args.blocks)
        line["cpu_baseline"] = {
            "value": cpu_value, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"1 DiT block forward of the step shape on the host ({cpu_model()}), "
                      f"scaled to {args.blocks} blocks"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)  # rank 0 only; other ranks exit without work
        return
    if args.only:
        run_only(args, local_rank)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        # NCCL prints its version on stdout at init; keep stdout for the one JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    try:
        run_b200(args, world, rank, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
