"""Generate golden fixtures by running the reference itself (build container only).

    python tests/golden/make_golden.py [--reference /path/to/flashvsr-sm89-ops]

Imports aireet/flashvsr-sm89-ops from its checkout and runs the parts of the hot
path that execute on a CPU, with their own code:
  * fp8_linear.FP8Linear: weight codes + w_scale (fp8_linear.py:17-26) and a full
    forward on a non-contiguous input, i.e. the eager activation quantisation of
    fp8_linear.py:38-40 followed by torch._scaled_mm on the CPU (:28-30); the
    quantised activation handed to _mm is captured too;
  * lcsa/reference.py: window_partition, build_local_block_mask, draft_block_mask,
    sparse_attention_ref, lcsa_forward_ref (the reference's own oracle);
  * lcsa/triton_lcsa.py: build_csr (pure torch);
  * tiling.py: plan_tiles / tile_weight / _limits_for_free_bytes / render_tiled with
    the identity pipeline of comfyui/test_tiling.py.
The Triton kernels themselves need a GPU; their formulas are pinned through the
reference's declared equalities (gate-add == eager, GELU codes == quantize(gelu)).
Outputs: tests/golden/*.pt (a few hundred KB).
"""
import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FVB_REFERENCE"),
                    help="checkout of the reference package (or set FVB_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path to the reference checkout> or set FVB_REFERENCE")
    sys.path.insert(0, args.reference)
    from flashvsr_sm89_ops import fp8_linear as R_lin
    from flashvsr_sm89_ops import tiling as R_til
    from flashvsr_sm89_ops.lcsa import reference as R_ref
    from flashvsr_sm89_ops.lcsa.triton_lcsa import build_csr as R_csr

    g = torch.Generator().manual_seed(1234)

    # ---------------------------------------------------------------- FP8 linear
    fp8 = {}
    for name, (M, K, N, wdtype) in {"bf16w": (48, 256, 64, torch.bfloat16),
                                    "f32w": (33, 128, 40, torch.float32)}.items():
        lin = torch.nn.Linear(K, N)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
            lin.bias.copy_(torch.randn(N, generator=g) * 0.02)
        lin = lin.to(wdtype)
        ref = R_lin.FP8Linear(lin)
        xw = torch.randn(M, 2 * K, generator=g)
        xw[torch.rand(M, 2 * K, generator=g) < 0.01] *= 20
        x = xw.to(torch.bfloat16)[:, ::2]  # non-contiguous -> the eager quant branch
        captured = {}
        orig = ref._mm

        def spy(x8, s, _orig=orig):
            captured["x8"], captured["s"] = x8.clone(), s.clone()
            return _orig(x8, s)

        ref._mm = spy
        y = ref(x)
        fp8[name] = {
            "w": lin.weight.detach().clone(), "b": lin.bias.detach().clone(),
            "w8": ref.weight.detach().view(torch.uint8).clone(), "w_scale": ref.w_scale.clone(),
            "x": x.contiguous(), "x8": captured["x8"].view(torch.uint8), "x_scale": captured["s"],
            "y": y.detach().clone(),
        }
    torch.save(fp8, os.path.join(HERE, "fp8_linear.pt"))

    # ---------------------------------------------------------------- LCSA
    lc = {}
    H, Dh, S = 4, 32, 128
    for name, (f, h_lat, w_lat, ratio, rng) in {"a": (2, 16, 24, 0.4, 11), "b": (4, 8, 16, 0.3, 3)}.items():
        L = f * h_lat * w_lat
        q = torch.randn(1, L, H * Dh, generator=g).to(torch.bfloat16)
        k = torch.randn(1, L, H * Dh, generator=g).to(torch.bfloat16)
        v = torch.randn(1, L, H * Dh, generator=g).to(torch.bfloat16)
        bh, bw = h_lat // 8, w_lat // 8
        q_w = R_ref.window_partition(q.view(1, f, h_lat, w_lat, H * Dh))
        k_w = R_ref.window_partition(k.view(1, f, h_lat, w_lat, H * Dh))
        v_w = R_ref.window_partition(v.view(1, f, h_lat, w_lat, H * Dh))
        local = R_ref.build_local_block_mask(bh, bw, rng, "cpu")
        Nq = q_w.shape[0]
        topk = int(Nq * Nq * ratio)
        keep = R_ref.draft_block_mask(q_w, k_w, H, f // 2, local, topk)
        att = R_ref.sparse_attention_ref(q_w, k_w, v_w, keep)
        out_full, keep_full = R_ref.lcsa_forward_ref(q, k, v, f, h_lat, w_lat, H, topk, rng)
        assert torch.equal(keep_full, keep) and torch.equal(out_full.view(-1), att.reshape(-1))
        sel, cnt, maxk = R_csr(keep)
        lc[name] = {"fhw": (f, h_lat, w_lat), "H": H, "topk": topk, "rng": rng,
                    "q": q, "k": k, "v": v, "q_w": q_w, "local": local, "keep": keep,
                    "att": att.to(torch.bfloat16), "att_sum": att.double().sum().item(),
                    "sel": sel, "cnt": cnt, "maxk": maxk}
    torch.save(lc, os.path.join(HERE, "lcsa.pt"))

    # ---------------------------------------------------------------- tiling
    plans = {}
    for W in range(640, 4097, 128):
        for Hh in range(512, 2177, 128):
            plans[(W, Hh, R_til.TILE_TARGET)] = R_til.plan_tiles(W, Hh)
    for W, Hh in [(3840, 2048), (2560, 1408), (4096, 2304), (1920, 1024)]:
        for tgt in (700_000, 1_000_000, 640_000):
            plans[(W, Hh, tgt)] = R_til.plan_tiles(W, Hh, target=tgt, threshold=min(tgt, R_til.TILE_THRESHOLD))
    weights = {}  # per tile: the middle row and middle column of its [h, w] map, and its sum
    for key in [(3840, 2048, R_til.TILE_TARGET), (2560, 1408, R_til.TILE_TARGET), (3840, 2048, 700_000)]:
        tiles = plans[key]
        prof = []
        for (x, y, w, h) in tiles:
            m = R_til.tile_weight(x, y, tiles)
            prof.append((m[h // 2].clone(), m[:, w // 2].clone(), m.double().sum().item()))
        weights[key] = prof
    limits = {}
    G = 2 ** 30
    for fb in [0, int(4.5 * G), 13 * G, 20 * G, 60 * G, 170 * G]:
        for nf in (25, 85, 169):
            limits[(fb, nf)] = R_til._limits_for_free_bytes(fb, nf)
    canvas = torch.rand(1, 3, 512, 1152, generator=g) * 2 - 1
    calls = []

    def fake_pipe(LQ_video, num_frames, height, width, **kw):
        lq = LQ_video[0] if LQ_video.dim() == 5 else LQ_video
        calls.append((height, width, num_frames, kw.get("topk_ratio")))
        return lq

    rendered = R_til.render_tiled(fake_pipe, canvas, num_frames=3, prompt="", topk_ratio=0.5,
                                  tile_threshold=300_000, tile_target=300_000)
    torch.save({"plans": plans, "weights": weights, "limits": limits,
                "constants": {k: getattr(R_til, k) for k in ("MULT", "OVERLAP", "TILE_THRESHOLD",
                                                             "TILE_TARGET", "_TILE_FLOOR")},
                "render_seed_canvas_shape": tuple(canvas.shape), "render_calls": calls,
                "render_plan": R_til.plan_tiles(1152, 512, target=300_000, threshold=300_000),
                "render_maxdiff": (rendered - canvas).abs().max().item(),
                "render_sum": rendered.double().sum().item(), "render_in_sum": canvas.double().sum().item()},
               os.path.join(HERE, "tiling.pt"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
