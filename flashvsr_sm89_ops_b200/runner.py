"""Streaming driver of a FlashVSR-Tiny-shaped DiT on this pack (benchmark and smoke use).

Builds the stand-in Wan DiT (``wan_video_dit``) with random-init weights on one
GPU, wires it with the real ``enable()``, caches the cross-attention K/V of a
512-token context, primes the per-block self-attention KV caches with the f=6
start chunk, and then runs steady-state f=2 chunks exactly like the FlashVSR
streaming loop (integrate.py:51-54, :81-83, :108-115): Nq = 1 time row of
windows, Nk = kv_len cached rows + the new row.  ``capture()`` records one step
in a CUDA graph (every op launches on the current stream, allocates from the
caching allocator and never synchronises, so the whole 30-block step replays
as one graph).
"""
from __future__ import annotations

import torch

from . import wan_video_dit as W
from .integrate import enable


class StreamingDiT:
    def __init__(self, num_layers=30, dim=1536, heads=12, ffn=8960, height=768, width=1408,
                 ctx_len=512, kv_len=3, mask_rule="causal", topk=None, seed=0, device="cuda",
                 verbose=False):
        self.device = torch.device(device)
        self.h, self.w = height // 16, width // 16
        self.kv_len = kv_len
        self.dim = dim
        self.topk = topk
        W.MASK_RULE = mask_rule
        with torch.device(self.device):
            dit = W.WanDiT(num_layers, dim, heads, ffn)
        dit = dit.to(torch.bfloat16)
        self._init(dit, seed)
        self.dit = dit
        self.applied = enable(W.DiTPipe(dit), dit_module=W, verbose=verbose)
        g = torch.Generator(device=self.device).manual_seed(seed + 1)
        ctx = torch.randn(1, ctx_len, dim, generator=g, device=self.device).to(torch.bfloat16)
        dit.init_cross_kv(ctx)
        self.ctx = ctx
        self.t_mod = torch.randn(1, 6, dim, generator=g, device=self.device).to(torch.bfloat16)
        self.caches = None
        self.graph = None

    @torch.no_grad()
    def _init(self, dit, seed):
        g = torch.Generator(device=self.device).manual_seed(seed)
        for name, p in dit.named_parameters():
            if name.endswith("modulation"):
                t = torch.randn(p.shape, generator=g, device=self.device)
            elif ".norm" in name and name.endswith("weight"):
                t = 1 + 0.1 * torch.randn(p.shape, generator=g, device=self.device)
            elif ".norm" in name and name.endswith("bias"):
                t = 0.1 * torch.randn(p.shape, generator=g, device=self.device)
            else:
                t = 0.02 * torch.randn(p.shape, generator=g, device=self.device)
            p.copy_(t.to(p.dtype))

    def tokens(self, f):
        return f * self.h * self.w

    def make_input(self, f, seed=7):
        g = torch.Generator(device=self.device).manual_seed(seed)
        return torch.randn(1, self.tokens(f), self.dim, generator=g, device=self.device).to(torch.bfloat16)

    @torch.no_grad()
    def prime(self):
        """Start chunk (f=6): fills every block's KV cache with 3 time rows."""
        x = self.make_input(6, seed=3)
        fr = self.dit.chunk_freqs(6, self.h, self.w, 0, self.device)
        _, self.caches = self.dit.forward_chunk(x, self.t_mod, fr, (6, self.h, self.w), None,
                                                topk=self.topk, kv_len=self.kv_len)
        self.freqs2 = self.dit.chunk_freqs(2, self.h, self.w, 6, self.device)
        return self.caches

    @torch.no_grad()
    def step(self, x):
        """One steady-state f=2 chunk through every block (caches are inputs, unchanged)."""
        if self.caches is None:
            self.prime()
        y, _ = self.dit.forward_chunk(x, self.t_mod, self.freqs2, (2, self.h, self.w), self.caches,
                                      topk=self.topk, kv_len=self.kv_len)
        return y

    @torch.no_grad()
    def capture(self, x_static):
        """Record step(x_static) in a CUDA graph; returns (graph, output tensor)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step(x_static)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            y = self.step(x_static)
        self.graph = (g, y)
        return g, y


class HostStream:
    """Steps from pinned host inputs to pinned host outputs with the copies off the compute
    stream: while step i runs, a copy stream uploads step i+1's input into a device staging
    buffer and downloads step i-1's output, so the host transfers overlap the DiT instead of
    adding to it.  Each step costs two device-to-device copies (the step's static input and
    output buffers to and from staging, ~10 us each at the 1408x768 shape).

    step_fn() runs one step reading x_static and writing y_static (a graph replay or an
    eager call).  run(x_hosts, y_hosts) takes equal-length lists of pinned host tensors
    (the same tensor may repeat) and returns when every output has landed.
    """

    def __init__(self, step_fn, x_static: torch.Tensor, y_static: torch.Tensor):
        self.step_fn = step_fn
        self.x, self.y = x_static, y_static
        dev = x_static.device
        self.copy = torch.cuda.Stream(dev)
        self.xs = [torch.empty_like(x_static) for _ in range(2)]
        self.ys = [torch.empty_like(y_static) for _ in range(2)]
        ev = lambda: [torch.cuda.Event() for _ in range(2)]  # noqa: E731
        self.x_up, self.x_used, self.y_ready, self.y_down = ev(), ev(), ev(), ev()

    def run(self, x_hosts, y_hosts):
        n = len(x_hosts)
        if len(y_hosts) != n:
            raise ValueError("HostStream.run: x_hosts and y_hosts differ in length")
        if n == 0:
            return
        comp = torch.cuda.current_stream(self.x.device)
        with torch.cuda.stream(self.copy):
            self.xs[0].copy_(x_hosts[0], non_blocking=True)
            self.x_up[0].record(self.copy)
        for i in range(n):
            b = i & 1
            comp.wait_event(self.x_up[b])
            self.x.copy_(self.xs[b], non_blocking=True)
            self.x_used[b].record(comp)
            if i + 1 < n:  # upload the next input while this step computes
                nb = b ^ 1
                with torch.cuda.stream(self.copy):
                    if i >= 1:
                        self.copy.wait_event(self.x_used[nb])
                    self.xs[nb].copy_(x_hosts[i + 1], non_blocking=True)
                    self.x_up[nb].record(self.copy)
            self.step_fn()
            if i >= 2:  # staging buffer b is free once step i-2's output is on the host
                comp.wait_event(self.y_down[b])
            self.ys[b].copy_(self.y, non_blocking=True)
            self.y_ready[b].record(comp)
            with torch.cuda.stream(self.copy):
                self.copy.wait_event(self.y_ready[b])
                y_hosts[i].copy_(self.ys[b], non_blocking=True)
                self.y_down[b].record(self.copy)
        comp.wait_stream(self.copy)


class TiledDiTPipe:
    """Stand-in FlashVSR pipeline for ``render_tiled`` (the 4K tiled workload).

    Per tile: the LQ crop [C, F, h, w] is patch-embedded (16x16 px x 4 frames per token, one
    bf16 linear), run through the DiT's streaming schedule (integrate.py:51-54): one f=6
    chunk, then f=2 chunks whose self-attention reads the KV caches of the last ``kv_len``
    time rows, and each chunk's output is unpatchified back to frames (one bf16 linear).
    The patch embedding and the decoder are plain linears standing in for the pipeline's
    LQ projection and VAE, which are not part of this operator pack.  Returns
    [3, 4 * (6 + 2 * n_steps), h, w] bf16 frames.
    """

    def __init__(self, runner: StreamingDiT, n_steps: int = 7, seed: int = 5, graph: bool = True):
        self.r = runner
        self.n_steps = n_steps
        dev = runner.device
        g = torch.Generator(device=dev).manual_seed(seed)
        patch = 3 * 4 * 16 * 16
        self.emb = (0.02 * torch.randn(patch, runner.dim, generator=g, device=dev)).to(torch.bfloat16)
        self.unemb = (0.02 * torch.randn(runner.dim, patch, generator=g, device=dev)).to(torch.bfloat16)
        self.tokens = 0
        # graph=True: a tile's whole schedule (patch-embed, every chunk through every block,
        # unpatchify) is captured once per crop shape as one CUDA graph and replayed for each
        # tile of that shape, so a tile costs one launch on the host instead of thousands.
        # The returned frames then live in the graph's output buffer, valid until the next call.
        self.graph = graph and torch.device(dev).type == "cuda"
        self._graphs = {}
        self._freqs = {}

    def latent_frames(self):
        return 6 + 2 * self.n_steps

    @torch.no_grad()
    def __call__(self, LQ_video, num_frames=None, height=None, width=None, **kwargs):
        crop = LQ_video[0] if LQ_video.dim() == 5 else LQ_video
        C, F, h, w = crop.shape
        lf = self.latent_frames()
        if C != 3 or F < 4 * lf + 1 or h % 16 or w % 16:
            raise ValueError(f"TiledDiTPipe: crop {tuple(crop.shape)} needs 3 channels, "
                             f">= {4 * lf + 1} frames and 16-px multiples")
        tokens = lf * (h // 16) * (w // 16)
        if not self.graph:
            self.tokens += tokens
            return self._forward(crop)
        key = (tuple(crop.shape), crop.dtype)
        st = self._graphs.get(key)
        if st is None:
            static_in = crop.clone()
            self._forward(static_in)  # eager warm-up: lazy allocations and caches
            side = torch.cuda.Stream(self.r.device)
            side.wait_stream(torch.cuda.current_stream(self.r.device))
            with torch.cuda.stream(side):
                self._forward(static_in)
            torch.cuda.current_stream(self.r.device).wait_stream(side)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                static_out = self._forward(static_in)
            st = (gr, static_in, static_out)
            self._graphs[key] = st
        gr, static_in, static_out = st
        static_in.copy_(crop)
        gr.replay()
        self.tokens += tokens
        return static_out

    def _forward(self, crop):
        r = self.r
        C, F, h, w = crop.shape
        lf = self.latent_frames()
        hh, ww = h // 16, w // 16
        # [3, 4*lf, h, w] -> tokens [lf*hh*ww, 3*4*16*16] in (f, h, w) raster order
        v = crop[:, 1:1 + 4 * lf].to(torch.bfloat16)
        v = v.reshape(C, lf, 4, hh, 16, ww, 16).permute(1, 3, 5, 0, 2, 4, 6)
        x = (v.reshape(lf * hh * ww, -1) @ self.emb).unsqueeze(0)
        per = hh * ww
        dit = r.dit
        outs = []
        f0 = 0
        caches = None
        for f in [6] + [2] * self.n_steps:
            xc = x[:, f0 * per:(f0 + f) * per]
            fkey = (f, hh, ww, f0)
            fr = self._freqs.get(fkey)
            if fr is None:  # built on the host once per chunk shape, before any capture
                fr = dit.chunk_freqs(f, hh, ww, f0, r.device)
                self._freqs[fkey] = fr
            y, caches = dit.forward_chunk(xc, r.t_mod, fr, (f, hh, ww), caches, topk=r.topk,
                                          kv_len=r.kv_len)
            outs.append(y[0])
            f0 += f
        p = torch.cat(outs) @ self.unemb  # [lf*hh*ww, 3*4*16*16]
        p = p.reshape(lf, hh, ww, C, 4, 16, 16).permute(3, 0, 4, 1, 5, 2, 6)
        return p.reshape(C, 4 * lf, h, w)
