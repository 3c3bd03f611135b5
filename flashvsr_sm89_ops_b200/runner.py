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
