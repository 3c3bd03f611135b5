"""Spatially tiled rendering, sharded over the GPUs of one box.

Drop-in for ``flashvsr_sm89_ops.tiling`` (tiling.py:19-205): the same module
constants, ``plan_tiles`` / ``tile_weight`` / ``auto_tile_limits`` /
``render_tiled`` with identical plans and weights (the planner is a pure
function of the canvas, so it must agree exactly).  The B200 changes are in
``render_tiled``:
  * blending happens on the GPU in fp32 (the reference blends on the host,
    tiling.py:203), so a tile's frames never leave HBM until the end;
  * under ``torch.distributed`` with world size N > 1, tile i is rendered by rank
    i % N, each rank accumulates its weighted tiles into its own partial canvas,
    and one ``dist.reduce`` (NCCL over NVLink on GPUs, gloo on CPU) sums the
    partial canvases into rank 0.  The weights form a partition of unity, so the
    sum is the blended canvas.  Rank 0 returns it; the other ranks return None.
"""
from __future__ import annotations

import os

import torch

MULT = 128                # pipeline output grid (px)
OVERLAP = 256             # shared pixels between neighbouring tiles
TILE_THRESHOLD = 2_200_000
TILE_TARGET = 2_100_000
_GIB_PER_MP = 8.6
_REFERENCE_FRAMES = 85
_SAFETY_GIB = 1.25
_TILE_FLOOR = 640_000


def _round_up(v: int, mult: int = MULT) -> int:
    return ((v + mult - 1) // mult) * mult


def _limits_for_free_bytes(free_bytes, num_frames=_REFERENCE_FRAMES, safety_gib=_SAFETY_GIB):
    """(threshold, target) for `free_bytes` of device memory, or None if nothing is left.

    Same VRAM model as tiling.py:45-61: activation GiB per output megapixel scales
    linearly with the frame count; target is clamped to [floor, TILE_TARGET] and
    the threshold follows it down.
    """
    usable = free_bytes - int(safety_gib * (1 << 30))
    if usable <= 0:
        return None
    per_mp = _GIB_PER_MP * max(num_frames, 1) / _REFERENCE_FRAMES
    tgt = int(usable / (per_mp * (1 << 30)) * 1e6)
    tgt = max(min(TILE_TARGET, tgt), _TILE_FLOOR)
    return min(TILE_THRESHOLD, tgt), tgt


def auto_tile_limits(num_frames=_REFERENCE_FRAMES, device="cuda", safety_gib=_SAFETY_GIB):
    """(threshold, target) sized to the memory actually free now (tiling.py:64-82)."""
    if device != "cuda" or not torch.cuda.is_available():
        return TILE_THRESHOLD, TILE_TARGET
    try:
        torch.cuda.empty_cache()
        free, _ = torch.cuda.mem_get_info()
    except Exception:
        return TILE_THRESHOLD, TILE_TARGET
    lim = _limits_for_free_bytes(free, num_frames, safety_gib)
    return lim if lim is not None else (TILE_THRESHOLD, TILE_TARGET)


def _strip_starts(canvas, piece, n):
    """Offsets of n pieces covering [0, canvas): evenly strided, last one flush right."""
    step = (canvas - piece) // (n - 1)
    out = [k * step for k in range(n - 1)]
    out.append(canvas - piece)
    return out


def _piece(canvas, n, overlap):
    return _round_up((canvas + (n - 1) * overlap + n - 1) // n)


def plan_tiles(W, H, target=TILE_TARGET, threshold=TILE_THRESHOLD, overlap=OVERLAP, mult=MULT):
    """Cover W x H with overlapping tiles on the mult grid -> [(x, y, w, h), ...].

    Order of preference (tiling.py:96-137): the full frame when W*H <= threshold;
    2..8 full-height vertical strips; 2..8 full-width horizontal strips; otherwise
    a cols x rows grid (2..6 each) with the fewest seams, then the fewest pieces.
    """
    if W * H <= threshold:
        return [(0, 0, W, H)]
    smallest = overlap + mult

    def usable(p, canvas, cross):
        return smallest <= p <= canvas and p * cross <= target

    for n in range(2, 9):
        p = _piece(W, n, overlap)
        if usable(p, W, H):
            return [(x, 0, p, H) for x in _strip_starts(W, p, n)]
    for n in range(2, 9):
        p = _piece(H, n, overlap)
        if usable(p, H, W):
            return [(0, y, W, p) for y in _strip_starts(H, p, n)]
    choice = None
    for cols in range(2, 7):
        for rows in range(2, 7):
            pw, ph = _piece(W, cols, overlap), _piece(H, rows, overlap)
            if pw * ph > target or pw < smallest or ph < smallest:
                continue
            rank = (cols + rows - 2, cols * rows)
            if choice is None or rank < choice[0]:
                choice = (rank, pw, ph, cols, rows)
    if choice is None:
        raise ValueError(f"cannot tile {W}x{H} into ~{target} px pieces")
    _, pw, ph, cols, rows = choice
    return [(x, y, pw, ph) for y in _strip_starts(H, ph, rows) for x in _strip_starts(W, pw, cols)]


def _axis_weights(starts, piece):
    """Per-piece 1-D weights: linear ramps across each shared span, summing to 1."""
    ws = []
    last = len(starts) - 1
    for i, s in enumerate(starts):
        w = torch.ones(piece, dtype=torch.float32)
        if i > 0:
            span = starts[i - 1] + piece - s
            w[:span] = torch.linspace(0.0, 1.0, span + 2)[1:-1]
        if i < last:
            span = s + piece - starts[i + 1]
            w[piece - span:] = torch.linspace(1.0, 0.0, span + 2)[1:-1]
        ws.append(w)
    return ws


def tile_weight(x, y, tiles):
    """Blending weight of the tile at (x, y) as an [h, w] map; all tiles sum to 1."""
    xs = sorted({t[0] for t in tiles})
    ys = sorted({t[1] for t in tiles})
    wx = _axis_weights(xs, tiles[0][2])[xs.index(x)]
    wy = _axis_weights(ys, tiles[0][3])[ys.index(y)]
    return wy[:, None] * wx[None, :]


def assign_tiles(n_tiles: int, world: int, rank: int):
    """Tile indices rendered by `rank` (round-robin; every tile exactly once)."""
    return list(range(rank, n_tiles, world))


def _dist_info(group):
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


class _Staging:
    """Two device buffers (and, for a pageable host video, two pinned host buffers) for one
    device and dtype, with the events that order their reuse, kept across render_tiled
    calls: pinning a few hundred MB of host memory takes a large fraction of a second, which
    a fresh allocation per call would add to every render.  Calls on one device share them,
    so render_tiled calls on the same device must not run concurrently from several host
    threads."""

    def __init__(self, device, dtype, numel, host=True):
        self.stage = [torch.empty(numel, dtype=dtype, pin_memory=True)
                      for _ in range(2)] if host else []
        self.dev = [torch.empty(numel, dtype=dtype, device=device) for _ in range(2)]
        self.up_done = [None, None]    # upload into device buffer b (from stage b) finished
        self.used = [None, None]       # render of the tile in device buffer b finished

    def numel(self):
        return self.dev[0].numel()


_STAGING = {}


def _staging_for(device, dtype, numel, host=True):
    key = (str(torch.device(device)), dtype, host)
    st = _STAGING.get(key)
    if st is None or st.numel() < numel:
        if st is not None:  # the old buffers may still feed work in flight
            for ev in st.up_done + st.used:
                if ev is not None:
                    ev.synchronize()
        st = _Staging(device, dtype, numel, host)
        _STAGING[key] = st
    return st


def _dma_source(lq, device):
    """A pinned, contiguous host video: crops go to the device as one strided copy-engine
    transfer each (fvb_copy_window_h2d), with no host-side packing."""
    return (torch.device(device).type == "cuda" and lq.device.type == "cpu"
            and lq.is_pinned() and lq.is_contiguous())


def _crop_numel(lq, tiles, order):
    return max((tiles[i][2] * tiles[i][3] for i in order), default=0) * lq.shape[0] * lq.shape[1]


def reserve_staging(lq_video, *, overlap=OVERLAP, tile_target=TILE_TARGET,
                    tile_threshold=TILE_THRESHOLD, device=None, group=None):
    """Allocate this rank's crop staging for render_tiled(lq_video, ...) ahead of the first
    call (same tiling arguments), so that call does not pay for pinning host memory.  The
    buffers stay allocated until release_staging()."""
    lq = lq_video[0] if lq_video.dim() == 5 else lq_video
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if lq.device == device or device.type != "cuda":
        return
    C, F, H, W = lq.shape
    tiles = plan_tiles(W, H, target=tile_target, threshold=tile_threshold, overlap=overlap)
    world, rank = _dist_info(group)
    n = _crop_numel(lq, tiles, assign_tiles(len(tiles), world, rank))
    if n:
        _staging_for(device, lq.dtype, n, host=not _dma_source(lq, device))


def release_staging():
    """Free the crop staging buffers kept by render_tiled / reserve_staging."""
    for st in _STAGING.values():
        for ev in st.up_done + st.used:
            if ev is not None:
                ev.synchronize()
    _STAGING.clear()


class _TileLoader:
    """Brings the LQ crops of one rank's tiles onto its GPU ahead of use.

    A crop of a host video is a strided view; copying it as is costs a contiguous host copy
    plus a synchronous pageable transfer per tile, in series with the tile's compute.  Here
    a worker thread packs crop k+1 into a pinned staging buffer while the GPU renders tile k,
    a side stream uploads it, and the render stream waits on an event.  Two staging and two
    device buffers rotate (kept across calls, see _Staging); the side stream reuses a device
    buffer only after the render of the tile that used it (an event recorded after its
    blend).  A video already on the device is cropped there.
    A pinned contiguous host video needs no packing: the side stream copies each crop
    straight from it with one strided copy-engine transfer (crop k+1 is queued when tile k
    starts), so no host thread touches the pixels and ranks sharing a host do not compete
    for its memory bandwidth.
    """

    def __init__(self, lq, tiles, order, device):
        device = torch.device(device)
        self.lq, self.tiles, self.order, self.device = lq, tiles, list(order), device
        self.direct = lq.device == device or device.type != "cuda"
        self.dma = False
        if self.direct:
            return
        from concurrent.futures import ThreadPoolExecutor
        self.dma = _dma_source(lq, device)
        self.st = _staging_for(device, lq.dtype, _crop_numel(lq, tiles, self.order),
                               host=not self.dma)
        self.copy_stream = torch.cuda.Stream(device)
        if self.dma:
            self.uploaded = {}
            if self.order:
                self._upload(0)
            return
        self.pool = ThreadPoolExecutor(1)
        # a crop is copied by several host threads, split by frames (torch's copy releases
        # the GIL); the host's cores are shared by the ranks of this machine
        nproc = os.cpu_count() or 1
        local = max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
        self.n_copy = max(1, min(8, nproc // local, lq.shape[1]))
        self.copiers = ThreadPoolExecutor(self.n_copy) if self.n_copy > 1 else None
        self.pending = self.pool.submit(self._pack, 0) if self.order else None

    def _shape(self, k):
        x, y, w, h = self.tiles[self.order[k]]
        return self.lq.shape[0], self.lq.shape[1], h, w

    def _pack(self, k):
        x, y, w, h = self.tiles[self.order[k]]
        b = k & 1
        if self.st.up_done[b] is not None:
            self.st.up_done[b].synchronize()  # stage b still feeds an upload in flight
        shp = self._shape(k)
        n = shp[0] * shp[1] * shp[2] * shp[3]
        dst = self.st.stage[b][:n].view(shp)
        src = self.lq[:, :, y:y + h, x:x + w]
        if self.copiers is None:
            dst.copy_(src)
            return k
        F = shp[1]
        cuts = [F * i // self.n_copy for i in range(self.n_copy + 1)]
        jobs = [self.copiers.submit(dst[:, f0:f1].copy_, src[:, f0:f1])
                for f0, f1 in zip(cuts[:-1], cuts[1:]) if f1 > f0]
        for j in jobs:
            j.result()
        return k

    def _upload(self, k):
        """Queue crop k on the side stream as one strided transfer from the pinned video
        into device buffer k & 1, after the render of the tile that last used it."""
        from . import _lib
        x, y, w, h = self.tiles[self.order[k]]
        b, st = k & 1, self.st
        C, F, H, W = self.lq.shape
        es = self.lq.element_size()
        with torch.cuda.stream(self.copy_stream):
            # after the tile that last read buffer b, and after any earlier upload into it
            # (a render that stopped early can leave one in flight on its own side stream)
            for prev in (st.used[b], st.up_done[b]):
                if prev is not None:
                    self.copy_stream.wait_event(prev)
            _lib.call("fvb_copy_window_h2d", self.lq.data_ptr(), W * es, H, C * F, x * es, y,
                      w * es, h, st.dev[b].data_ptr(), self.copy_stream.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        st.up_done[b] = ev
        self.uploaded[k] = ev

    def get(self, k):
        """Crop of tile order[k] on the device, usable on the current stream."""
        x, y, w, h = self.tiles[self.order[k]]
        if self.direct:
            return self.lq[:, :, y:y + h, x:x + w].to(self.device)
        if self.dma:
            ev = self.uploaded.pop(k)
            if k + 1 < len(self.order):
                self._upload(k + 1)  # its buffer's last tile, k - 1, is marked done by now
            torch.cuda.current_stream(self.device).wait_event(ev)
            shp = self._shape(k)
            return self.st.dev[k & 1][:shp[0] * shp[1] * shp[2] * shp[3]].view(shp)
        self.pending.result()
        b = k & 1
        shp = self._shape(k)
        n = shp[0] * shp[1] * shp[2] * shp[3]
        st = self.st
        with torch.cuda.stream(self.copy_stream):
            if st.used[b] is not None:
                self.copy_stream.wait_event(st.used[b])
            st.dev[b][:n].copy_(st.stage[b][:n], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        st.up_done[b] = ev
        self.pending = self.pool.submit(self._pack, k + 1) if k + 1 < len(self.order) else None
        torch.cuda.current_stream(self.device).wait_event(ev)
        return st.dev[b][:n].view(shp)

    def done(self, k):
        """The render stream has finished with tile order[k]'s device buffer."""
        if self.direct:
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.st.used[k & 1] = ev

    def close(self):
        if self.dma:
            # a render that stopped early may leave a prefetched crop in flight: finish it
            # before the caller may free or refill the host video it reads
            for ev in self.uploaded.values():
                ev.synchronize()
            self.uploaded.clear()
            return
        if not self.direct:
            if self.pending is not None:
                self.pending.result()
            self.pool.shutdown()
            if self.copiers is not None:
                self.copiers.shutdown()


def render_tiled(pipe, lq_video, *, overlap=OVERLAP, tile_target=TILE_TARGET,
                 tile_threshold=TILE_THRESHOLD, device=None, group=None, timings=None,
                 **pipe_kwargs):
    """Render lq_video [C,F,H,W] (or [1,C,F,H,W], in [-1, 1]) through `pipe` one tile at a time.

    Same contract as tiling.py:164-205: per-tile LQ crop, height/width and an
    area-scaled topk_ratio; returns [C, F', H, W] in lq_video's dtype.  Blending
    runs on `device` (default: this rank's CUDA device, else CPU).  With a
    process group of N ranks each rank renders tiles i % N == rank and rank 0
    returns the reduced canvas (other ranks return None).

    timings (optional dict, CUDA devices): filled with "events" (CUDA events at the start,
    after this rank's last tile is blended, and after the cross-rank reduce), "load_wait_s"
    (host seconds spent waiting for the next crop to be packed) and "tiles" (this rank's
    tile count), so a caller can split the render into tile work, crop loading and the
    exchange.
    """
    import time

    import torch.distributed as dist

    batched = lq_video.dim() == 5
    lq = lq_video[0] if batched else lq_video
    C, F, H, W = lq.shape
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    pipe_kwargs.setdefault("num_frames", F)
    tiles = plan_tiles(W, H, target=tile_target, threshold=tile_threshold, overlap=overlap)
    world, rank = _dist_info(group)
    if len(tiles) == 1 and world == 1:
        return pipe(LQ_video=lq_video.to(device), height=H, width=W, **pipe_kwargs)

    num_frames = pipe_kwargs.pop("num_frames")
    base_topk = pipe_kwargs.pop("topk_ratio", None)
    mine = assign_tiles(len(tiles), world, rank)
    canvas = None
    n_out = torch.zeros(1, dtype=torch.int64, device=device)
    events = None
    if timings is not None and torch.device(device).type == "cuda":
        events = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        events[0].record(torch.cuda.current_stream(device))
    wait = 0.0
    loader = _TileLoader(lq, tiles, mine, device)
    try:
        for k, i in enumerate(mine):
            x, y, w, h = tiles[i]
            t0 = time.perf_counter()
            crop = loader.get(k)
            wait += time.perf_counter() - t0
            extra = {"topk_ratio": base_topk * (W * H) / (w * h)} if base_topk is not None else {}
            frames = pipe(LQ_video=crop.unsqueeze(0) if batched else crop, num_frames=num_frames,
                          height=h, width=w, **extra, **pipe_kwargs)
            if canvas is None:
                canvas = torch.zeros((C, frames.shape[-3], H, W), dtype=torch.float32, device=device)
                n_out.fill_(frames.shape[-3])
            elif canvas.shape[1] != frames.shape[-3]:
                raise RuntimeError(f"tile frame counts diverge: {canvas.shape[1]} vs {frames.shape[-3]}")
            wgt = tile_weight(x, y, tiles).to(device)
            canvas[:, :, y:y + h, x:x + w] += frames.to(device=device, dtype=torch.float32) * wgt
            loader.done(k)
            del frames, crop
    finally:
        loader.close()
    if events is not None:
        events[1].record(torch.cuda.current_stream(device))
    if timings is not None:
        timings.update(events=events, load_wait_s=wait, tiles=len(mine))
    if world == 1:
        if events is not None:
            events[2].record(torch.cuda.current_stream(device))
        return canvas.to(dtype=lq_video.dtype)
    # every rank needs the output frame count to size its (possibly empty) canvas
    dist.all_reduce(n_out, op=dist.ReduceOp.MAX, group=group)
    if canvas is None:
        canvas = torch.zeros((C, int(n_out.item()), H, W), dtype=torch.float32, device=device)
    elif canvas.shape[1] != int(n_out.item()):
        raise RuntimeError(f"rank {rank}: tile frame count {canvas.shape[1]} != {int(n_out.item())}")
    dist.reduce(canvas, dst=0, op=dist.ReduceOp.SUM, group=group)
    if events is not None:
        events[2].record(torch.cuda.current_stream(device))
    if rank == 0:
        return canvas.to(dtype=lq_video.dtype)
    return None
