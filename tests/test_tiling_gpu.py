"""render_tiled on the GPU: the prefetching host-crop path equals cropping on the device.

A pageable host video takes the pinned-staging / side-stream upload path of the tile
loader, a pinned one the strided copy-engine path; the same video already on the device is
cropped there.  A deterministic per-tile pipe (a crop
transform, frame count changed like the real pipeline) makes any mix-up of tiles, buffers
or stream ordering visible in the blended canvas.
"""
import pytest
import torch

from flashvsr_sm89_ops_b200.tiling import render_tiled

pytestmark = pytest.mark.gpu


def _pipe(LQ_video, num_frames, height, width, **kw):
    v = LQ_video[0] if LQ_video.dim() == 5 else LQ_video
    # drop the first frame, scale by a tile-size dependent factor: depends on crop content
    return (v[:, 1:].float() * 0.5 + 0.001 * (height + width)).to(v.dtype)


@pytest.mark.parametrize("pinned", [True, False])
def test_host_crops_match_device_crops(pinned):
    g = torch.Generator().manual_seed(3)
    C, F, H, W = 3, 5, 1536, 2688
    lq = (torch.rand(C, F, H, W, generator=g) * 2 - 1).to(torch.bfloat16)
    if pinned:
        lq = lq.pin_memory()
    kw = dict(num_frames=F, tile_target=700_000, tile_threshold=700_000, device="cuda")
    ref = render_tiled(_pipe, lq.cuda(), **kw)
    out = render_tiled(_pipe, lq, **kw)
    torch.cuda.synchronize()
    assert out.shape == (C, F - 1, H, W)
    assert torch.equal(out, ref)


def test_tiled_pipe_graph_replay_equals_eager():
    """The 4K workload's stand-in pipe replays one captured CUDA graph per tile shape; each
    replay (new crop copied into the graph's input) equals the eager schedule bit for bit."""
    from flashvsr_sm89_ops_b200.runner import StreamingDiT, TiledDiTPipe
    dev = torch.device("cuda:0")
    r = StreamingDiT(num_layers=2, height=256, width=256, device=dev)
    eager = TiledDiTPipe(r, n_steps=2, graph=False)
    graphed = TiledDiTPipe(r, n_steps=2, graph=True)
    F = 4 * eager.latent_frames() + 1
    g = torch.Generator(device=dev).manual_seed(3)
    for _ in range(3):  # capture on the first call, replay on the next two
        crop = (torch.rand(3, F, 256, 384, generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
        a = eager(LQ_video=crop).clone()
        b = graphed(LQ_video=crop).clone()
        torch.cuda.synchronize(dev)
        assert torch.equal(a, b)
    assert graphed.tokens == eager.tokens


@pytest.mark.parametrize("pinned", [False, True])
def test_crop_staging_is_reused_across_renders(pinned):
    """render_tiled keeps its crop staging between calls (reserve_staging allocates it
    ahead): back-to-back renders of different host videos through the same buffers each
    equal the render of that video cropped on the device.  Pageable videos are packed into
    pinned staging; pinned ones are copied by strided transfers (fvb_copy_window_h2d)."""
    from flashvsr_sm89_ops_b200 import tiling
    g = torch.Generator().manual_seed(9)
    C, F, H, W = 3, 5, 1536, 2688
    kw = dict(num_frames=F, tile_target=700_000, tile_threshold=700_000, device="cuda")
    videos = [(torch.rand(C, F, H, W, generator=g) * 2 - 1).to(torch.bfloat16) for _ in range(2)]
    if pinned:
        videos = [v.pin_memory() for v in videos]
    tiling.release_staging()
    tiling.reserve_staging(videos[0], tile_target=700_000, tile_threshold=700_000, device="cuda")
    st = next(iter(tiling._STAGING.values()))
    outs = [render_tiled(_pipe, v, **kw) for v in videos]
    torch.cuda.synchronize()
    assert next(iter(tiling._STAGING.values())) is st
    for v, out in zip(videos, outs):
        assert torch.equal(out, render_tiled(_pipe, v.cuda(), **kw))
    tiling.release_staging()
    assert not tiling._STAGING
