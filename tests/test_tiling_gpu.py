"""render_tiled on the GPU: the prefetching host-crop path equals cropping on the device.

The host video takes the pinned-staging / side-stream upload path of the tile loader; the
same video already on the device is cropped there.  A deterministic per-tile pipe (a crop
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
