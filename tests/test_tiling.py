"""Tiling contract (CPU only): the reference's own offline tests (comfyui/test_tiling.py)
restated against this pack, plus exact agreement with plans / weights / limits produced
by the reference planner (tests/golden/tiling.pt)."""
import os

import pytest
import torch

from flashvsr_sm89_ops_b200.tiling import (MULT, OVERLAP, TILE_TARGET, TILE_THRESHOLD,
                                           _limits_for_free_bytes, auto_tile_limits, plan_tiles,
                                           render_tiled, tile_weight)

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiling.pt")


def check_plan(W, H, tiles, tiled_expected, target=TILE_TARGET):
    assert (len(tiles) > 1) == tiled_expected, (W, H, tiles)
    for x, y, w, h in tiles:
        assert w % MULT == 0 and h % MULT == 0
        if tiled_expected:
            assert w * h <= target
        assert 0 <= x and x + w <= W and 0 <= y and y + h <= H
    cov = torch.zeros(H, W)
    for x, y, w, h in tiles:
        cov[y:y + h, x:x + w] += 1
    assert (cov >= 1).all(), f"{W}x{H}: uncovered pixels"
    xs = sorted({t[0] for t in tiles})
    for a, b in zip(xs, xs[1:]):
        assert a + tiles[0][2] - b >= OVERLAP


def test_buckets():
    check_plan(1280, 640, plan_tiles(1280, 640), False)
    check_plan(1920, 1024, plan_tiles(1920, 1024), False)
    check_plan(2560, 1408, plan_tiles(2560, 1408), True)
    check_plan(3840, 2048, plan_tiles(3840, 2048), True)


def test_sweep():
    for W in range(640, 4097, 128):
        for H in range(512, 2177, 128):
            check_plan(W, H, plan_tiles(W, H), W * H > TILE_THRESHOLD)


def test_weights_partition_of_unity():
    for W, H in [(2560, 1408), (3840, 2048), (1728, 2304), (4096, 2304)]:
        tiles = plan_tiles(W, H)
        if len(tiles) == 1:
            continue
        acc = torch.zeros(H, W)
        for x, y, w, h in tiles:
            acc[y:y + h, x:x + w] += tile_weight(x, y, tiles)
        assert torch.allclose(acc, torch.ones(H, W), atol=1e-5)


def test_render_identity():
    calls = []

    def fake_pipe(LQ_video, num_frames, height, width, **kw):
        lq = LQ_video[0] if LQ_video.dim() == 5 else LQ_video
        calls.append((lq.shape[-2], lq.shape[-1], num_frames, kw.get("topk_ratio")))
        return lq

    torch.manual_seed(0)
    canvas = torch.rand(3, 5, 1408, 2560) * 2 - 1
    out = render_tiled(fake_pipe, canvas, num_frames=5, prompt="",
                       topk_ratio=2.0 * 768 * 1280 / (2560 * 1408), device="cpu")
    assert out.shape == canvas.shape
    assert (out.float() - canvas).abs().max().item() < 1e-4
    assert len(calls) == 2 and all(c[1] < 2560 and c[0] == 1408 for c in calls)
    assert abs(calls[0][3] - calls[1][3]) < 1e-9
    calls.clear()
    out5 = render_tiled(fake_pipe, canvas.unsqueeze(0), num_frames=5, prompt="", device="cpu")
    assert out5.dim() == 4 and out5.shape == canvas.shape


def test_vram_sizing():
    G = 2 ** 30
    th20, tg20 = _limits_for_free_bytes(20 * G, 85)
    assert tg20 == TILE_TARGET and th20 == tg20
    th16, tg16 = _limits_for_free_bytes(13 * G, 85)
    assert tg16 < TILE_TARGET and th16 == tg16
    check_plan(1920, 1024, plan_tiles(1920, 1024, target=tg16, threshold=th16), True, tg16)
    assert _limits_for_free_bytes(13 * G, 169)[1] <= tg16
    assert _limits_for_free_bytes(13 * G, 25)[1] <= TILE_TARGET
    th0, tg0 = _limits_for_free_bytes(int(4.5 * G), 85)
    assert tg0 == 640_000 and th0 == tg0
    assert _limits_for_free_bytes(0, 85) is None
    assert auto_tile_limits(device="cpu") == (TILE_THRESHOLD, TILE_TARGET)


def test_plan_errors():
    with pytest.raises(ValueError):
        plan_tiles(4096, 4096, target=100_000, threshold=100_000)


@pytest.fixture(scope="module")
def gold():
    return torch.load(GOLD, weights_only=False)


def test_constants_match_reference(gold):
    import flashvsr_sm89_ops_b200.tiling as T
    for k, v in gold["constants"].items():
        assert getattr(T, k) == v


def test_plans_match_reference(gold):
    for (W, H, tgt), plan in gold["plans"].items():
        thr = TILE_THRESHOLD if tgt == TILE_TARGET else min(tgt, TILE_THRESHOLD)
        assert plan_tiles(W, H, target=tgt, threshold=thr) == plan, (W, H, tgt)


def test_weights_match_reference(gold):
    for key, prof in gold["weights"].items():
        tiles = gold["plans"][key]
        for (x, y, w, h), (row, col, total) in zip(tiles, prof):
            m = tile_weight(x, y, tiles)
            assert torch.equal(m[h // 2], row) and torch.equal(m[:, w // 2], col)
            assert abs(m.double().sum().item() - total) < 1e-6


def test_limits_match_reference(gold):
    for (fb, nf), lim in gold["limits"].items():
        assert _limits_for_free_bytes(fb, nf) == lim


def test_render_calls_match_reference(gold):
    C, F, H, W = gold["render_seed_canvas_shape"]
    canvas = torch.rand(C, F, H, W, generator=torch.Generator().manual_seed(5)) * 2 - 1
    calls = []

    def fake_pipe(LQ_video, num_frames, height, width, **kw):
        calls.append((height, width, num_frames, kw.get("topk_ratio")))
        return LQ_video

    out = render_tiled(fake_pipe, canvas, num_frames=3, prompt="", topk_ratio=0.5,
                       tile_threshold=300_000, tile_target=300_000, device="cpu")
    assert plan_tiles(W, H, target=300_000, threshold=300_000) == gold["render_plan"]
    assert calls == gold["render_calls"]
    assert (out - canvas).abs().max().item() <= max(gold["render_maxdiff"], 1e-6) * 4
