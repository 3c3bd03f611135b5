"""enable() wiring on CPU (no kernels run): flag handling, FP8 conversion counts, the
upstream-drift guard, idempotent re-enable, and the fused-QKV weight packing."""
import types

import pytest
import torch

from flashvsr_sm89_ops_b200 import wan_video_dit as W
from flashvsr_sm89_ops_b200.fp8_ffn import FP8FFN
from flashvsr_sm89_ops_b200.fp8_linear import FP8Linear
from flashvsr_sm89_ops_b200.integrate import _check_dit_structure, _qkv_pack, _row_maps, enable


def small_pipe(layers=2, dim=256, heads=2, ffn=512):
    dit = W.WanDiT(num_layers=layers, dim=dim, num_heads=heads, ffn_dim=ffn).to(torch.bfloat16)
    dit.init_random(seed=0)
    return W.DiTPipe(dit)


def test_enable_converts_and_patches(monkeypatch):
    monkeypatch.setenv("FS89_FP8_SCALE", "token")
    pipe = small_pipe()
    applied = enable(pipe, dit_module=W, verbose=False)
    assert applied["fp8_linears"] == 2 * 10 and applied["fp8_ffn_blocks"] == 2
    assert applied["fused_rope"] and applied["fused_adaln"] and applied["lcsa_backend"] == "b200"
    blk = pipe.dit.blocks[0]
    assert isinstance(blk.self_attn.q, FP8Linear) and isinstance(blk.ffn, FP8FFN)
    assert W._FS89_PATCHED and W.FUSED_ROPE_FN is not None
    again = enable(pipe, dit_module=W, verbose=False)  # idempotent
    assert again["fp8_linears"] == 0 and again["fp8_ffn_blocks"] == 0


def test_flags_turn_parts_off(monkeypatch):
    monkeypatch.setenv("FS89_FP8", "")
    monkeypatch.setenv("FS89_FUSED_ROPE", "0")
    monkeypatch.setenv("FS89_FUSED_ADALN", "0")
    pipe = small_pipe(layers=1)
    applied = enable(pipe, dit_module=W, verbose=False)
    assert "fp8_linears" not in applied
    assert W.FUSED_ROPE_FN is None and W.FUSED_ADALN is None
    monkeypatch.setenv("FS89_FUSED_ROPE", "1")
    monkeypatch.setenv("FS89_FUSED_ADALN", "1")
    enable(pipe, dit_module=W, verbose=False)
    assert W.FUSED_ROPE_FN is not None


def test_structure_guard():
    bad = types.ModuleType("bad_dit")
    with pytest.raises(RuntimeError, match="no SelfAttention"):
        _check_dit_structure(bad)

    class SelfAttention:
        def forward(self, x, freqs):
            pass

    bad.SelfAttention = SelfAttention
    with pytest.raises(RuntimeError, match="lacks args"):
        _check_dit_structure(bad)


def test_qkv_pack_is_exact_concatenation(monkeypatch):
    for mode in ("tensor", "token"):
        monkeypatch.setenv("FS89_FP8_SCALE", mode)
        pipe = small_pipe(layers=1)
        enable(pipe, dit_module=W, verbose=False)
        att = pipe.dit.blocks[0].self_attn
        _, Wq, S, Bv, m = _qkv_pack(att)
        D = att.q.out_features
        assert m == mode and Wq.shape == (3 * D, D) and S.shape == (3 * D,)
        for i, lin in enumerate((att.q, att.k, att.v)):
            assert torch.equal(Wq[i * D:(i + 1) * D].view(torch.uint8), lin.weight.view(torch.uint8))
            s = lin.w_scale.expand(D) if lin.w_scale.numel() == 1 else lin.w_scale
            assert torch.equal(S[i * D:(i + 1) * D], s)


def test_row_maps_invert_window_partition():
    from oracle import ops as O
    r2w, w2r = _row_maps(2, 16, 24, "cpu")
    idx = torch.arange(2 * 16 * 24).view(1, 2, 16, 24, 1)
    assert torch.equal(O.window_partition(idx).reshape(-1).int(), w2r)
    assert torch.equal(r2w[w2r.long()], torch.arange(2 * 16 * 24, dtype=torch.int32))


def test_forward_refuses_cpu(monkeypatch):
    monkeypatch.setenv("FS89_FP8_SCALE", "token")
    lin = torch.nn.Linear(32, 16).to(torch.bfloat16)
    fl = FP8Linear(lin)
    with pytest.raises(ValueError, match="CUDA"):
        fl(torch.zeros(2, 32, dtype=torch.bfloat16))


def test_kv_arena_reuses_only_unheld_windows():
    """The streaming KV arena (host-side bookkeeping, CPU tensors here): a new row goes right
    after the given cache when no live handed-out cache covers those windows; otherwise the
    cache is copied into a fresh arena, so a cache a caller still holds never changes."""
    import gc

    from flashvsr_sm89_ops_b200.integrate import _arena_slot
    D, row = 8, 2  # 8 channels, 2 windows per time row
    cpu = torch.device("cpu")
    ar, a, b = _arena_slot(None, 6, row, D, cpu)  # start chunk: 3 rows, no cache
    assert (a, b) == (0, 0) and ar.cap == 6 + 4 * row
    ar.rows(0, 6).copy_(torch.arange(6 * 128 * D, dtype=torch.float32).view(-1, D))
    c0 = ar.hand_out(0, 6)
    # a step given c0 appends in place after it
    ar1, a1, b1 = _arena_slot(c0, row, row, D, cpu)
    assert ar1 is ar and (a1, b1) == (0, 6)
    c1 = ar.hand_out(2, 8)  # the step's returned cache (oldest row dropped)
    # c1 is alive and covers windows [6, 8): the same step given c0 again must not reuse them
    ar2, a2, b2 = _arena_slot(c0, row, row, D, cpu)
    assert ar2 is not ar and (a2, b2) == (0, 6)
    assert torch.equal(ar2.rows(0, 6), c0.reshape(-1, D))
    # once c1 is gone the windows are free again
    del c1
    gc.collect()
    ar3, a3, b3 = _arena_slot(c0, row, row, D, cpu)
    assert ar3 is ar and (a3, b3) == (0, 6)
    # a real stream (each step gets the previous step's cache): 4 in-place appends fill the
    # 4 spare rows, the 5th step copies the cache into a new arena
    c, arenas = c0, []
    for _ in range(5):
        arx, ax, bx = _arena_slot(c, row, row, D, cpu)
        arenas.append(arx)
        c = arx.hand_out(ax + row, bx + row)
        assert c.shape[0] == 6  # always 3 time rows of 2 windows
    assert all(x is ar for x in arenas[:4]) and arenas[4] is not ar
    # a tensor that did not come from an arena is copied
    plain = torch.zeros(6, 128, D)
    arp, ap, bp = _arena_slot(plain, row, row, D, cpu)
    assert (ap, bp) == (0, 6) and torch.equal(arp.rows(0, 6), plain.reshape(-1, D))


def test_new_entry_points_refuse_cpu_tensors():
    """The fused gated norms, block pooling and the pooled keep rule follow the pack's
    contract for CPU tensors: ValueError naming CUDA, before any library call."""
    from flashvsr_sm89_ops_b200 import lcsa
    from flashvsr_sm89_ops_b200.fused_adaln import gate_add_layer_norm, gate_add_ln_modulate
    x = torch.zeros(1, 128, 64, dtype=torch.bfloat16)
    v = torch.zeros(1, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        gate_add_ln_modulate(x, v, x, v, v, emit_fp8=True)
    with pytest.raises(ValueError, match="CUDA"):
        gate_add_layer_norm(x, v, x, None, None)
    with pytest.raises(ValueError, match="CUDA"):
        lcsa.block_mean_pool(x.view(128, 64))
    with pytest.raises(ValueError, match="CUDA"):
        lcsa.causal_topk_mask(x.view(128, 64), x.view(128, 64), 1, 1, k_pool_prefix=None,
                              return_k_pool=True)
