"""Pin the CPU oracle against fixtures produced by running the reference itself
(tests/golden/make_golden.py): FP8Linear / torch._scaled_mm, lcsa/reference.py,
build_csr.  CPU only."""
import os

import pytest
import torch

from oracle import ops as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return torch.load(os.path.join(GOLD, name), weights_only=False)


@pytest.mark.parametrize("case", ["bf16w", "f32w"])
def test_fp8_weight_quant_matches_reference(case):
    g = load("fp8_linear.pt")[case]
    q, s = O.fp8_weight(g["w"], "tensor")
    assert torch.equal(q.view(torch.uint8), g["w8"])
    assert torch.equal(s.reshape(()), g["w_scale"].reshape(()))


@pytest.mark.parametrize("case", ["bf16w", "f32w"])
def test_fp8_mm_matches_reference_scaled_mm(case):
    """The restated _mm reproduces torch._scaled_mm (as the reference calls it) bit for bit."""
    g = load("fp8_linear.pt")[case]
    y = O.fp8_mm(g["x8"].view(torch.float8_e4m3fn), g["x_scale"], g["w8"].view(torch.float8_e4m3fn),
                 g["w_scale"], g["b"].to(torch.bfloat16) if g["b"].dtype != torch.bfloat16 else g["b"])
    if g["b"].dtype == torch.bfloat16:
        assert torch.equal(y, g["y"])
    else:  # fp32 bias: the reference output keeps the bias dtype path of _scaled_mm
        assert (y.float() - g["y"].float()).abs().max().item() <= 2 ** -7 * g["y"].float().abs().max().item()


@pytest.mark.parametrize("case", ["bf16w", "f32w"])
def test_eager_activation_quant_branch(case):
    """fp8_linear.py:38-40 (non-contiguous inputs): amax of a bf16 tensor stays bf16, so the
    eager scale is bf16(amax/448) and the codes are e4m3(bf16(x/s)).  The kernel path
    (fp8_quant.py:25-35, what the oracle and the B200 kernels follow) keeps the scale in
    fp32 and rounds the codes once; the two agree to one code."""
    g = load("fp8_linear.pt")[case]
    x = g["x"]
    s = (x.abs().amax() / O.FP8_MAX).clamp(min=1e-12).float()
    eager = (x / s).to(torch.float8_e4m3fn)
    assert torch.equal(eager.view(torch.uint8), g["x8"])
    assert torch.equal(s.reshape(()), g["x_scale"].reshape(()))
    q, sk = O.quantize_fp8(x, "tensor")
    assert sk.to(torch.bfloat16).float().item() == g["x_scale"].item()
    d = (q.view(torch.uint8).to(torch.int16) - g["x8"].to(torch.int16)).abs()
    assert (q.float() - eager.float()).abs().max().item() <= 32  # one e4m3 step at |v| <= 448
    assert (d > 0).float().mean().item() < 0.5


@pytest.mark.parametrize("case", ["a", "b"])
def test_lcsa_oracle_matches_reference(case):
    g = load("lcsa.pt")[case]
    f, h, w = g["fhw"]
    H = g["H"]
    C = g["q"].shape[-1]
    q_w = O.window_partition(g["q"].view(1, f, h, w, C))
    assert torch.equal(q_w, g["q_w"])
    k_w = O.window_partition(g["k"].view(1, f, h, w, C))
    v_w = O.window_partition(g["v"].view(1, f, h, w, C))
    local = O.local_block_mask(h // 8, w // 8, g["rng"])
    assert torch.equal(local, g["local"])
    keep = O.draft_block_mask(q_w, k_w, H, f // 2, local, g["topk"])
    assert torch.equal(keep, g["keep"])
    att = O.sparse_attention(q_w, k_w, v_w, keep)
    assert torch.equal(att.to(torch.bfloat16), g["att"])
    assert abs(att.double().sum().item() - g["att_sum"]) <= 1e-6 * max(1.0, abs(g["att_sum"]))
    sel, cnt = O.build_csr(keep)
    assert torch.equal(cnt, g["cnt"])
    assert torch.equal(sel[..., :g["maxk"]], g["sel"])


@pytest.mark.parametrize("case", ["a", "b"])
def test_online_attention_order_matches_reference(case):
    """The kernel-order restatement (bf16 P, online softmax) agrees with the reference's fp32
    oracle at the reference test's tolerance (lcsa/test_correctness.py:59)."""
    g = load("lcsa.pt")[case]
    f, h, w = g["fhw"]
    C = g["q"].shape[-1]
    k_w = O.window_partition(g["k"].view(1, f, h, w, C))
    v_w = O.window_partition(g["v"].view(1, f, h, w, C))
    on = O.sparse_attention_online(g["q_w"], k_w, v_w, g["keep"])
    assert torch.allclose(on, g["att"].float(), atol=1e-2, rtol=1e-2)


def test_window_reverse_roundtrip():
    x = torch.randn(1, 4, 16, 24, 8)
    xw = O.window_partition(x)
    assert torch.equal(O.window_reverse(xw, (2, 8, 8), (4, 16, 24)), x)


def test_causal_rule_counts():
    """Benchmark keep rule: Nq=132 (2 rows of 66) -> 12*(66*66 + 66*82) kept pairs."""
    g = torch.Generator().manual_seed(0)
    q_w = torch.randn(132, 128, 1536, generator=g).to(torch.bfloat16)
    keep = O.causal_topk_mask(q_w, q_w, 12, 66, 0.25)
    assert keep.sum().item() == 117_216
    assert not keep[:, :66, 66:].any()  # never a future row


def test_quantize_formula_edges():
    x = torch.tensor([[0.0, 1.0, -448.0 * 3, 2.0 ** -20]], dtype=torch.bfloat16)
    q, s = O.quantize_fp8(x, "tensor")
    assert s.item() == pytest.approx(3.0, rel=0, abs=0)
    assert q.float()[0, 2].item() == -448.0
    z, sz = O.quantize_fp8(torch.zeros(2, 4, dtype=torch.bfloat16), "token")
    assert z.float().abs().max().item() == 0 and sz.abs().max().item() == 0
    e, se = O.quantize_fp8(torch.zeros(0, 4, dtype=torch.bfloat16), "tensor")
    assert e.numel() == 0 and se.item() == 0
