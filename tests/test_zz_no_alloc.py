"""fvb_quant_fp8_tensor_noalloc: the per-tensor FP8 quantiser for callers that cannot
allocate device memory (an FFI host passing only pointers, a process whose device memory
belongs to another framework's pool, a loop that must avoid cudaMalloc's synchronisation).
Its reduction scratch is a fixed device array inside the library instead of a
caller-provided workspace.

Checked through the C ABI against the regular fvb_quant_fp8 (per-tensor, with a
workspace) on two calls in a row: codes and scale must be identical, which is this
suite's bar for FP8 quantisation.  The second call is smaller than the first, so stale
scratch from the first call must not leak into it.  Collected last (file name) so a run
that stops at the first failure has run everything else first; it also passes alone in a
fresh process.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _regular(lib, x, stream):
    from flashvsr_sm89_ops_b200 import _lib
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    ws = torch.empty(64, dtype=torch.float32, device=x.device)
    rc = lib.fvb_quant_fp8(x.data_ptr(), M, K, q.data_ptr(), s.data_ptr(), _lib.FVB_SCALE_TENSOR,
                           ws.data_ptr(), stream)
    assert rc == _lib.FVB_OK, lib.fvb_last_error()
    return q, s


def _noalloc(lib, x, stream):
    from flashvsr_sm89_ops_b200 import _lib
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    rc = lib.fvb_quant_fp8_tensor_noalloc(x.data_ptr(), M, K, q.data_ptr(), s.data_ptr(), stream)
    assert rc == _lib.FVB_OK, lib.fvb_last_error()
    return q, s


def test_noalloc_matches_regular_entry_point_twice():
    from flashvsr_sm89_ops_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator().manual_seed(11)
    big = torch.randn(4224, 1536, generator=g)
    big[torch.rand(big.shape, generator=g) < 0.01] *= 20
    small = (torch.randn(333, 1000, generator=g) * 0.5).to(torch.bfloat16)  # ragged: 333000 % 8 == 0
    tail = torch.randn(7, 13, generator=g).to(torch.bfloat16)               # n % 8 != 0
    nan = torch.randn(2555, generator=g).to(torch.bfloat16)  # 2555 % 8 == 3
    nan[123] = float("nan")   # a NaN stays NaN (clamp-then-cast keeps it): vector part
    nan[2553] = float("nan")  # ... and in the scalar tail
    nan = nan.reshape(511, 5)
    for x in (big.to(torch.bfloat16), small, tail, nan):
        xd = x.to(dev)
        qr, sr = _regular(lib, xd, stream)
        qn, sn = _noalloc(lib, xd, stream)
        torch.cuda.synchronize(dev)
        assert torch.equal(qn.view(torch.uint8), qr.view(torch.uint8))
        assert torch.equal(sn, sr) or (torch.isnan(sn).all() and torch.isnan(sr).all())
    assert _lib.device_error() == 0


def test_noalloc_rejects_oversize_and_handles_empty():
    from flashvsr_sm89_ops_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev).cuda_stream
    s = torch.full((1,), 7.0, device=dev)
    # 2^31 elements > the 2^30-element limit: rejected on the host before any device work
    rc = lib.fvb_quant_fp8_tensor_noalloc(None, 1 << 20, 1 << 11, None, s.data_ptr(), stream)
    assert rc == _lib.FVB_ERR_INVALID
    assert b"scratch limit" in lib.fvb_last_error()
    # 2^32 x 2^32 would overflow int64 if multiplied before the check
    rc = lib.fvb_quant_fp8_tensor_noalloc(None, 1 << 32, 1 << 32, None, s.data_ptr(), stream)
    assert rc == _lib.FVB_ERR_INVALID
    assert b"scratch" in lib.fvb_last_error()
    rc = lib.fvb_quant_fp8_tensor_noalloc(None, 0, 1536, None, s.data_ptr(), stream)
    assert rc == _lib.FVB_OK
    torch.cuda.synchronize(dev)
    assert s.item() == 0.0
