"""yb_attention_dev_noalloc — attention for callers that must not allocate device memory at call
time (a plugin inside a framework whose allocator owns the device memory, a serving loop that
forbids allocation after start-up).  Checked through the C ABI against yb_attention_dev, which takes
a caller-allocated scratch buffer, on two calls in a row (the library's fixed scratch array keeps the
previous call's contents, so the second call checks it is reused correctly).  Kept in a file of its
own that pytest collects last; it passes alone in a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest

from yalm_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 2e-5  # the attention parity tolerance of tests/test_kernels_gpu.py


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("nh,nkv,hd,msl,kv_len", [(32, 8, 128, 4096, 3232), (8, 2, 64, 1024, 65),
                                                  (32, 8, 128, 4096, 1), (64, 8, 128, 8192, 1152)])
def test_noalloc_attention_matches_allocating_entry_point(gpu, nh, nkv, hd, msl, kv_len):
    import torch
    g = torch.Generator(device="cuda").manual_seed(kv_len + nh)
    q = torch.randn(nh * hd, device="cuda", generator=g)
    k = torch.randn(nkv, msl, hd, device="cuda", generator=g).half()
    v = torch.randn(nkv, msl, hd, device="cuda", generator=g).half()
    scratch = torch.zeros(_lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl), dtype=torch.uint8, device="cuda")
    ref = torch.zeros(nh * hd, device="cuda")
    _lib.call("yb_attention_dev", _p(ref), _p(q), _p(k), _p(v), nh, nkv, hd, msl, kv_len, _p(scratch), None)
    torch.cuda.synchronize()
    for call in range(2):
        out = torch.full((nh * hd,), float("nan"), device="cuda")
        _lib.call("yb_attention_dev_noalloc", _p(out), _p(q), _p(k), _p(v), nh, nkv, hd, msl, kv_len, None)
        torch.cuda.synchronize()
        got, exp = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(got).all(), call
        assert np.allclose(got, exp, rtol=RTOL, atol=ATOL), (call, np.abs(got - exp).max())


def test_noalloc_attention_rejects_oversized_shapes(gpu):
    import torch
    nh, nkv, hd, msl = 64, 8, 128, 32768  # needs 64 * 256 * 130 * 4 bytes of scratch > 4 MiB
    assert _lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl) > (4 << 20)
    q = torch.zeros(nh * hd, device="cuda")
    kv = torch.zeros(1, dtype=torch.float16, device="cuda")
    out = torch.zeros(nh * hd, device="cuda")
    rc = _lib.lib().yb_attention_dev_noalloc(_p(out), _p(q), _p(kv), _p(kv), nh, nkv, hd, msl, 100, None)
    assert rc == _lib.YB_E_INVALID
    assert "exceeds" in _lib.last_error()
