"""yb_attention_dev_noalloc — attention for callers that must not allocate device memory at call
time (a plugin inside a framework whose allocator owns the device memory, a serving loop that
forbids allocation after start-up).  Checked through the C ABI against yb_attention_dev, which takes
a caller-allocated scratch buffer, on two calls in a row (the library's fixed scratch array keeps the
previous call's contents, so the second call checks it is reused correctly), and against the CPU
oracle of yalm's attention.  Kept in a file of its own that pytest collects last; it passes alone in
a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest

import oracle
from yalm_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 2e-5  # the attention parity tolerance of tests/test_kernels_gpu.py


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(nh, nkv, hd, msl, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(nh * hd, device="cuda", generator=g)
    k = torch.randn(nkv, msl, hd, device="cuda", generator=g).half()
    v = torch.randn(nkv, msl, hd, device="cuda", generator=g).half()
    return q, k, v


def _allocating(q, k, v, nh, nkv, hd, msl, kv_len):
    import torch
    scratch = torch.zeros(_lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl), dtype=torch.uint8, device="cuda")
    ref = torch.zeros(nh * hd, device="cuda")
    _lib.call("yb_attention_dev", _p(ref), _p(q), _p(k), _p(v), nh, nkv, hd, msl, kv_len, _p(scratch), None)
    torch.cuda.synchronize()
    return ref.cpu().numpy()


def _noalloc(q, k, v, nh, nkv, hd, msl, kv_len):
    import torch
    out = torch.full((nh * hd,), float("nan"), device="cuda")
    _lib.call("yb_attention_dev_noalloc", _p(out), _p(q), _p(k), _p(v), nh, nkv, hd, msl, kv_len, None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _oracle(q, k, v, nh, nkv, hd, msl, kv_len):
    """yalm's attention (src/infer.cpp:394-415) restated in oracle/yalm_oracle.c."""
    kc = k.cpu().numpy().view(np.uint16)[:, :kv_len]
    vc = v.cpu().numpy().view(np.uint16)[:, :kv_len]
    kb, vb = oracle.to_ref_kv_layout(kc, vc, msl)
    return oracle.mha(q.cpu().numpy(), kb, vb, hd, kv_len, msl, nh, nkv)


@pytest.mark.parametrize("nh,nkv,hd,msl,kv_len", [(32, 8, 128, 4096, 3232), (8, 2, 64, 1024, 65),
                                                  (32, 8, 128, 4096, 1), (64, 8, 128, 8192, 1152),
                                                  (8, 2, 128, 8192, 6000), (4, 1, 128, 32768, 30000)])
def test_noalloc_attention_matches_allocating_entry_point(gpu, nh, nkv, hd, msl, kv_len):
    q, k, v = _inputs(nh, nkv, hd, msl, kv_len + nh)
    exp = _allocating(q, k, v, nh, nkv, hd, msl, kv_len)
    cpu = _oracle(q, k, v, nh, nkv, hd, msl, kv_len)
    for call in range(2):
        got = _noalloc(q, k, v, nh, nkv, hd, msl, kv_len)
        assert np.isfinite(got).all(), call
        assert np.allclose(got, exp, rtol=RTOL, atol=ATOL), (call, np.abs(got - exp).max())
        assert np.allclose(got, cpu, rtol=RTOL, atol=ATOL), (call, np.abs(got - cpu).max())


def test_noalloc_attention_shape_changes_reuse_the_array(gpu):
    """Shape A, then B, then A again, both long caches of two kv heads, whose clusters merge through
    the array: B's cluster records take more of it than A's, so the place of A's merge counters lies
    inside B's records and holds B's data when A runs again.  Each call must clear what it needs and
    give the allocating entry point's result."""
    shapes = [(8, 2, 128, 32768, 20000), (16, 2, 128, 32768, 30000), (8, 2, 128, 32768, 20000)]
    sizes = [_lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl) for nh, nkv, hd, msl, _ in shapes]
    assert sizes[1] > sizes[0]
    for i, (nh, nkv, hd, msl, kv_len) in enumerate(shapes):
        q, k, v = _inputs(nh, nkv, hd, msl, 100 + i)
        exp = _allocating(q, k, v, nh, nkv, hd, msl, kv_len)
        got = _noalloc(q, k, v, nh, nkv, hd, msl, kv_len)
        assert np.allclose(got, exp, rtol=RTOL, atol=ATOL), (i, np.abs(got - exp).max())


def test_noalloc_attention_rejects_oversized_shapes(gpu):
    import torch
    # needs 64 kv heads * 31 clusters * 8 heads * (128 + 2) floats * 4 bytes of records > 4 MiB
    nh, nkv, hd, msl = 512, 64, 128, 4096
    assert _lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl) > (4 << 20)
    q = torch.zeros(nh * hd, device="cuda")
    kv = torch.zeros(1, dtype=torch.float16, device="cuda")
    out = torch.zeros(nh * hd, device="cuda")
    rc = _lib.lib().yb_attention_dev_noalloc(_p(out), _p(q), _p(kv), _p(kv), nh, nkv, hd, msl, 100, None)
    assert rc == _lib.YB_E_INVALID
    assert "exceeds" in _lib.last_error()
