"""Kernel-level parity on the GPU: every decode kernel through the C ABI against the CPU oracle
(oracle/yalm_oracle.c, pinned to yalm's own CPU path in test_oracle.py), on seeded inputs, with
edge shapes (odd row counts, columns not a multiple of 256, kv_len 1 / 31 / 33 / 65 / 129)."""
import ctypes

import numpy as np
import pytest

import oracle
from yalm_b200 import _lib

pytestmark = pytest.mark.gpu


_ALIVE = []


def _t(a):
    """Device copy of a numpy array, kept alive until the test module ends (a temporary freed while
    its kernel is still queued would be handed to the next allocation by torch's caching allocator)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _ALIVE.append(t)
    return t


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    import torch
    torch.cuda.synchronize()
    _ALIVE.clear()


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _sync():
    import torch
    torch.cuda.synchronize()


def _tol(w16, x):
    """Reassociation bound for an fp32 dot product: a small multiple of sum |w| |x|."""
    w = w16.view(np.float16).astype(np.float64)
    return 2e-6 * np.abs(w) @ np.abs(x.astype(np.float64)) * np.sqrt(w.shape[1] / 64) + 1e-7


@pytest.mark.parametrize("rows,cols", [(33, 512), (768, 512), (512, 1408), (4096, 4096), (4096, 14336),
                                       (2047, 4096), (1000, 7168), (96, 28672 // 2)])
def test_gemv_matches_oracle(gpu, rows, cols):
    import torch
    rng = np.random.default_rng(rows * 7 + cols)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    dw, dx = _t(w), _t(x)
    _lib.call("yb_gemv_dev", _ptr(y), _ptr(dx), _ptr(dw), rows, cols, None, 0.0, 0, None)
    _sync()
    ref = oracle.matmul_f16(x, w)
    got = y.cpu().numpy()
    assert np.all(np.abs(got - ref) <= _tol(w, x)), np.abs(got - ref).max()
    # accumulate mode: y += W x
    base = rng.standard_normal(rows).astype(np.float32)
    y2 = _t(base)
    _lib.call("yb_gemv_dev", _ptr(y2), _ptr(dx), _ptr(dw), rows, cols, None, 0.0, 1, None)
    _sync()
    assert np.all(np.abs(y2.cpu().numpy() - (base + ref)) <= _tol(w, x) + 1e-6)


@pytest.mark.parametrize("accumulate", [0, 1])
def test_gemv_column_panels_70b_w2(gpu, accumulate):
    """The 70B-class w2 (dim 8192 x hidden 28672): rows wider than one kernel covers run as two
    14336-column panels with the full row stride, the second accumulating onto the first — the same
    kernel instance and strides the engine launches for config 5's w2."""
    import torch
    rows, cols = 8192, 28672
    rng = np.random.default_rng(70)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(cols).astype(np.float32)
    base = rng.standard_normal(rows).astype(np.float32)
    y = _t(base) if accumulate else torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    _lib.call("yb_gemv_dev", _ptr(y), _ptr(_t(x)), _ptr(_t(w)), rows, cols, None, 0.0, accumulate, None)
    _sync()
    ref = oracle.matmul_f16(x, w) + (base if accumulate else 0)
    assert np.all(np.abs(y.cpu().numpy() - ref) <= _tol(w, x) + 1e-6), np.abs(y.cpu().numpy() - ref).max()


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (32000, 4096), (4096, 512), (6, 8192)])
def test_gemv_rmsnorm_prologue(gpu, rows, cols):
    import torch
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16).view(np.uint16)
    x = (rng.standard_normal(cols) * 3).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    _lib.call("yb_gemv_dev", _ptr(y), _ptr(_t(x)), _ptr(_t(w)), rows, cols, _ptr(_t(nw)), 1e-5, 0, None)
    _sync()
    xn = oracle.rmsnorm(x, nw, 1e-5)
    ref = oracle.matmul_f16(xn, w)
    assert np.all(np.abs(y.cpu().numpy() - ref) <= 2 * _tol(w, xn) + 1e-6)


@pytest.mark.parametrize("hidden,dim,act", [(1408, 512, 1), (14336, 4096, 1), (256, 256, 0), (1792, 4096, 1)])
def test_gateup_swiglu(gpu, hidden, dim, act):
    import torch
    rng = np.random.default_rng(hidden + dim)
    w1 = (rng.standard_normal((hidden, dim)) * 0.02).astype(np.float16).view(np.uint16)
    w3 = (rng.standard_normal((hidden, dim)) * 0.02).astype(np.float16).view(np.uint16)
    w13 = np.empty((2 * hidden, dim), np.uint16)
    w13[0::2], w13[1::2] = w1, w3
    x = rng.standard_normal(dim).astype(np.float32)
    nw = np.ones(dim, np.float32)
    hb = torch.zeros(hidden, dtype=torch.float32, device="cuda")
    _lib.call("yb_gateup_dev", _ptr(hb), _ptr(_t(x)), _ptr(_t(w13)), hidden, dim, _ptr(_t(nw)), 1e-5, act, None)
    _sync()
    xn = oracle.rmsnorm(x, nw, 1e-5)
    g, u = oracle.matmul_f16(xn, w1), oracle.matmul_f16(xn, w3)
    if act == 1:
        ref = g / (1 + np.exp(-g.astype(np.float64))) * u
    else:
        ref = 0.5 * g * (1 + np.tanh(0.797885 * (g + 0.044715 * g ** 3))) * u
    assert np.allclose(hb.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)


def _inv_freq(head_dim, rotary_dim, theta):
    """1 / powf(theta, j / rotary_dim) with the C library's powf, as yalm and the oracle compute it
    (src/infer.cpp:205); numpy's float32 power can differ by an ulp, which at position 3000 moves
    the RoPE angle by ~1e-4 rad."""
    libm = ctypes.CDLL("libm.so.6")
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    out = []
    for j in range(0, head_dim, 2):
        if j >= rotary_dim:
            out.append(0.0)
        else:
            e = np.float32(j) / np.float32(rotary_dim)
            out.append(np.float32(1.0) / np.float32(libm.powf(np.float32(theta), e)))
    return np.array(out, np.float32)


@pytest.mark.parametrize("nh,nkv,hd,dim,pos,msl", [(8, 2, 64, 512, 5, 64), (32, 8, 128, 4096, 3000, 4096),
                                                  (8, 2, 64, 512, 200, 64)])
def test_qkv_rope_kv_append(gpu, nh, nkv, hd, dim, pos, msl):
    """q -> fp32 (clip + RoPE), k/v -> fp16 cache slot kv_pos; sinks re-rotated past the context."""
    import torch
    from yalm_b200.model import positions
    rng = np.random.default_rng(pos + hd)
    rows = (nh + 2 * nkv) * hd
    w = (rng.standard_normal((rows, dim)) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(dim).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    theta = 1e6
    kv_sink, kv_pos, kv_len = positions(pos, msl)
    kc0 = (rng.standard_normal((nkv, msl, hd)) * 0.5).astype(np.float16).view(np.uint16)
    vc0 = (rng.standard_normal((nkv, msl, hd)) * 0.5).astype(np.float16).view(np.uint16)
    q = torch.zeros(nh * hd, dtype=torch.float32, device="cuda")
    kc, vc = _t(kc0), _t(vc0)
    inv = _inv_freq(hd, hd, theta)
    clip = 0.05  # small enough to bite
    _lib.call("yb_qkv_dev", _ptr(q), _ptr(kc), _ptr(vc), _ptr(_t(x)), _ptr(_t(w)), _ptr(_t(nw)), 1e-5, dim, nh, nkv, hd,
              hd, msl, pos, kv_pos, kv_sink, clip, _ptr(_t(inv)), None)
    _sync()
    xn = oracle.rmsnorm(x, nw, 1e-5)
    out = np.clip(oracle.matmul_f16(xn, w), -clip, clip)
    qr = oracle.rope(out[:nh * hd], hd, pos, theta, hd)
    kr = oracle.rope(out[nh * hd:(nh + nkv) * hd], hd, pos, theta, hd)
    vr = out[(nh + nkv) * hd:]
    assert np.allclose(q.cpu().numpy(), qr, rtol=1e-4, atol=2e-6)
    kc1, vc1 = kc.cpu().numpy(), vc.cpu().numpy()
    kexp = kc0.copy()
    vexp = vc0.copy()
    kexp[:, kv_pos, :] = oracle.f2h(kr.reshape(nkv, hd))
    vexp[:, kv_pos, :] = oracle.f2h(vr.reshape(nkv, hd))
    for r in range(kv_sink):  # src/infer.cpp:311-325
        for g in range(nkv):
            kexp[g, r] = oracle.f2h(oracle.rope(oracle.h2f(kc0[g, r]), hd, 1, theta, hd))
    # untouched slots are bit-identical; written slots agree to within one fp16 ulp
    touched = np.zeros(msl, bool)
    touched[kv_pos] = True
    touched[:kv_sink] = True
    assert np.array_equal(kc1[:, ~touched], kc0[:, ~touched]) and np.array_equal(vc1[:, ~touched], vc0[:, ~touched])
    for got, exp in ((kc1[:, touched], kexp[:, touched]), (vc1[:, touched], vexp[:, touched])):
        d = np.abs(oracle.h2f(got) - oracle.h2f(exp))
        ulp = np.abs(oracle.h2f(exp)) * 2.0 ** -10 + 2.0 ** -24
        assert np.all(d <= ulp * 1.01), d.max()


@pytest.mark.parametrize("pos,msl", [(0, 64), (17, 64), (63, 64), (64, 64), (65, 64), (200, 64), (1000, 64)])
def test_kv_append_indexing_integer_coded(gpu, pos, msl):
    """Bit-exact KV indexing: W has one non-zero column, so row r of [q;k;v] equals code(r) exactly
    (small integers are exact in fp16); RoPE is off (rotary_dim 0) and x is a unit vector."""
    import torch
    from yalm_b200.model import positions
    nh, nkv, hd, dim = 4, 2, 64, 64
    rows = (nh + 2 * nkv) * hd
    codes = np.arange(rows, dtype=np.float32) % 1000 + 1  # exact in fp16
    w = np.zeros((rows, dim), np.float16)
    w[:, 0] = codes
    w = w.view(np.uint16)
    x = np.zeros(dim, np.float32)
    x[0] = 1.0
    kv_sink, kv_pos, _ = positions(pos, msl)
    kc = torch.zeros((nkv, msl, hd), dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    q = torch.zeros(nh * hd, dtype=torch.float32, device="cuda")
    inv = np.zeros(hd // 2, np.float32)
    _lib.call("yb_qkv_dev", _ptr(q), _ptr(kc), _ptr(vc), _ptr(_t(x)), _ptr(_t(w)), None, 1e-5, dim, nh, nkv, hd, 0,
              msl, pos, kv_pos, kv_sink, float(np.finfo(np.float32).max), _ptr(_t(inv)), None)
    _sync()
    k = kc.cpu().numpy().view(np.uint16)
    v = vc.cpu().numpy().view(np.uint16)
    assert np.array_equal(q.cpu().numpy(), codes[:nh * hd])
    kexp = np.zeros_like(k)
    vexp = np.zeros_like(v)
    kexp[:, kv_pos] = codes[nh * hd:(nh + nkv) * hd].astype(np.float16).view(np.uint16).reshape(nkv, hd)
    vexp[:, kv_pos] = codes[(nh + nkv) * hd:].astype(np.float16).view(np.uint16).reshape(nkv, hd)
    assert np.array_equal(k, kexp) and np.array_equal(v, vexp)


@pytest.mark.parametrize("nh,nkv,hd,msl,kv_len", [
    (8, 2, 64, 1024, 1), (8, 2, 64, 1024, 2), (8, 2, 64, 1024, 31), (8, 2, 64, 1024, 33), (8, 2, 64, 1024, 96),
    (32, 8, 128, 4096, 1), (32, 8, 128, 4096, 65), (32, 8, 128, 4096, 129), (32, 8, 128, 4096, 3232),
    (32, 8, 128, 4096, 4096), (64, 8, 128, 8192, 1152), (16, 16, 128, 512, 300), (16, 8, 64, 512, 511),
    (32, 8, 128, 32768, 16384), (32, 8, 128, 32768, 32768), (8, 2, 128, 8192, 8192), (4, 1, 128, 16384, 16000),
    (8, 1, 64, 4096, 2049), (64, 8, 128, 8192, 8192), (4, 1, 128, 32768, 30000), (8, 2, 128, 32768, 32768),
    # one tensor-parallel rank's share of the 7B shape (2, 4, 8 ranks) at the scaling bench's kv_len
    (16, 4, 128, 4096, 100), (8, 2, 128, 4096, 136), (4, 1, 128, 4096, 17), (4, 1, 128, 4096, 129)])
def test_attention_matches_oracle(gpu, nh, nkv, hd, msl, kv_len):
    """Includes config 4's long caches (kv_len 16384 and 32768 at max_seq_len 32768: over 3000 slots
    per CTA of a 10-CTA cluster on a B200) and long caches of one or two kv heads, which several
    clusters per kv
    head share and merge through the scratch records."""
    import torch
    rng = np.random.default_rng(kv_len + nh)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal((nkv, msl, hd), dtype=np.float32).astype(np.float16).view(np.uint16)
    v = rng.standard_normal((nkv, msl, hd), dtype=np.float32).astype(np.float16).view(np.uint16)
    nbytes = _lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl)
    assert nbytes > 0
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    out = torch.zeros(nh * hd, dtype=torch.float32, device="cuda")
    dq, dk, dv = _t(q), _t(k), _t(v)
    for _ in range(2):  # the second call checks the scratch counters were left at zero
        _lib.call("yb_attention_dev", _ptr(out), _ptr(dq), _ptr(dk), _ptr(dv), nh, nkv, hd, msl, kv_len,
                  _ptr(scratch), None)
        _sync()
        kb, vb = oracle.to_ref_kv_layout(k[:, :kv_len], v[:, :kv_len], msl)
        ref = oracle.mha(q, kb, vb, hd, kv_len, msl, nh, nkv)
        assert np.allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=2e-5), np.abs(out.cpu().numpy() - ref).max()


def test_reference_test_hooks(gpu):
    """yb_matmul / yb_mha / yb_ffn take the same arguments as yalm's matmul_cuda / mha_cuda /
    ffn_cuda test hooks (src/test.cpp:147-233 shapes: head_dim 16 x 16 heads, 8 kv heads, seq 4)
    and agree with the reference CPU hooks."""
    L = _lib.lib()
    rng = np.random.default_rng(0)
    head_dim, n_heads, n_kv, msl, kv_len = 16, 16, 8, 4, 4
    dim = head_dim * n_heads
    # matmul
    w = (rng.standard_normal((head_dim, dim))).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(dim).astype(np.float32)
    out = np.zeros(head_dim, np.float32)
    _lib.check(L.yb_matmul(out.ctypes.data, x.ctypes.data, w.ctypes.data, dim, head_dim))
    ref = np.zeros(head_dim, np.float32)
    oracle.ref_lib().ref_matmul_f16(ref.ctypes.data, x.ctypes.data, w.ctypes.data, dim, head_dim)
    assert np.allclose(out, ref, atol=1e-4)
    # ffn (fp16 weights, GELU as in the reference test)
    w1 = (rng.standard_normal((dim, dim)) / np.sqrt(dim)).astype(np.float16).view(np.uint16)
    w2 = (rng.standard_normal((dim, dim)) / np.sqrt(dim)).astype(np.float16).view(np.uint16)
    w3 = (rng.standard_normal((dim, dim)) / np.sqrt(dim)).astype(np.float16).view(np.uint16)
    out = np.zeros(dim, np.float32)
    _lib.check(L.yb_ffn(out.ctypes.data, x.ctypes.data, w1.ctypes.data, w2.ctypes.data, w3.ctypes.data, dim, dim, 0))
    f = [oracle.h2f(m).reshape(dim, dim) for m in (w1, w2, w3)]
    ref = np.zeros(dim, np.float32)
    oracle.ref_lib().ref_ffn_f32(ref.ctypes.data, x.ctypes.data, *(np.ascontiguousarray(m).ctypes.data for m in f),
                                 dim, dim, 0)
    assert np.allclose(out, ref, atol=1e-4)
    # mha: head_dim 16 is not a decode shape of this engine -> clean error, never a crash
    kb = rng.standard_normal(msl * n_kv * head_dim).astype(np.float16).view(np.uint16)
    vb = rng.standard_normal(msl * n_kv * head_dim).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(n_heads * head_dim).astype(np.float32)
    out = np.zeros(n_heads * head_dim, np.float32)
    rc = L.yb_mha(out.ctypes.data, None, kb.ctypes.data, vb.ctypes.data, q.ctypes.data, head_dim, kv_len, msl,
                  n_heads, n_kv)
    assert rc == _lib.YB_E_UNSUPPORTED
    # the same hook at a supported head_dim
    hd = 64
    kb = rng.standard_normal(msl * n_kv * hd).astype(np.float16).view(np.uint16)
    vb = rng.standard_normal(msl * n_kv * hd).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(n_heads * hd).astype(np.float32)
    out = np.zeros(n_heads * hd, np.float32)
    _lib.check(L.yb_mha(out.ctypes.data, None, kb.ctypes.data, vb.ctypes.data, q.ctypes.data, hd, kv_len, msl,
                        n_heads, n_kv))
    ref = np.zeros(n_heads * hd, np.float32)
    att = np.zeros(n_heads * msl, np.float32)
    oracle.ref_lib().ref_mha(ref.ctypes.data, att.ctypes.data, kb.ctypes.data, vb.ctypes.data, q.ctypes.data, hd,
                             kv_len, msl, n_heads, n_kv)
    assert np.allclose(out, ref, atol=1e-4)
