"""Batched-prefill causal attention (yb_prefill_attention_dev, the tensor-core kernel yb_prefill runs
per layer) against yalm's attention arithmetic (src/infer.cpp:218-250: s = q.k / sqrt(head_dim),
softmax over slots 0..pos, out = sum p v) restated in numpy fp64, per token, for every head-group
size the kernel is built for, both head dims, prompts that start at slot 0 and prompts appended to
a cache that already holds earlier slots, and prompt lengths that are not multiples of the tiles."""
import ctypes

import numpy as np
import pytest

from yalm_b200 import _lib

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _reference(q, k, v, T, pos0, nh, nkv, hd):
    gq = nh // nkv
    out = np.zeros((T, nh, hd))
    kf, vf = k.astype(np.float64), v.astype(np.float64)
    for t in range(T):
        n = pos0 + t + 1
        for h in range(nh):
            g = h // gq
            s = kf[g, :n] @ q[t, h].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[t, h] = p @ vf[g, :n] / p.sum()
    return out


@pytest.mark.parametrize("nh,nkv,hd,msl,T,pos0", [
    (8, 2, 64, 512, 100, 0), (8, 4, 64, 256, 33, 0), (32, 8, 128, 1024, 300, 0), (32, 8, 128, 1024, 77, 50),
    (64, 8, 128, 512, 130, 0), (16, 16, 128, 256, 65, 3), (8, 8, 64, 128, 1, 0), (32, 8, 128, 4096, 17, 4000)])
def test_prefill_attention_matches_reference(gpu, nh, nkv, hd, msl, T, pos0):
    import torch
    rng = np.random.default_rng(T + 7 * nh + pos0)
    q = rng.standard_normal((T, nh, hd)).astype(np.float32)
    k = rng.standard_normal((nkv, msl, hd)).astype(np.float16)
    v = rng.standard_normal((nkv, msl, hd)).astype(np.float16)
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(k.view(np.int16)).cuda()
    dv = torch.from_numpy(v.view(np.int16)).cuda()
    out = torch.zeros(T * nh * hd, dtype=torch.int16, device="cuda")
    _lib.call("yb_prefill_attention_dev", _ptr(out), _ptr(dq), _ptr(dk), _ptr(dv), T, pos0, nh, nkv, hd, msl, None)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.float16).astype(np.float64).reshape(T, nh, hd)
    ref = _reference(q, k, v, T, pos0, nh, nkv, hd)
    # the outputs are stored as fp16: half an fp16 ulp of |ref| plus the fp32-path rounding
    err = np.abs(got - ref) - (2.0 ** -11 * np.abs(ref) + 2e-4)
    assert err.max() <= 0, float(np.abs(got - ref).max())


@pytest.mark.parametrize("nh,nkv,hd,msl,T,pos0", [(32, 8, 128, 512, 77, 50), (8, 2, 64, 256, 33, 10)])
def test_prefill_attention_ignores_slots_past_the_prompt(gpu, nh, nkv, hd, msl, T, pos0):
    """Cache slots past the last query's position hold NaN (never-written cache memory may hold any
    bits): the kernel stages whole key tiles, and the slots past the causal range must contribute
    nothing — a zero probability times a NaN value would poison the row."""
    import torch
    rng = np.random.default_rng(11 * T + pos0)
    q = rng.standard_normal((T, nh, hd)).astype(np.float32)
    k = rng.standard_normal((nkv, msl, hd)).astype(np.float16)
    v = rng.standard_normal((nkv, msl, hd)).astype(np.float16)
    k[:, pos0 + T:] = np.nan
    v[:, pos0 + T:] = np.nan
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(k.view(np.int16)).cuda()
    dv = torch.from_numpy(v.view(np.int16)).cuda()
    out = torch.zeros(T * nh * hd, dtype=torch.int16, device="cuda")
    _lib.call("yb_prefill_attention_dev", _ptr(out), _ptr(dq), _ptr(dk), _ptr(dv), T, pos0, nh, nkv, hd, msl, None)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.float16).astype(np.float64).reshape(T, nh, hd)
    assert np.isfinite(got).all()
    ref = _reference(q, k, v, T, pos0, nh, nkv, hd)
    err = np.abs(got - ref) - (2.0 ** -11 * np.abs(ref) + 2e-4)
    assert err.max() <= 0, float(np.abs(got - ref).max())
