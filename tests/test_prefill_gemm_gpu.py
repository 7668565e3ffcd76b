"""Batched-prefill tensor-core GEMM (tcgen05, yb_prefill_gemm_dev) against torch in fp32 on the same
fp16 inputs: C = A @ B^T with fp32 accumulation, every epilogue, tile tails in M and N, and the
prefill shapes of the 7B config; and the two-plane form the prefill runs (A as fp16 values plus
their fp16 remainders against an fp32 A, fp16 outputs with their remainders)."""
import ctypes

import numpy as np
import pytest

from yalm_b200 import _lib

pytestmark = pytest.mark.gpu

_ALIVE = []


def _p(t):
    _ALIVE.append(t)
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _run(M, N, K, epi, seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.randn(M, K, device="cuda", generator=g)).half()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    ref = A.float() @ B.float().T
    if epi in (0, 1):
        out = torch.randn(M, N, device="cuda", generator=g) if epi == 1 else torch.full((M, N), float("nan"), device="cuda")
        base = out.clone()
        _lib.call("yb_prefill_gemm_dev", _p(out), None, _p(A), _p(B), M, N, K, epi, N, None)
        exp = ref + base if epi == 1 else ref
        got = out
    elif epi == 2:
        out = torch.zeros(M, N // 2, dtype=torch.float16, device="cuda")
        _lib.call("yb_prefill_gemm_dev", None, _p(out), _p(A), _p(B), M, N, K, epi, N // 2, None)
        gt, up = ref[:, 0::2], ref[:, 1::2]
        exp = gt / (1 + torch.exp(-gt)) * up
        got = out.float()
    else:
        out = torch.zeros(M, N, dtype=torch.float16, device="cuda")
        _lib.call("yb_prefill_gemm_dev", None, _p(out), _p(A), _p(B), M, N, K, epi, N, None)
        exp, got = ref, out.float()
    torch.cuda.synchronize()
    return got.cpu().numpy(), exp.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (128, 256, 1024), (200, 520, 256), (1, 8, 64), (3202, 6144, 4096)])
def test_store_matches_fp32_reference(gpu, M, N, K):
    got, exp = _run(M, N, K, 0)
    assert np.isfinite(got).all()
    scale = np.abs(exp).max()
    assert np.abs(got - exp).max() <= 1e-4 * scale + 1e-5, np.abs(got - exp).max()


@pytest.mark.parametrize("epi", [1, 2, 3])
def test_epilogues(gpu, epi):
    got, exp = _run(300, 1024, 512, epi, seed=epi)
    tol = 2e-3 if epi in (2, 3) else 1e-4  # fp16 outputs round to 2^-11 relative
    assert np.allclose(got, exp, rtol=tol, atol=tol * np.abs(exp).max()), np.abs(got - exp).max()


def test_rejects_bad_shapes(gpu):
    import torch
    A = torch.zeros(64, 100, dtype=torch.float16, device="cuda")
    out = torch.zeros(64, 64, device="cuda")
    rc = _lib.lib().yb_prefill_gemm_dev(_p(out), None, _p(A), _p(A), 64, 64, 100, 0, 64, None)
    assert rc == _lib.YB_E_INVALID


def _split(x):
    """fp32 tensor -> [2][...] fp16 planes: the value rounded to fp16 and its fp16 remainder."""
    import torch
    hi = x.half()
    lo = (x - hi.float()).half()
    return torch.stack([hi, lo])


@pytest.mark.parametrize("M,N,K,epi", [(300, 1024, 512, 0), (3202, 6144, 4096, 0), (200, 520, 256, 1),
                                       (300, 1024, 512, 2), (257, 512, 1024, 3)])
def test_two_plane_activations(gpu, M, N, K, epi):
    """A in fp32 goes in as two fp16 planes (epi | 4) and fp16 outputs come back as value + remainder
    (epi | 8): the result matches an fp32 GEMM on the fp32 A to 3e-5 of the output scale, where
    the one-plane form is off by the fp16 rounding of A (2^-11)."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(M + N)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    ref = (A.double() @ B.double().T)
    planes = _split(A).contiguous()
    if epi in (0, 1):
        base = torch.randn(M, N, device="cuda", generator=g) if epi == 1 else torch.zeros(M, N, device="cuda")
        out = base.clone()
        _lib.call("yb_prefill_gemm_dev", _p(out), None, _p(planes), _p(B), M, N, K, epi | 4, N, None)
        got = out.double() - base.double()
        exp = ref
    else:
        cols = N // 2 if epi == 2 else N
        out = torch.zeros(2, M, cols, dtype=torch.float16, device="cuda")
        _lib.call("yb_prefill_gemm_dev", None, _p(out), _p(planes), _p(B), M, N, K, epi | 4 | 8, cols, None)
        got = out[0].double() + out[1].double()
        if epi == 2:
            gt, up = ref[:, 0::2], ref[:, 1::2]
            exp = gt / (1 + torch.exp(-gt)) * up
        else:
            exp = ref
    torch.cuda.synchronize()
    err = (got - exp).abs().max().item()
    scale = exp.abs().max().item()
    assert err <= 3e-5 * scale + 1e-6, (err, scale)

