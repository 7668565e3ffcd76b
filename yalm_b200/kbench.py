"""Isolated decode-kernel benchmark (benchmark config 4; the counterpart of yalm's
`build/test -bk {matmul,matmul-wide,mha,ffn}`, src/test.cpp:339-405).

    python -m yalm_b200.kbench [--kernel gemv|gateup|qkv|attention|prefill_attention|prefill_gemm|prefill|all]
                               [--iters N] [--warm W] [--quick]

Each launch goes through the C ABI (yb_gemv_dev, yb_gateup_dev, yb_qkv_dev, yb_attention_dev) on
seeded inputs: W ~ N(0, 0.02) fp16, x ~ N(0, 1), q/K/V ~ N(0, 1) fp16.  Launches rotate over enough
distinct weight / cache copies to cover at least 4x the 126 MB L2, so every launch streams from HBM.
Time is measured with CUDA events around `iters` back-to-back launches on one stream (the mean; a
second pass with an event after every launch gives the per-launch p10 / p50 / p90, which include
that event's drain); GB/s counts algorithmic bytes (weights + activations in/out; for attention
K + V + q + out).  Prints one JSON line per case.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math

import numpy as np

from . import _lib

L2_BYTES = 126 * 2 ** 20


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _copies(nbytes):
    if _RESIDENT:
        return 1
    return max(1, math.ceil(4 * L2_BYTES / nbytes))


_WARM = 3
_RESIDENT = False  # --resident: one copy of the operands, which stays in L2 when it fits


_LAST_SPREAD: dict = {}


def _time(fn, iters, warm=None):
    """Mean milliseconds per launch over `iters` back-to-back launches, and (kept in _LAST_SPREAD for
    the caller's JSON line) the per-launch p10 / p50 / p90 in microseconds from a second pass with an
    event recorded after every launch, when iters >= 3.  An event makes the stream drain the kernel
    before the next one starts, so the spread pass reads 1-3 us per launch above the mean pass for
    the short kernels; the mean is the throughput figure.  Both passes queue their launches behind a
    device-side spin (~30 us of SM cycles per launch), so host launch overhead enters neither."""
    import torch
    for i in range(_WARM if warm is None else warm):
        fn(i)
    torch.cuda.synchronize()
    spin = 60_000 * max(1, iters)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(spin)
    a.record()
    for i in range(iters):
        fn(i)
    b.record()
    b.synchronize()
    mean_ms = a.elapsed_time(b) / iters
    _LAST_SPREAD.clear()
    if iters < 3:  # too few launches for percentiles; one pass keeps a profiler's launch count simple
        return mean_ms
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(iters + 1)]
    torch.cuda._sleep(spin)
    ev[0].record()
    for i in range(iters):
        fn(i)
        ev[i + 1].record()
    ev[-1].synchronize()
    per = np.array([ev[i].elapsed_time(ev[i + 1]) for i in range(iters)]) * 1000.0
    _LAST_SPREAD.update({f"p{q}_us": round(float(np.percentile(per, q)), 2) for q in (10, 50, 90)})
    return mean_ms


def bench_gemv(rows, cols, iters, kind="gemv", seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    wbytes = rows * cols * 2
    n = _copies(wbytes)
    ws = [(torch.randn(rows, cols, device="cuda", generator=g) * 0.02).half() for _ in range(n)]
    x = torch.randn(cols, device="cuda", generator=g)
    nw = torch.ones(cols, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if kind == "gateup":
        out = torch.zeros(rows // 2, device="cuda")

        def fn(i):
            _lib.call("yb_gateup_dev", _p(out), _p(x), _p(ws[i % n]), rows // 2, cols, _p(nw), 1e-5, 1, stream)
        ybytes = rows // 2 * 4
    else:
        out = torch.zeros(rows, device="cuda")

        def fn(i):
            _lib.call("yb_gemv_dev", _p(out), _p(x), _p(ws[i % n]), rows, cols, None, 0.0, 0, stream)
        ybytes = rows * 4
    ms = _time(fn, iters)
    nbytes = wbytes + cols * 4 + ybytes
    return {"kernel": kind, "rows": rows, "cols": cols, "us": round(ms * 1000, 2),
            "gbs": round(nbytes / (ms / 1000) / 1e9, 1), "bytes": nbytes, "copies": n, **_LAST_SPREAD}


def bench_qkv(dim, nh, nkv, hd, msl, iters, seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows = (nh + 2 * nkv) * hd
    wbytes = rows * dim * 2
    n = _copies(wbytes)
    ws = [(torch.randn(rows, dim, device="cuda", generator=g) * 0.02).half() for _ in range(n)]
    x = torch.randn(dim, device="cuda", generator=g)
    nw = torch.ones(dim, device="cuda")
    q = torch.zeros(nh * hd, device="cuda")
    kc = torch.zeros(nkv, msl, hd, device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    inv = torch.tensor([1.0 / (1e6 ** (j / hd)) for j in range(0, hd, 2)], device="cuda", dtype=torch.float32)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def fn(i):
        pos = i % msl
        _lib.call("yb_qkv_dev", _p(q), _p(kc), _p(vc), _p(x), _p(ws[i % n]), _p(nw), 1e-5, dim, nh, nkv, hd, hd, msl,
                  pos, pos, 0, 3.0e38, _p(inv), stream)
    ms = _time(fn, iters)
    nbytes = wbytes + dim * 8 + nh * hd * 4 + 2 * nkv * hd * 2
    return {"kernel": "qkv+rope+kv_append", "rows": rows, "cols": dim, "us": round(ms * 1000, 2),
            "gbs": round(nbytes / (ms / 1000) / 1e9, 1), "bytes": nbytes, "copies": n, **_LAST_SPREAD}


def bench_attention(nh, nkv, hd, kv_len, iters, seed=0, msl=None):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    msl = kv_len if msl is None else max(msl, kv_len)
    kvbytes = 2 * nkv * msl * hd * 2
    n = _copies(2 * nkv * kv_len * hd * 2)  # copies enough that the rows read rotate through > 4 x L2
    ks = [torch.randn(nkv, msl, hd, device="cuda", generator=g).half() for _ in range(n)]
    vs = [torch.randn(nkv, msl, hd, device="cuda", generator=g).half() for _ in range(n)]
    q = torch.randn(nh * hd, device="cuda", generator=g)
    out = torch.zeros(nh * hd, device="cuda")
    scratch = torch.zeros(_lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl), dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def fn(i):
        _lib.call("yb_attention_dev", _p(out), _p(q), _p(ks[i % n]), _p(vs[i % n]), nh, nkv, hd, msl, kv_len,
                  _p(scratch), stream)
    ms = _time(fn, iters)
    info = (ctypes.c_int * 20)()
    _lib.call("yb_attention_plan_info", nh, nkv, hd, msl, info)
    nbytes = 2 * nkv * kv_len * hd * 2 + 2 * nh * hd * 4  # the K / V rows read, q in, out
    return {"kernel": "attention", "n_heads": nh, "n_kv_heads": nkv, "head_dim": hd, "kv_len": kv_len, "max_seq_len": msl,
            "us": round(ms * 1000, 2), "gbs": round(nbytes / (ms / 1000) / 1e9, 1), "bytes": nbytes, "copies": n,
            "cluster": info[0], "clusters_per_kv_head": info[1], "ctas": info[2],
            "max_active_clusters": list(info[4:20]), **_LAST_SPREAD}


def bench_prefill_gemm(M, N, K, planes, swiglu, iters, seed=0):
    """One batched-prefill GEMM (yb_prefill_gemm_dev): C[M][N] = A[M][K] . W[N][K]^T on tcgen05, A as
    one fp16 plane or as the prefill's two (value, remainder: 2M rows, each product two MMAs); the
    fp32 store epilogue, or with `swiglu` the gate/up form the prefill runs (SwiGLU of column pairs
    to fp16, with the remainder plane written when A has two).  FLOP counts the useful 2 M N K."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn(planes * M, K, device="cuda", generator=g)).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    epi = (2 if swiglu else 0) | (4 if planes == 2 else 0) | (8 if swiglu and planes == 2 else 0)
    if swiglu:
        out = torch.empty(2 * M * (N // 2), dtype=torch.float16, device="cuda")
        args = (None, _p(out), N // 2)
    else:
        out = torch.empty(M, N, device="cuda")
        args = (_p(out), None, N)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def fn(i):
        _lib.call("yb_prefill_gemm_dev", args[0], args[1], _p(a), _p(b), M, N, K, epi, args[2], stream)
    ms = _time(fn, iters)
    return {"kernel": "prefill_gemm", "M": M, "N": N, "K": K, "a_planes": planes,
            "epilogue": "swiglu_f16" if swiglu else "store_f32", "us": round(ms * 1000, 2),
            "tflops": round(2.0 * M * N * K / (ms / 1000) / 1e12, 1), **_LAST_SPREAD}


def bench_prefill_attention(nh, nkv, hd, T, iters, seed=0):
    """Causal attention of a T-token prompt (yb_prefill_attention_dev); the caches fit in L2, as in
    the prefill where each layer's K/V were just written."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(T, nh * hd, device="cuda", generator=g)
    k = torch.randn(nkv, T, hd, device="cuda", generator=g).half()
    v = torch.randn(nkv, T, hd, device="cuda", generator=g).half()
    out = torch.zeros(T * nh * hd, dtype=torch.float16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def fn(i):
        _lib.call("yb_prefill_attention_dev", _p(out), _p(q), _p(k), _p(v), T, 0, nh, nkv, hd, T, stream)
    ms = _time(fn, iters)
    flop = 4.0 * nh * hd * T * (T + 1) / 2  # q.k and p.v over the causal triangle
    return {"kernel": "prefill_attention", "n_heads": nh, "n_kv_heads": nkv, "head_dim": hd, "tokens": T,
            "us": round(ms * 1000, 2), "tflops": round(flop / (ms / 1000) / 1e12, 1), **_LAST_SPREAD}


def bench_prefill(tokens, iters, config="mistral-7b", seed=0):
    """The whole batched prompt pass (yb_prefill, every layer's GEMMs, norms, RoPE / KV append and
    attention, then the classifier) of the seeded synthetic checkpoint.  Per prompt length one
    untimed call sizes the buffers and loads the kernels; then `iters` calls are timed, each by
    wall clock around the call and a yb_sync."""
    import os
    import time
    from . import synth
    from .codec import YALMData
    from .model import Model
    shape = synth.shape_with(config)
    path = os.path.join(synth.scratch_dir(synth.file_bytes(shape)), f"yalm_{config}_seed0.yalm")
    synth.write_yalm(path, shape, seed=0)
    m = Model(YALMData(path)).cuda(0)
    rng = np.random.default_rng(seed)
    rows = []
    try:
        for t in tokens:
            prompt = rng.integers(0, m.config.vocab_size, t)
            m.prefill(prompt, 0)
            m.sync()
            best = total = 0.0
            for i in range(iters):
                t0 = time.perf_counter()
                m.prefill(prompt, 0)
                m.sync()
                dt = time.perf_counter() - t0
                total += dt
                best = dt if i == 0 else min(best, dt)
            rows.append({"kernel": "prefill", "config": config, "tokens": t, "iters": iters,
                         "mean_s": round(total / iters, 4), "best_s": round(best, 4),
                         "tok_s": round(t * iters / total, 1)})
    finally:
        m.close()
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="all",
                    choices=["gemv", "gateup", "qkv", "attention", "prefill_attention", "prefill_gemm", "prefill",
                             "all"])
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--quick", action="store_true", help="one shape per kernel (for profiler captures)")
    ap.add_argument("--kv-lens", default="", help="attention: comma-separated kv_len values")
    ap.add_argument("--msl", type=int, default=0, help="attention: cache capacity (default: kv_len)")
    ap.add_argument("--heads", default="32,8", help="attention: n_heads,n_kv_heads (head_dim 128)")
    ap.add_argument("--tokens", default="", help="prefill_attention, prefill: comma-separated prompt lengths")
    ap.add_argument("--warm", type=int, default=3, help="untimed launches per case before the timed ones")
    ap.add_argument("--resident", action="store_true",
                    help="one copy of each operand (L2-resident when it fits) instead of rotating over > 4 x L2")
    args = ap.parse_args(argv)
    global _WARM, _RESIDENT
    _WARM = args.warm
    _RESIDENT = args.resident
    import torch
    torch.cuda.set_device(0)
    rows = []
    if args.kernel in ("gemv", "all"):
        shapes = [(32000, 4096)] if args.quick else [(4096, 4096), (4096, 14336), (32000, 4096), (6144, 4096)]
        for r, c in shapes:
            rows.append(bench_gemv(r, c, args.iters))
    if args.kernel in ("gateup", "all"):
        rows.append(bench_gemv(2 * 14336, 4096, args.iters, kind="gateup"))
    if args.kernel in ("qkv", "all"):
        rows.append(bench_qkv(4096, 32, 8, 128, 4096, args.iters))
    if args.kernel in ("attention", "all"):
        lens = [4096] if args.quick else [128, 1024, 4096, 16384, 32768]
        if args.kv_lens:
            lens = [int(v) for v in args.kv_lens.split(",")]
        nh, nkv = (int(v) for v in args.heads.split(","))
        for kv in lens:
            rows.append(bench_attention(nh, nkv, 128, kv, args.iters, msl=args.msl or None))
    if args.kernel in ("prefill_attention", "all"):
        lens = [int(v) for v in args.tokens.split(",")] if args.tokens else ([1024] if args.quick else [1024, 3202])
        for t in lens:
            rows.append(bench_prefill_attention(32, 8, 128, t, max(3, args.iters // 20)))
    if args.kernel == "prefill_gemm":
        T = int(args.tokens.split(",")[0]) if args.tokens else 3202
        for planes in (1, 2):
            for M, N, K, sw in ((T, 6144, 4096, False), (T, 4096, 4096, False), (T, 28672, 4096, False),
                                (T, 4096, 14336, False), (T, 28672, 4096, True)):
                rows.append(bench_prefill_gemm(M, N, K, planes, sw, max(3, args.iters // 10)))
    if args.kernel == "prefill":  # not part of "all": it writes and loads the 14 GB 7B checkpoint
        lens = [int(v) for v in args.tokens.split(",")] if args.tokens else [3202, 1024]
        rows.extend(bench_prefill(lens, max(1, args.iters // 100)))
    for r in rows:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
