"""Per-kernel timeline of one decode step (graph executor), from the engine's %globaltimer stamps.

    python -m yalm_b200.timeline [--config mistral-7b] [--prompt 100] [--steps 4] [--context 0]

Creates the engine with YB_TRACE=1 (yb_trace_read, include/yalm_b200.h), fills the KV cache with a
random prompt of --prompt tokens (yb_prefill), runs --steps decode steps and reads the last step's
stamps.  Prints one JSON line: per kernel of a layer (QKV, attention, wo, gate/up, w2) the phase
times in microseconds (first, median and last CTA to reach each stamp), median over the layers,
measured from the end of the previous kernel (the last CTA's epilogue stamp; for attention the QKV
kernel's).  Under torchrun (--gpus N > 1) every
rank builds its tensor-parallel shard and rank 0 prints, with the exchange latencies
(exchange_latency_us): from this rank's last writer CTA (wo, w2 epilogue end) to the reader kernel's
last CTA having the all-reduced input (gate/up, next QKV), the max over ranks per exchange point.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import time

import numpy as np

from . import _lib

# stamps per kernel (yb_trace_read): matvecs 0 entry, 1 input loaded, 2 tensor-parallel all-reduce
# done, 3 last weight stage consumed, 4 epilogue done; attention 0 entry, 7 early copies issued,
# 1 inputs ready, 2 first chunk staged, 5 slots folded, 6 warp weights formed, 3 record written,
# 4 exit
MATVEC = {"entry": 0, "input": 1, "allreduce": 2, "last_stage": 3, "epilogue": 4}
ATTN = {"entry": 0, "early_issued": 7, "ready": 1, "first_chunk": 2, "folded": 5, "weights": 6, "record": 3,
        "exit": 4}


def read(engine) -> np.ndarray:
    """The last step's stamps as int64 [CTAs][kernels][8] (0 = not reached)."""
    L = _lib.lib()
    grid, events = ctypes.c_int(), ctypes.c_int()
    _lib.call("yb_trace_read", engine, None, 0, ctypes.byref(grid), ctypes.byref(events))
    out = np.zeros(grid.value * events.value, np.uint64)
    _lib.call("yb_trace_read", engine, out.ctypes.data, out.size, ctypes.byref(grid), ctypes.byref(events))
    del L
    return out.reshape(grid.value, events.value // 8, 8).astype(np.int64)


def _col(tr, k, j):
    v = tr[:, k, j]
    return v[v > 0]


def layer_phases(tr: np.ndarray, n_layers: int, w2_panels: int = 1) -> dict:
    """Median over layers of each kernel's phases, in us after the previous kernel's last epilogue."""
    per = 4 + w2_panels
    rows = {"qkv": [], "attention": [], "wo": [], "gateup": [], "w2": []}
    for l in range(n_layers):
        ks = {"qkv": l * per, "attention": l * per + 1, "wo": l * per + 2, "gateup": l * per + 3,
              "w2": l * per + 4 + w2_panels - 1}
        prev_end = None
        if l > 0:
            e = _col(tr, (l - 1) * per + 4 + w2_panels - 1, 4)
            prev_end = e.max() if e.size else None
        for name in ("qkv", "attention", "wo", "gateup", "w2"):
            k = ks[name]
            stamps = ATTN if name == "attention" else MATVEC
            end_prev = prev_end
            d = {}
            if end_prev is not None:
                for ph, j in stamps.items():
                    c = _col(tr, k, j)
                    if c.size:
                        d[ph + "_first"] = (c.min() - end_prev) / 1e3
                        d[ph + "_median"] = (float(np.median(c)) - end_prev) / 1e3
                        d[ph + "_last"] = (c.max() - end_prev) / 1e3
                rows[name].append(d)
            e = _col(tr, k, 4)
            prev_end = e.max() if e.size else prev_end
    out = {}
    for name, ds in rows.items():
        if not ds:
            continue
        keys = sorted(set().union(*ds))
        out[name] = {k: round(float(np.median([d[k] for d in ds if k in d])), 2) for k in keys}
    return out


def exchange_latency(tr: np.ndarray, n_layers: int) -> dict:
    """Tensor parallel: per exchange point, the reader kernel's last all-reduced stamp minus this
    rank's last writer epilogue stamp (us); medians over the layers."""
    per = 5
    a, b = [], []
    for l in range(n_layers):
        wo_end = _col(tr, l * per + 2, 4)
        gu_in = _col(tr, l * per + 3, 2)
        if wo_end.size and gu_in.size:
            a.append((gu_in.max() - wo_end.max()) / 1e3)
        if l + 1 < n_layers:
            w2_end = _col(tr, l * per + 4, 4)
            qkv_in = _col(tr, (l + 1) * per, 2)
            if w2_end.size and qkv_in.size:
                b.append((qkv_in.max() - w2_end.max()) / 1e3)
    return {"wo_to_gateup_us": round(float(np.median(a)), 2) if a else None,
            "w2_to_qkv_us": round(float(np.median(b)), 2) if b else None}


def w2_panels_of(c, world: int = 1) -> int:
    """Column panels of the w2 matvec (the engine splits rows wider than 14336 fp16 columns)."""
    hid = c.hidden_dim // world
    p = 1
    while hid // p > 14336 or (hid // p) % 8 or hid % p:
        p += 1
    return p


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="mistral-7b")
    ap.add_argument("--prompt", type=int, default=100)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--context", type=int, default=0)
    args = ap.parse_args()
    os.environ["YB_TRACE"] = "1"
    import torch
    from . import InferenceMode, Model, YALMData, synth
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        dist.barrier()
    shape = synth.SHAPES[args.config]
    path = os.path.join(synth.scratch_dir(synth.file_bytes(shape)), f"yalm_{args.config}_seed0.yalm")
    if rank == 0:
        synth.write_yalm(path, shape, seed=0)
    if dist:
        dist.barrier()
    m = Model(YALMData(path), context=args.context).cuda(local, rank, world)
    if world > 1:
        def ag(blob):
            out = [None] * world
            dist.all_gather_object(out, blob)
            return out
        m.tp_join(ag)
    c = m.config
    rng = np.random.default_rng(5)
    prompt = [int(t) for t in rng.integers(0, c.vocab_size, args.prompt)]
    m.prefill(prompt, 0)
    for i in range(args.steps):
        m.forward_async(int(rng.integers(0, c.vocab_size)), args.prompt + i, InferenceMode.OUTPUT_LOGITS)
    m.sync()
    time.sleep(0.01)
    tr = read(m.engine)
    res = {"config": args.config, "kv_len": args.prompt + args.steps, "tp": world,
           "phases_us": layer_phases(tr, c.n_layers, w2_panels_of(c, world))}
    if world > 1:
        ex = exchange_latency(tr, c.n_layers)
        t = torch.tensor([ex["wo_to_gateup_us"] or 0.0, ex["w2_to_qkv_us"] or 0.0], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res["exchange_latency_us"] = {"wo_to_gateup": round(float(t[0]), 2), "w2_to_qkv": round(float(t[1]), 2)}
    if rank == 0:
        print(json.dumps(res))
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
