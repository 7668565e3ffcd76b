"""Batch-1 decode benchmark (the BASELINE.json metric): decode tok/s of the Mistral-7B architecture
(fp16 weights, seeded synthetic .yalm checkpoint, 4k context) on N B200s, with the fraction of the
HBM weight-streaming roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config mistral-7b|tiny|llama-70b]
    python bench.py --impl reference ...     # yalm's own CPU decode path (oracle/_ref) on the host cores

Workload: a 16-token random prompt (HYDRATE, last token OUTPUT_LOGITS),
then decode steps at positions 16..135 (120 decode tokens), wrapping back to 16 for K > 120 so the
KV length distribution stays that of the config.  One step = one decode token = one forward pass.

  value  tok/s with everything resident on the device: K back-to-back yb_forward_async steps
         (teacher-forced tokens), CUDA events on the engine stream, max over ranks.
  e2e    the same metric through the public C-ABI call a yalm decode loop makes, wall clock around
         the K calls: yb_forward_sample (Model::forward + Sampler::sample at temperature 0 with the
         sampler on the device: token id in, next id out).  e2e.logits_to_host is the same loop
         through yb_forward with 128 KB of fp32 logits copied to pinned host memory and the argmax
         taken on the host.
Under torchrun (N > 1) each rank is one tensor-parallel shard (heads, kv heads, FFN hidden and
vocabulary split N ways); partial sums cross NVLink inside the wo / w2 kernels.
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# (prompt tokens, decode positions) per config: BASELINE.json configs 1, 2 and 5
WORKLOADS = {"tiny": (32, 64), "mistral-7b": (16, 120), "llama-70b": (1024, 128)}
PROMPT_LEN, DECODE_LEN = WORKLOADS["mistral-7b"]
METRIC = "batch-1 decode tok/s (Mistral-7B fp16, 4k ctx)"
METRICS = {"mistral-7b": METRIC, "tiny": "batch-1 decode tok/s (tiny Mistral-architecture fp16, ctx 1024)",
           "llama-70b": "batch-1 decode tok/s (70B-class fp16, 8k ctx)"}
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


class _StdoutToStderr:
    """Sends file descriptor 1 to stderr for a while (NCCL prints its version banner on stdout when
    a communicator is created; the bench's stdout carries only the JSON line)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def workload_name(config: str) -> str:
    """The workload both arms name in their `config` (the reference arm times a bounded sample of it)."""
    return (f"{config} batch-1 decode: {PROMPT_LEN}-token prompt, decode positions "
            f"{PROMPT_LEN}..{PROMPT_LEN + DECODE_LEN - 1}")


def yalm_generation_stats(prompt_len: int, decode_len: int, hydrate_s: float, s_per_token: float) -> dict:
    """yalm's throughput definition (src/main.cpp:195-206): every token of the sequence (prompt and
    generated) over the time of the prompt's hydrate plus the decode loop."""
    total = hydrate_s + decode_len * s_per_token
    n = prompt_len + decode_len
    return {"tokens": n, "hydrate_s": round(hydrate_s, 4), "total_s": round(total, 4),
            "throughput_tok_s": round(n / total, 1) if total > 0 else None}


def context_of(config: str) -> int:
    """The context each config's checkpoint is opened with: yalm caps max_seq_len at 4096 unless a
    context is given (src/model.cpp:30-34); the 70B config asks for 8192."""
    from yalm_b200 import synth
    return 8192 if config == "llama-70b" else min(4096, synth.SHAPES[config].max_seq_len)


def model_file(config: str, rank: int, world: int, dist, dtype: str = "fp16"):
    from yalm_b200 import synth
    shape = synth.shape_with(config, dtype=dtype)
    d = synth.scratch_dir(synth.file_bytes(shape))
    path = os.path.join(d, f"yalm_{config}_seed0.yalm" if dtype == "fp16" else f"yalm_{config}_{dtype}_seed0.yalm")
    if rank == 0:
        t = time.time()
        synth.write_yalm(path, shape, seed=0)
        log(f"[bench] checkpoint {path} ready in {time.time() - t:.1f}s")
    if world > 1:
        dist.barrier()
    return path


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region.  The sampler
    starts before the region and the region starts only once its first sample has arrived
    (nvidia-smi takes a few hundred ms to start); samples taken inside the region are kept, and the
    first one after it when the region is shorter than the sampling period."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.samples = []  # (monotonic time, line)
        self.lines = []

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self.samples.append((time.monotonic(), line))

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            t_wait = time.monotonic() + 5.0
            while not self.samples and time.monotonic() < t_wait and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.proc:
            t_wait = self.t1 + 0.6
            while not any(t >= self.t0 for t, _ in self.samples) and time.monotonic() < t_wait:
                time.sleep(0.01)
            self.proc.send_signal(signal.SIGTERM)
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.reader.join(timeout=2)
            inside = [l for t, l in self.samples if self.t0 <= t <= self.t1]
            after = [l for t, l in self.samples if t > self.t1]
            self.lines = inside if inside else after[:1]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def bench_prompt(vocab_size: int):
    """The workload's prompt: PROMPT_LEN seeded random ids (both arms, and the GPU parity tests of
    the benchmark configs, use these ids)."""
    rng = np.random.default_rng(1234)
    return [int(t) for t in rng.integers(0, vocab_size, PROMPT_LEN)]


def host_cpu() -> dict:
    """The host's CPU model and logical core count (from /proc/cpuinfo), for the CPU baseline record."""
    model, n = None, 0
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    n += 1
                    model = model or line.split(":", 1)[1].strip()
    except OSError:
        pass
    return {"cpu_model": model, "host_logical_cpus": n or os.cpu_count()}


def cpu_baseline(path: str, context: int, n_decode: int, prompt):
    """yalm's own CPU decode path (oracle/_ref/ref_decode, built from the reference sources) on a
    bounded sample of the same workload — the same prompt, then n_decode greedy steps at positions
    len(prompt).. — with all host cores.  Returns its JSON record (per-step seconds, greedy ids)."""
    import oracle
    if not os.path.exists(oracle.REF_BIN):
        return None
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    env = dict(os.environ, OMP_NUM_THREADS=str(threads))
    r = subprocess.run([oracle.REF_BIN, path, str(context), str(n_decode), str(threads)] + [str(t) for t in prompt],
                       capture_output=True, text=True, env=env, timeout=1800)
    line = [l for l in r.stdout.splitlines() if l.startswith("{")]
    if r.returncode != 0 or not line:
        log("[bench] reference CPU run failed:", r.stderr[-2000:])
        return None
    d = json.loads(line[-1])
    d["threads"] = threads
    return d


def run_reference(args):
    """--impl reference: yalm's CPU decode path on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from yalm_b200 import synth
    shape = synth.SHAPES[args.config]
    if args.dtype != "fp16":
        print(json.dumps({"impl": "reference", "unavailable": "yalm's runtime rejects fp8 checkpoints (src/model.cpp:61-70)"}))
        return 0
    path = model_file(args.config, 0, 1, None)
    context = 8192 if args.config == "llama-70b" else 0
    # The same prompt and positions as the GPU arm: W warm-up decode steps at PROMPT_LEN.., then the
    # timed steps.  Each step is one full decode token of the reference; the sample stays inside the
    # workload's decode positions (no wrap) and, for the 70B config (~4.5 s per CPU token), is
    # bounded to keep the run to a few minutes.
    cap = args.ref_max_steps if args.ref_max_steps else (8 if args.config == "llama-70b" else DECODE_LEN - args.warmup)
    n = max(1, min(args.steps, cap))
    prompt = bench_prompt(synth.SHAPES[args.config].vocab_size)
    d = cpu_baseline(path, context, n + args.warmup, prompt)
    if d is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/ref_decode missing or failed"}))
        return 0
    steps = d["step_s"][args.warmup:]
    t = sum(steps)
    v = len(steps) / t
    ref_gpu = reference_gpu(path, context, n + args.warmup, args.warmup, prompt, d["tokens"]) \
        if args.config != "llama-70b" and not args.no_reference_gpu else None
    sample = (f"{len(steps)} timed decode tokens at positions {PROMPT_LEN + args.warmup}..{PROMPT_LEN + args.warmup + len(steps) - 1} "
              f"(+{args.warmup} warm-up) of the full {args.config} model after the workload's {PROMPT_LEN}-token "
              f"prompt, yalm -d cpu code path (Model::forward) via oracle/_ref/ref_decode")
    print(json.dumps({
        "impl": "reference", "metric": METRICS[args.config], "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": len(steps), "warmup": args.warmup, "ms_per_step": round(1000 * t / len(steps), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 weights, f32 compute",
        "data": "synthetic (seeded N(0,0.02) fp16 weights, random token ids)",
        "config": {"workload": workload_name(args.config), "model": args.config, "global_batch": 1,
                   "seq_len": PROMPT_LEN + DECODE_LEN, "context": context_of(args.config),
                   "parallelism": "cpu (yalm -d cpu, OpenMP)"},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": d["threads"], "kind": "reference",
                         "sample": sample, **host_cpu()},
        "greedy_ids": d["tokens"],
        "reference_gpu": ref_gpu,
        "gpu_launches": 0,
    }))
    return 0


def reference_gpu(path, context, n_decode, warmup, prompt, cpu_ids):
    """yalm's own GPU backends on this box, beside the reference arm's CPU figure (not its value):
    oracle/_ref/ref_decode_gpu (yalm's sources built for sm_100a) with -d cuda (the CUDA-graph
    backend, src/infer.cu:1274-1378) and -d cuda-coop (the cooperative kernel, src/coop.cu:378-415)
    on the same checkpoint, prompt and positions, wall clock per decode step (each step syncs for
    its logits, as run_completion's loop does); and oracle/_ref/ref_kernels: yalm's per-layer decode
    kernels alone with the launch shapes of Block::_block_cuda (src/infer.cu:891-1072), CUDA events
    over 64 launches rotating over more than 4 x L2 of weights / cache."""
    import oracle
    if not (os.path.exists(oracle.REF_BIN_GPU) and os.path.exists(oracle.REF_KERNELS)):
        return {"unavailable": "oracle/_ref/ref_decode_gpu or ref_kernels not built"}
    out = {}
    for dev in ("cuda", "cuda-coop"):
        r = subprocess.run([oracle.REF_BIN_GPU, path, str(context), str(n_decode), "1", "-d", dev] +
                           [str(t) for t in prompt], capture_output=True, text=True, timeout=900)
        line = [l for l in r.stdout.splitlines() if l.startswith("{")]
        if r.returncode != 0 or not line:
            out[dev] = {"failed": (r.stderr or r.stdout)[-300:]}
            continue
        rec = json.loads(line[-1])
        st = rec["step_s"][warmup:]
        out[dev] = {"tok_s": round(len(st) / sum(st), 2), "ms_per_step": round(1000 * sum(st) / len(st), 4),
                    "steps": len(st), "greedy_ids_equal_cpu": rec["tokens"] == list(cpu_ids)}
    r = subprocess.run([oracle.REF_KERNELS, "64", str(PROMPT_LEN + DECODE_LEN // 2), "3232"], capture_output=True,
                       text=True, timeout=600)
    line = [l for l in r.stdout.splitlines() if l.startswith("{")]
    out["kernels"] = json.loads(line[-1])["kernels"] if r.returncode == 0 and line else {"failed": r.stderr[-300:]}
    out["how"] = ("yalm's -d cuda / -d cuda-coop decode loop (oracle/_ref/ref_decode_gpu, built from its sources for "
                  "sm_100a) and its per-layer kernels alone (oracle/_ref/ref_kernels), same box")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=480)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--config", default="mistral-7b", choices=["tiny", "mistral-7b", "llama-70b"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-max-steps", type=int, default=0,
                    help="cap on the reference arm's timed steps (default: the workload's decode positions)")
    ap.add_argument("--cpu-baseline-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="reference arm: skip timing yalm's own GPU backends beside its CPU path")
    ap.add_argument("--no-profile", action="store_true")
    ap.add_argument("--no-long-context", action="store_true", help="skip the config-3 (3202-token prefill) phase")
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "fp8"],
                    help="weight dtype of the synthetic checkpoint (fp8 = E5M2, as convert.py writes it)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    global PROMPT_LEN, DECODE_LEN
    PROMPT_LEN, DECODE_LEN = WORKLOADS[args.config]
    if args.impl == "reference":
        return run_reference(args)

    import torch
    from yalm_b200 import InferenceMode, InferenceState, Model, YALMData, build, _lib
    build.build_all()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        with _StdoutToStderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
            dist.barrier()  # the communicator exists after the first collective

    tp_check = tp_parity(world, rank, local, dist)
    log(f"[bench] rank {rank}: tensor-parallel check {tp_check}")
    path = model_file(args.config, rank, world, dist, args.dtype)
    context = 8192 if args.config == "llama-70b" else 0
    y = YALMData(path)
    t = time.time()
    m = Model(y, context=context).cuda(local, rank, world)
    t_load = time.time() - t
    if world > 1:
        def ag(b):
            out = [None] * world
            dist.all_gather_object(out, b)
            return out
        m.tp_join(ag)
    log(f"[bench] rank {rank}: engine ready in {time.time() - t:.1f}s")
    c = m.config
    prompt = np.array(bench_prompt(c.vocab_size))
    stream_toks = np.random.default_rng(1235).integers(0, c.vocab_size, 4096)
    s = InferenceState(c)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    m.prefill([int(t) for t in prompt], 0, s)  # batched when the engine supports it, else per token
    t_prompt = time.perf_counter() - t0

    def pos_of(i):
        return PROMPT_LEN + (i % DECODE_LEN)

    stream = torch.cuda.ExternalStream(m.stream_ptr())
    # ---------------------------------------------------------------- device-resident value
    for i in range(args.warmup):
        m.forward_async(int(stream_toks[i % 4096]), pos_of(i))
    m.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            j = args.warmup + i
            m.forward_async(int(stream_toks[j % 4096]), pos_of(j))
        ev1.record(stream)
        ev1.synchronize()
        m.sync()
    ms_dev = ev0.elapsed_time(ev1)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if world > 1:
        tt = torch.tensor([ms_dev], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_dev = float(tt.item())
    value = args.steps / (ms_dev / 1000.0)
    clocks = clk.summary()
    if world > 1:
        # every rank sampled its own GPU: the slowest median, all reasons, per-rank detail
        per = [None] * world
        dist.all_gather_object(per, clocks)
        meds = [p["sm_mhz"] for p in per if p["sm_mhz"] is not None]
        clocks = {"sm_mhz": min(meds) if meds else None,
                  "sm_max_mhz": max((p["sm_max_mhz"] for p in per if p["sm_max_mhz"] is not None), default=None),
                  "reasons": sorted(set().union(*(p["reasons"] for p in per))),
                  "samples": sum(p["samples"] for p in per), "per_rank_sm_mhz": [p["sm_mhz"] for p in per]}

    # ---------------------------------------------------------------- end to end through the C ABI
    # (a) yb_forward_sample: the decode loop of yalm's main.cpp (forward + Sampler::sample at
    # temperature 0) with the sampler on the device: token id in, next token id (4 bytes) out.
    e2e_steps = args.steps
    tok = int(prompt[-1])
    for pos, t_ in enumerate(prompt[:-1]):
        m.forward_async(int(t_), pos, InferenceMode.HYDRATE_KV_CACHE)
    tok = m.forward_sample(tok, PROMPT_LEN - 1)
    greedy = [tok]  # free-running greedy ids from the prompt (positions PROMPT_LEN.. until the wrap)
    for i in range(args.warmup):
        tok = m.forward_sample(tok, pos_of(i))
        greedy.append(tok)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        tok = m.forward_sample(tok, pos_of(args.warmup + i))
        greedy.append(tok)
    t_e2e = time.perf_counter() - t0
    greedy = greedy[:DECODE_LEN]
    if world > 1:
        tt = torch.tensor([t_e2e], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = float(tt.item())
    e2e = e2e_steps / t_e2e

    # (b) yb_forward with the full logits copied to pinned host memory and greedy argmax on the host
    logits_host = torch.empty(c.vocab_size, dtype=torch.float32, pin_memory=True)
    lg = logits_host.numpy()

    class PinnedState(InferenceState):
        def logits(self):
            return lg

    ps = PinnedState(c)
    for pos, t_ in enumerate(prompt[:-1]):
        m.forward_async(int(t_), pos, InferenceMode.HYDRATE_KV_CACHE)
    m.forward(ps, int(prompt[-1]), PROMPT_LEN - 1, InferenceMode.OUTPUT_LOGITS)
    for i in range(args.warmup):
        m.forward(ps, int(np.argmax(lg)), pos_of(i))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        m.forward(ps, int(np.argmax(lg)), pos_of(args.warmup + i))  # greedy, sampler.cpp:27-38
    t_l = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([t_l], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_l = float(tt.item())
    e2e_logits = e2e_steps / t_l

    # ---------------------------------------------------------------- dominant kernel roofline
    peak, peak_kind = measured_peaks()
    kv_mean = PROMPT_LEN + (DECODE_LEN + 1) / 2.0
    step_bytes = c.weight_bytes_per_token(world) + c.kv_bytes_per_token(int(round(kv_mean)), world) + \
        c.n_layers * 2 * (c.n_kv_heads // world) * c.head_dim * 2
    step_gbs = step_bytes / (ms_dev / args.steps / 1000.0) / 1e9
    executor = m.executor()
    roofline = None
    kernels = {}
    if executor == "persistent":
        # the persistent kernel is the whole step: one launch per token
        achieved = step_bytes / (ms_dev / args.steps / 1000.0) / 1e9
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
                traffic = json.load(f).get(f"{args.config}:persistent_step")
        except Exception:
            traffic = None
        roofline = {"bound": "hbm", "kernel": "persistent_step_kernel (one cooperative launch per decode step)",
                    "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else
                    "fallback 6650 GB/s", "traffic": traffic, "algorithmic_bytes_per_launch": step_bytes}
    if world == 1 and not args.no_profile:
        names = ["qkv", "attention", "wo", "gateup", "w2", "classifier"]
        hid, dim = c.hidden_dim, c.dim
        q_dim, kv_dim = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        wb = c.weight_bytes
        kbytes = {"qkv": (q_dim + 2 * kv_dim) * dim * wb + dim * 8 + (q_dim + 2 * kv_dim) * 4,
                  "wo": dim * q_dim * wb + q_dim * 4 + dim * 8,
                  "gateup": 2 * hid * dim * wb + dim * 8 + hid * 4,
                  "w2": dim * hid * wb + hid * 4 + dim * 8,
                  "classifier": c.vocab_size * dim * wb + dim * 8 + c.vocab_size * 4}
        import ctypes
        for wi, nm in enumerate(names):
            msv = ctypes.c_float()
            _lib.call("yb_profile_kernel", m.engine, wi, c.n_layers * 4, ctypes.byref(msv))
            kernels[nm] = {"us": round(msv.value * 1000, 2)}
            if nm in kbytes:
                kernels[nm]["gbs"] = round(kbytes[nm] / (msv.value / 1000) / 1e9, 1)
        if executor == "graph":
            dom = "gateup"
            achieved = kernels[dom]["gbs"]
            traffic = None
            try:
                with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
                    traffic = json.load(f).get(f"{args.config}:{dom}" + ("" if args.dtype == "fp16" else f":{args.dtype}"))
            except Exception:
                traffic = None
            roofline = {"bound": "hbm", "kernel": f"gemv gate/up (fused W1/W3 + SwiGLU, {2 * hid}x{dim} "
                                                  f"{'fp16' if args.dtype == 'fp16' else 'fp8 E5M2'})",
                        "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else
                        "fallback 6650 GB/s", "traffic": traffic,
                        "algorithmic_bytes_per_launch": kbytes[dom]}

    long_ctx = None
    if args.config == "mistral-7b" and not args.no_long_context:
        long_ctx = long_context(m, c, args, stream, world, dist, peak)

    cpu = None
    greedy_match = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config != "llama-70b" and args.dtype == "fp16":
        d = cpu_baseline(path, context, args.cpu_baseline_steps, [int(t) for t in prompt])
        if d:
            st = d["step_s"]
            cpu = {"value": round(len(st) / sum(st), 4), "unit": "tok/s", "cores": d["threads"], "kind": "reference",
                   "sample": f"{len(st)} greedy decode tokens of the full {args.config} model after the workload's "
                             f"{PROMPT_LEN}-token prompt, yalm -d cpu code path (oracle/_ref/ref_decode), "
                             f"{d['threads']} OpenMP threads", **host_cpu()}
            ref_ids = [int(t) for t in d["tokens"]]
            n = min(len(ref_ids), len(greedy))
            greedy_match = {"steps": n, "match": greedy[:n] == ref_ids[:n], "engine": greedy[:n], "reference": ref_ids[:n],
                            "how": "free-running greedy ids after the workload's prompt: yb_forward_sample (this arm's "
                                   "e2e loop) vs yalm's CPU path (ref_decode, argmax, sampler.cpp:27-38)"}

    tp_ex = None
    if world > 1 and executor == "graph":
        m.close()
        tp_ex = tp_exchange(args.config, path, context, world, rank, local, dist)
    if world > 1:
        dist.barrier()
    if rank == 0:
        if executor == "persistent":
            launches_per_step = 1
        else:
            launches_per_step = 1 + c.n_layers * (4 + m_w2_panels(m)) + 1 + (1 if world > 1 else 0)
        # the timed `value` region runs K logits-mode steps (no sampler kernel)
        out = {
            "metric": METRICS[args.config] if args.dtype == "fp16" else METRICS[args.config] + ", fp8 E5M2 weights",
            "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_dev / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("f16" if args.dtype == "fp16" else "f8e5m2") + " weights, f32 accumulate/activations",
            "data": "synthetic (seeded N(0,0.02) fp16 weights in the .yalm layout, random token ids)",
            "config": {"workload": workload_name(args.config), "model": args.config,
                       "global_batch": 1, "seq_len": PROMPT_LEN + DECODE_LEN, "context": c.max_seq_len,
                       "parallelism": f"tp{world}", "l2": "inputs larger than L2 (weights streamed every step: "
                                                          f"{step_bytes / 1e9:.2f} GB/step/rank)"},
            "e2e": {"value": round(e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
                    "api": "yb_forward_sample (greedy on the device)",
                    "logits_to_host": {"value": round(e2e_logits, 3), "api": "yb_forward + host argmax",
                                       "d2h_bytes_per_step": 4 * c.vocab_size}},
            "roofline": roofline,
            "step_roofline": {"bytes_per_step_per_rank": step_bytes, "achieved_gbs": round(step_gbs, 1), "peak": peak,
                              "frac": round(step_gbs / peak, 4)},
            "executor": executor,
            "prompt": {"tokens": PROMPT_LEN, "seconds": round(t_prompt, 4),
                       "tok_s": round(PROMPT_LEN / max(t_prompt, 1e-9), 1), "api": "yb_prefill"},
            # yalm's own "Generation stats" (src/main.cpp:195-206): prompt plus generated tokens over the
            # hydrate plus the decode loop, for this workload's prompt and DECODE_LEN generated tokens,
            # the loop's per-token time taken from the yb_forward_sample loop above
            "yalm_generation_stats": yalm_generation_stats(PROMPT_LEN, DECODE_LEN, t_prompt, t_e2e / max(e2e_steps, 1)),
            "engine_load": {"seconds": round(t_load, 2), "weight_bytes_per_rank": c.weight_bytes_per_token(world),
                            "gb_s": round(c.weight_bytes_per_token(world) / max(t_load, 1e-9) / 1e9, 1),
                            "source": "checkpoint pages in the host page cache (tmpfs)"},
            "graph_kernels_us": kernels,
            "cpu_baseline": cpu,
            "greedy_match": greedy_match,
            "tp_check": tp_check,
            "tp_exchange_us": tp_ex,
            "long_context": long_ctx,
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(out))
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def tp_parity(world, rank, local, dist):
    """The tensor-parallel check the bench runs first at every N: the small 8-kv-head checkpoint of
    tests/golden/kv8_golden.npz (made by tests/golden/make_golden.py from yalm's CPU path), split
    over the N ranks as the benchmark model is; forced steps compared with the golden logits
    (max-abs <= 2e-2, cosine >= 0.9999), free-running greedy ids with the golden ones (up to the first
    step whose golden top-2 gap is under 2e-3), and every rank's logits bit-identical to rank 0's."""
    import hashlib
    import tempfile
    from yalm_b200 import InferenceMode, InferenceState, Model, YALMData, synth
    gold = dict(np.load(os.path.join(ROOT, "tests", "golden", "kv8_golden.npz")))
    shape = synth.shape_with("tiny", **json.loads(str(gold["shape_json"])))
    path = os.path.join(tempfile.gettempdir(), f"yalm_kv8_seed{int(gold['seed'])}.yalm")
    if rank == 0:
        synth.write_yalm(path, shape, seed=int(gold["seed"]))
    if world > 1:
        dist.barrier()
    m = Model(YALMData(path)).cuda(local, rank, world)
    if world > 1:
        def ag(b):
            out = [None] * world
            dist.all_gather_object(out, b)
            return out
        m.tp_join(ag)
    s = InferenceState(m.config)
    h = hashlib.sha256()
    steps = [int(x) for x in gold["logit_steps"]]
    worst, ok = 0.0, True
    for pos, tok in enumerate(gold["forced"]):
        m.forward(s, int(tok), pos, InferenceMode.OUTPUT_LOGITS)
        lg = s.logits()
        h.update(lg.tobytes())
        if pos in steps:
            exp = gold["logits"][steps.index(pos)]
            d = float(np.abs(lg - exp).max())
            c = float(lg @ exp / (np.linalg.norm(lg) * np.linalg.norm(exp)))
            worst = max(worst, d)
            ok = ok and d <= 2e-2 and c >= 0.9999
    prompt = [int(t) for t in gold["prompt"]]
    for pos, tok in enumerate(prompt):
        m.forward(s, tok, pos, InferenceMode.OUTPUT_LOGITS if pos + 1 == len(prompt) else InferenceMode.HYDRATE_KV_CACHE)
    greedy = []
    for i in range(len(gold["greedy"])):
        tok = int(np.argmax(s.logits()))
        greedy.append(tok)
        h.update(s.logits().tobytes())
        m.forward(s, tok, len(prompt) + i)
    n_sure = next((i for i, gp in enumerate(gold["greedy_gap"]) if gp < 2e-3), len(greedy))
    greedy_ok = greedy[:n_sure] == [int(t) for t in gold["greedy"][:n_sure]]
    status = m.status()
    m.close()
    digests = [h.hexdigest()]
    if world > 1:
        digests = [None] * world
        dist.all_gather_object(digests, h.hexdigest())
    return {"tp_parity_ok": bool(ok and greedy_ok and status == 0), "logits_bit_identical_across_ranks":
            len(set(digests)) == 1, "ranks": world, "worst_logit_max_abs": round(worst, 6),
            "logit_steps_compared": len(steps), "greedy_steps_equal": n_sure if greedy_ok else 0,
            "fixture": "tests/golden/kv8_golden.npz (dim 1024, 16 q / 8 kv heads, 4 layers; yalm's CPU path)"}


def tp_exchange(config, path, context, world, rank, local, dist):
    """Exchange latency of the tensor-parallel all-reduces, from the engine's timeline (YB_TRACE=1):
    a second engine of the benchmark model runs a few decode steps; per exchange point, the reader
    kernel's last CTA to hold the all-reduced input minus this rank's last writer CTA (wo, w2
    epilogue end), median over the layers, max over the ranks."""
    import torch
    from yalm_b200 import InferenceMode, Model, YALMData
    from yalm_b200 import timeline
    os.environ["YB_TRACE"] = "1"
    try:
        m = Model(YALMData(path), context=context).cuda(local, rank, world)
    finally:
        del os.environ["YB_TRACE"]

    def ag(b):
        out = [None] * world
        dist.all_gather_object(out, b)
        return out
    m.tp_join(ag)
    for i in range(8):
        m.forward_async(100 + i, PROMPT_LEN + i, InferenceMode.OUTPUT_LOGITS)
    m.sync()
    tr = timeline.read(m.engine)
    ex = timeline.exchange_latency(tr, m.config.n_layers)
    ph = timeline.layer_phases(tr, m.config.n_layers, timeline.w2_panels_of(m.config, world))
    m.close()
    t = torch.tensor([ex["wo_to_gateup_us"] or 0.0, ex["w2_to_qkv_us"] or 0.0], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {"wo_to_gateup_us": round(float(t[0]), 2), "w2_to_qkv_us": round(float(t[1]), 2),
            "per_exchange_us": round(float(t.mean()), 2), "exchanges_per_step": 2 * m.config.n_layers,
            "rank0_layer_phases_us": ph,
            "how": "engine timeline (YB_TRACE=1, %globaltimer): reader kernel's last all-reduced CTA minus this "
                   "rank's last writer epilogue, median over layers, max over ranks"}


LONG_PREFILL, LONG_DECODE = 3202, 30


def long_context(m, c, args, stream, world, dist, peak):
    """a 3202-token random prompt hydrated one token at a time (yalm's
    prefill, src/main.cpp:171-177), then 30 decode tokens timed with CUDA events on the engine stream
    (kv_len 3203..3232), plus the attention kernel alone at kv_len 3232 (yb_profile_kernel, one GPU)."""
    import ctypes
    import torch
    from yalm_b200 import InferenceMode, _lib
    rng = np.random.default_rng(4321)
    prompt = rng.integers(0, c.vocab_size, LONG_PREFILL)
    toks = rng.integers(0, c.vocab_size, LONG_DECODE)
    torch.cuda.synchronize()
    # yalm's prompt loop, one token per step (src/main.cpp:171-177)
    t0 = time.perf_counter()
    for pos, tok in enumerate(prompt):
        m.forward_async(int(tok), pos, InferenceMode.HYDRATE_KV_CACHE if pos + 1 < LONG_PREFILL else InferenceMode.OUTPUT_LOGITS)
    m.sync()
    t_prefill = time.perf_counter() - t0
    # the same prompt in one batched pass (yb_prefill: tensor-core GEMMs), which leaves the cache the
    # decode steps below read
    # (one untimed pass first on one GPU, where the batched path runs: its buffers are sized and its
    # kernels loaded on first use)
    if world == 1:
        m.prefill(prompt, 0)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    m.prefill(prompt, 0)
    t_batched = time.perf_counter() - t0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i, tok in enumerate(toks):
        m.forward_async(int(tok), LONG_PREFILL + i)
    ev1.record(stream)
    ev1.synchronize()
    m.sync()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    kv_mean = LONG_PREFILL + (LONG_DECODE + 1) / 2.0
    step_bytes = c.weight_bytes_per_token(world) + c.kv_bytes_per_token(int(round(kv_mean)), world)
    out = {"workload": f"{LONG_PREFILL}-token random prompt (HYDRATE), then {LONG_DECODE} decode tokens, "
                       f"kv_len {LONG_PREFILL + 1}..{LONG_PREFILL + LONG_DECODE}",
           "decode_tok_s": round(LONG_DECODE / (ms / 1000.0), 3), "ms_per_step": round(ms / LONG_DECODE, 4),
           "prefill_tok_s_one_token_steps": round(LONG_PREFILL / t_prefill, 1),
           "prefill_tok_s_batched": round(LONG_PREFILL / t_batched, 1),
           "prefill_batched_s": round(t_batched, 4),
           "step_roofline": {"bytes_per_step_per_rank": step_bytes,
                             "achieved_gbs": round(step_bytes / (ms / LONG_DECODE / 1000.0) / 1e9, 1),
                             "frac": round(step_bytes / (ms / LONG_DECODE / 1000.0) / 1e9 / peak, 4)}}
    if world == 1 and not args.no_profile:
        msv = ctypes.c_float()
        _lib.call("yb_profile_kernel", m.engine, 1, c.n_layers * 4, ctypes.byref(msv))
        kv_len = LONG_PREFILL + LONG_DECODE
        abytes = 2 * c.n_kv_heads * c.head_dim * 2 * kv_len + 2 * c.n_heads * c.head_dim * 4
        out["attention"] = {"kv_len": kv_len, "us": round(msv.value * 1000, 2),
                            "gbs": round(abytes / (msv.value / 1000) / 1e9, 1), "bytes": abytes}
    return out


def m_w2_panels(m) -> int:
    hid = m.config.hidden_dim // m.tp_size
    p = 1
    while hid // p > 14336 or (hid // p) % 8:
        p += 1
    return p


if __name__ == "__main__":
    sys.exit(main())
