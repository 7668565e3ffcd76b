"""Generates tests/golden/tiny_golden.npz from yalm's own CPU path (oracle/_ref, built from the
reference sources) on the seeded synthetic tiny checkpoint (config 1 of the benchmark configs), and
tests/golden/kv8_golden.npz (generate_kv8) on a small 8-kv-head checkpoint for the tensor-parallel
check of bench.py.

Contents:
  prompt          32 token ids, uniform in [0, 4096), numpy default_rng(1234)
  greedy          64 greedy ids decoded after the prompt (argmax of the logits)
  logit_steps     indices of the steps whose full logits are stored
  logits          float32 [len(logit_steps), 4096]
  top2_gap        float32 [96]: top-1 minus top-2 logit at every step (near-tie audit)
  kv_layers/kv_heads/kv_k/kv_v   fp16 bits of slots [0, 96) for a few (layer, kv head) pairs
  weight_crc      crc32 of the first 4096 bytes of every tensor (pins the synthetic generator)

Every step calls Model::forward with OUTPUT_LOGITS (as yalm's perplexity mode does).
Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from yalm_b200 import synth  # noqa: E402
from yalm_b200.codec import YALMData  # noqa: E402

N_PROMPT, N_DECODE = 32, 64
LOGIT_STEPS = [0, 1, 7, 31, 32, 47, 63, 95]
KV_PAIRS = [(0, 0), (1, 1), (3, 0), (3, 1)]


def generate(path: str):
    ref = oracle.RefModel(path)
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, ref.vocab_size, N_PROMPT).astype(np.int32)
    logits_keep, gaps, greedy = [], [], []
    tok = None
    for step in range(N_PROMPT + N_DECODE):
        tok = int(prompt[step]) if step < N_PROMPT else tok
        lg = ref.forward(tok, step, 1)
        srt = np.sort(lg)
        gaps.append(srt[-1] - srt[-2])
        if step in LOGIT_STEPS:
            logits_keep.append(lg.copy())
        if step >= N_PROMPT - 1 and len(greedy) < N_DECODE:
            tok = int(np.argmax(lg))
            greedy.append(tok)
    kv_k, kv_v = [], []
    for l, g in KV_PAIRS:
        k, v = ref.read_kv(l, g, 0, N_PROMPT + N_DECODE)
        kv_k.append(k)
        kv_v.append(v)
    y = YALMData(path)
    crc = {n: zlib.crc32(bytes(y.buf[t.offset:t.offset + min(4096, t.size)])) for n, t in y.tensors.items()}
    names = sorted(crc)
    return dict(prompt=prompt, greedy=np.array(greedy, np.int32), logit_steps=np.array(LOGIT_STEPS, np.int32),
                logits=np.stack(logits_keep).astype(np.float32), top2_gap=np.array(gaps, np.float32),
                kv_layers=np.array([p[0] for p in KV_PAIRS], np.int32),
                kv_heads=np.array([p[1] for p in KV_PAIRS], np.int32),
                kv_k=np.stack(kv_k), kv_v=np.stack(kv_v),
                weight_crc_names=np.array(names), weight_crc=np.array([crc[n] for n in names], np.uint32))


# The tensor-parallel check of bench.py --gpus N: a small checkpoint with 8 kv heads (so it splits 8
# ways), forced token ids with the reference's logits at a few steps, and a greedy run.
KV8_SHAPE = dict(dim=1024, n_heads=16, n_kv_heads=8, head_dim=64, hidden_dim=2816)
KV8_SEED = 3
KV8_FORCED, KV8_PROMPT, KV8_GREEDY = 24, 16, 16
KV8_LOGIT_STEPS = [0, 5, 11, 17, 22, 23]


def kv8_shape():
    return synth.shape_with("tiny", **KV8_SHAPE)


def generate_kv8(path: str):
    """kv8_golden.npz:
      shape_json, seed  the checkpoint (shape overrides of the tiny config, synthetic seed)
      forced          24 token ids (default_rng(8)), each step in OUTPUT_LOGITS mode from position 0
      logit_steps     steps whose logits are stored;  logits  float32 [len(logit_steps), 4096]
      prompt          16 token ids; greedy: 16 greedy ids after it;  greedy_gap: top-1 minus top-2
                      logit before each greedy id
      weight_crc      crc32 of the first 4096 bytes of every tensor (pins the synthetic generator)"""
    ref = oracle.RefModel(path)
    rng = np.random.default_rng(8)
    forced = rng.integers(0, ref.vocab_size, KV8_FORCED).astype(np.int32)
    prompt = rng.integers(0, ref.vocab_size, KV8_PROMPT).astype(np.int32)
    keep = []
    for pos, tok in enumerate(forced):
        lg = ref.forward(int(tok), pos, 1)
        if pos in KV8_LOGIT_STEPS:
            keep.append(lg.copy())
    ref.close()
    ref = oracle.RefModel(path)
    lg = None
    for pos, tok in enumerate(prompt):
        lg = ref.forward(int(tok), pos, 1 if pos + 1 == len(prompt) else 0)
    greedy, gaps = [], []
    for i in range(KV8_GREEDY):
        srt = np.sort(lg)
        gaps.append(srt[-1] - srt[-2])
        tok = int(np.argmax(lg))
        greedy.append(tok)
        lg = ref.forward(tok, len(prompt) + i, 1)
    y = YALMData(path)
    crc = {n: zlib.crc32(bytes(y.buf[t.offset:t.offset + min(4096, t.size)])) for n, t in y.tensors.items()}
    names = sorted(crc)
    import json
    return dict(shape_json=np.array(json.dumps(KV8_SHAPE, sort_keys=True)), seed=np.array(KV8_SEED, np.int32),
                forced=forced, logit_steps=np.array(KV8_LOGIT_STEPS, np.int32), logits=np.stack(keep).astype(np.float32),
                prompt=prompt, greedy=np.array(greedy, np.int32), greedy_gap=np.array(gaps, np.float32),
                weight_crc_names=np.array(names), weight_crc=np.array([crc[n] for n in names], np.uint32))


if __name__ == "__main__":
    import tempfile
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(tempfile.gettempdir(), "yalm_tiny_seed0.yalm")
    synth.write_yalm(path, synth.SHAPES["tiny"], seed=0)
    out = generate(path)
    dst = os.path.join(here, "tiny_golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes; greedy", out["greedy"][:16], "min top2 gap",
          float(out["top2_gap"].min()))
    path = os.path.join(tempfile.gettempdir(), f"yalm_kv8_seed{KV8_SEED}.yalm")
    synth.write_yalm(path, kv8_shape(), seed=KV8_SEED)
    out = generate_kv8(path)
    dst = os.path.join(here, "kv8_golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes; greedy", out["greedy"], "min gap", float(out["greedy_gap"].min()))
