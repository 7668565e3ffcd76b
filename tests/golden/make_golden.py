"""Generates tests/golden/tiny_golden.npz from yalm's own CPU path (oracle/_ref, built from the
reference sources) on the seeded synthetic tiny checkpoint (config 1 of the benchmark configs).

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


if __name__ == "__main__":
    import tempfile
    path = os.path.join(tempfile.gettempdir(), "yalm_tiny_seed0.yalm")
    synth.write_yalm(path, synth.SHAPES["tiny"], seed=0)
    out = generate(path)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tiny_golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes; greedy", out["greedy"][:16], "min top2 gap",
          float(out["top2_gap"].min()))
