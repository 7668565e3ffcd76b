"""End-to-end decode parity on the GPU (benchmark config 1, the tiny checkpoint): the engine behind
the C ABI against yalm's own CPU path — teacher-forced per-step logits (max-abs <= 2e-2 and
cosine >= 0.9999, the north-star gate), free-running greedy tokens, and the KV cache contents."""
import numpy as np
import pytest

import oracle
from yalm_b200 import Config, InferenceMode, InferenceState, Model, YALMData

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 2e-2
LOGIT_COS = 0.9999


def _cos(a, b):
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _make(path, executor, context=0):
    """Engine with the requested executor (yb_create reads YB_EXECUTOR)."""
    import os
    old = os.environ.get("YB_EXECUTOR")
    os.environ["YB_EXECUTOR"] = executor
    try:
        m = Model(YALMData(path), context=context).cuda(0)
    finally:
        if old is None:
            del os.environ["YB_EXECUTOR"]
        else:
            os.environ["YB_EXECUTOR"] = old
    assert m.executor() == executor
    return m


@pytest.fixture(scope="module", params=["persistent", "graph"])
def tiny_model(gpu, tiny_yalm, request):
    m = _make(tiny_yalm, request.param)
    yield m
    m.close()


def test_teacher_forced_logits_vs_reference(tiny_model, tiny_yalm, golden):
    """Every step in OUTPUT_LOGITS mode, fed the golden token stream; compared with yalm's CPU path
    live (oracle/_ref) at every step and with the stored golden logits."""
    m = tiny_model
    ref = oracle.RefModel(tiny_yalm)
    s = InferenceState(m.config)
    seq = list(golden["prompt"]) + list(golden["greedy"])
    steps = list(golden["logit_steps"])
    worst = 0.0
    for step, tok in enumerate(seq):
        m.forward(s, int(tok), step, InferenceMode.OUTPUT_LOGITS)
        got = s.logits().copy()
        exp = ref.forward(int(tok), step, 1)
        d = np.abs(got - exp).max()
        worst = max(worst, d)
        assert d <= LOGIT_MAX_ABS and _cos(got, exp) >= LOGIT_COS, (step, d)
        if step in steps:
            assert np.abs(got - golden["logits"][steps.index(step)]).max() <= LOGIT_MAX_ABS
    assert m.status() == 0
    print("worst max-abs logit diff", worst)


def test_greedy_generation_matches_golden(tiny_model, golden):
    """Prompt in HYDRATE mode except the last token (src/main.cpp:171-177), then 64 free-running
    greedy steps; identical ids to yalm's CPU path."""
    m = tiny_model
    s = InferenceState(m.config)
    prompt = golden["prompt"]
    for pos, tok in enumerate(prompt):
        mode = InferenceMode.OUTPUT_LOGITS if pos + 1 == len(prompt) else InferenceMode.HYDRATE_KV_CACHE
        m.forward(s, int(tok), pos, mode)
    out = []
    pos = len(prompt)
    for _ in range(len(golden["greedy"])):
        tok = int(np.argmax(s.logits()))
        out.append(tok)
        m.forward(s, tok, pos)
        pos += 1
    assert out == [int(t) for t in golden["greedy"]]


def test_kv_cache_matches_reference(tiny_model, golden):
    """After the golden run, the cache slots hold yalm's fp16 values (to one ulp: the reference is
    built with -ffast-math, so its rmsnorm sums are reassociated)."""
    m = tiny_model
    s = InferenceState(m.config)
    seq = list(golden["prompt"]) + list(golden["greedy"])
    for step, tok in enumerate(seq):
        m.forward(s, int(tok), step, InferenceMode.HYDRATE_KV_CACHE)
    m.sync()
    n = len(seq)
    for i, (l, g) in enumerate(zip(golden["kv_layers"], golden["kv_heads"])):
        k, v = m.read_kv(int(l), int(g), 0, n)
        for got, exp in ((k, golden["kv_k"][i]), (v, golden["kv_v"][i])):
            fg, fe = oracle.h2f(got), oracle.h2f(exp)
            assert np.abs(fg - fe).max() <= 2e-3
            assert (got != exp).mean() < 0.2


@pytest.mark.parametrize("executor", ["persistent", "graph"])
def test_ring_buffer_and_sinks_vs_reference(gpu, tiny_yalm, executor):
    """Context 48 (yalm -T 48): 120 steps run past max_seq_len, so the cache wraps in ring order
    and the two sink keys are re-rotated every step (src/infer.cpp:307-325, 489-494)."""
    m = _make(tiny_yalm, executor, context=48)
    ref = oracle.RefModel(tiny_yalm, context=48)
    s = InferenceState(m.config)
    rng = np.random.default_rng(9)
    toks = rng.integers(0, m.config.vocab_size, 120)
    for pos, tok in enumerate(toks):
        m.forward(s, int(tok), pos)
        exp = ref.forward(int(tok), pos, 1)
        got = s.logits()
        assert np.abs(got - exp).max() <= LOGIT_MAX_ABS and _cos(got, exp) >= LOGIT_COS, pos
    k, _ = m.read_kv(1, 0, 0, 48)
    kr, _ = ref.read_kv(1, 0, 0, 48)
    assert np.abs(oracle.h2f(k) - oracle.h2f(kr)).max() <= 5e-3
    m.close()


@pytest.mark.parametrize("executor", ["persistent", "graph"])
def test_context_growth_and_restart_vs_reference(gpu, tiny_yalm, executor):
    """Context 256: positions 0-127 fit one attention CTA (the graph executor replays its one-slice
    attention graph there), 128-255 split the cache over two slices with the log-sum-exp merge,
    256-299 wrap the ring with sinks; then a new sequence restarts at position 0, so the first
    steps see the previous sequence's cache length in the step state until they overwrite it."""
    m = _make(tiny_yalm, executor, context=256)
    ref = oracle.RefModel(tiny_yalm, context=256)
    s = InferenceState(m.config)
    rng = np.random.default_rng(11)
    toks = rng.integers(0, m.config.vocab_size, 312)
    for i, tok in enumerate(toks):
        pos = i if i < 300 else i - 300
        m.forward(s, int(tok), pos)
        exp = ref.forward(int(tok), pos, 1)
        got = s.logits()
        assert np.abs(got - exp).max() <= LOGIT_MAX_ABS and _cos(got, exp) >= LOGIT_COS, (i, pos)
    m.close()


def test_errors_are_returned_not_aborted(tiny_model):
    from yalm_b200 import YalmB200Error
    s = InferenceState(tiny_model.config)
    with pytest.raises(YalmB200Error):
        tiny_model.forward(s, tiny_model.config.vocab_size, 0)
    with pytest.raises(YalmB200Error):
        tiny_model.forward(s, 0, -1)
    with pytest.raises(YalmB200Error):
        tiny_model.read_kv(99, 0, 0, 1)
    # the engine is still usable afterwards
    tiny_model.forward(s, 1, 0)
    assert np.isfinite(s.logits()).all()
