"""Batched prefill (yb_prefill) against yalm's CPU path: the prompt's last logits against the
golden run (max-abs <= 2e-2, cosine >= 0.9999), the KV cache the batched pass leaves against the
reference's (fp16 activations: within 1e-2), a prompt split in two batched calls (attention over
cached and new slots), greedy decoding after the batched prompt equal to the golden ids, and the
per-token fallback for a one-token prompt."""
import numpy as np
import pytest

import oracle
from yalm_b200 import InferenceState, Model, YALMData

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 2e-2
LOGIT_COS = 0.9999


def _cos(a, b):
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.fixture(scope="module")
def model(gpu, tiny_yalm):
    m = Model(YALMData(tiny_yalm)).cuda(0)
    yield m
    m.close()


def _golden_logits(golden, step):
    return golden["logits"][list(golden["logit_steps"]).index(step)]


def test_prompt_logits_and_kv(model, golden):
    prompt = [int(t) for t in golden["prompt"]]
    s = InferenceState(model.config)
    model.prefill(prompt, 0, s)
    exp = _golden_logits(golden, len(prompt) - 1)
    got = s.logits()
    d = float(np.abs(got - exp).max())
    assert d <= LOGIT_MAX_ABS and _cos(got, exp) >= LOGIT_COS, d
    n = len(prompt)
    for i, (l, g) in enumerate(zip(golden["kv_layers"], golden["kv_heads"])):
        k, v = model.read_kv(int(l), int(g), 0, n)
        for got_kv, exp_kv in ((k, golden["kv_k"][i][:n]), (v, golden["kv_v"][i][:n])):
            assert np.abs(oracle.h2f(got_kv) - oracle.h2f(exp_kv)).max() <= 1e-2
    print("prefill last-token max-abs logit diff", d)


def test_split_prompt_and_greedy(model, golden):
    prompt = [int(t) for t in golden["prompt"]]
    s = InferenceState(model.config)
    model.prefill(prompt[:20], 0)
    model.prefill(prompt[20:], 20, s)
    exp = _golden_logits(golden, len(prompt) - 1)
    assert np.abs(s.logits() - exp).max() <= LOGIT_MAX_ABS and _cos(s.logits(), exp) >= LOGIT_COS
    # greedy continuation (first id from the prompt's logits)
    tok = int(np.argmax(s.logits()))
    out = []
    for i in range(len(golden["greedy"])):
        out.append(tok)
        tok = model.forward_sample(tok, len(prompt) + i)
    assert out == [int(t) for t in golden["greedy"]]
    assert model.status() == 0


def test_one_token_prompt_uses_steps(model, tiny_yalm):
    s = InferenceState(model.config)
    model.prefill([7], 0, s)
    exp = oracle.RefModel(tiny_yalm).forward(7, 0, 1)
    assert np.abs(s.logits() - exp).max() <= LOGIT_MAX_ABS
