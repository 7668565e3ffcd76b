"""fp8 (E5M2) weights — the dtype yalm's converter writes for `fp8` (convert.py:160, a plain cast to
float8_e5m2) and yalm's runtime rejects (src/model.cpp:61-70).  An E5M2 value is the top byte of
the fp16 with the same value, so the engine on an fp8 checkpoint must compute what yalm's fp16 CPU
path computes on the checkpoint's fp16 twin (every weight byte b stored as the fp16 b << 8).

CPU: the synthetic fp8 writer rounds like torch's float8_e5m2 cast, its bytes are the rounded fp16
values the fp16 writer produces, the twin expands them exactly and loads in yalm's CPU path.
GPU: teacher-forced logits (max-abs <= 2e-2, cosine >= 0.9999) and greedy ids against the twin."""
import os
import tempfile

import numpy as np
import pytest

LOGIT_MAX_ABS = 2e-2
LOGIT_COS = 0.9999


@pytest.fixture(scope="module")
def fp8_pair():
    from yalm_b200 import synth
    d = tempfile.gettempdir()
    shape = synth.shape_with("tiny", dtype="fp8")
    fp8 = synth.write_yalm(os.path.join(d, "yalm_tiny_fp8_seed0.yalm"), shape, seed=0)
    twin = synth.expand_fp8_to_fp16(fp8, os.path.join(d, "yalm_tiny_fp8_seed0_twin16.yalm"))
    return fp8, twin


def test_e5m2_rounding_matches_torch():
    import torch
    from yalm_b200 import synth
    h = np.random.default_rng(0).integers(0, 65536, 100000).astype(np.uint16)
    h = h[(h & 0x7C00) != 0x7C00]
    ref = torch.from_numpy(h.view(np.float16).astype(np.float32)).to(torch.float8_e5m2).view(torch.uint8).numpy()
    assert np.array_equal(synth.e5m2_from_f16_bits(h), ref)


def test_fp8_writer_and_twin(fp8_pair, tiny_yalm):
    from yalm_b200 import YALMData
    fp8, twin = fp8_pair
    y8, y16, yref = YALMData(fp8), YALMData(twin), YALMData(tiny_yalm)
    assert y8.metadata["dtype"] == "fp8" and y16.metadata["dtype"] == "fp16"
    for name in ("model.embed.weight", "model.layers.1.attn.wq.weight", "model.layers.3.mlp.w2.weight"):
        b = y8.tensors[name].array(y8)
        assert y8.tensors[name].dtype == "F8_E5M2" and b.dtype == np.uint8
        # same generator stream as the fp16 file, rounded to E5M2 ...
        from yalm_b200 import synth
        f16 = yref.tensors[name].array(yref).view(np.uint16)
        assert np.array_equal(b.reshape(-1), synth.e5m2_from_f16_bits(f16.reshape(-1)))
        # ... and the twin holds exactly those values as fp16
        t = y16.tensors[name].array(y16).view(np.uint16)
        assert np.array_equal(t.reshape(-1), b.reshape(-1).astype(np.uint16) << 8)
    assert np.array_equal(y16.tensors["model.norm.weight"].array(y16), y8.tensors["model.norm.weight"].array(y8))


def test_fp8_config_and_reference_twin(fp8_pair):
    import oracle
    from yalm_b200 import Config, Model, YALMData
    fp8, twin = fp8_pair
    c = Config.from_yalm(YALMData(fp8))
    assert c.weight_dtype == "F8_E5M2" and c.to_c().weight_dtype == 3
    assert c.weight_bytes_per_token() < Config.from_yalm(YALMData(twin)).weight_bytes_per_token()
    Model(YALMData(fp8))  # every tensor passes the shape / dtype checks
    lg = oracle.RefModel(twin).forward(1, 0, 1)
    assert np.isfinite(lg).all()


@pytest.mark.gpu
@pytest.mark.parametrize("executor", ["graph"])
def test_fp8_engine_matches_reference_on_twin(gpu, fp8_pair, executor):
    import oracle
    from yalm_b200 import InferenceState, Model, YALMData
    fp8, twin = fp8_pair
    m = Model(YALMData(fp8)).cuda(0)
    ref = oracle.RefModel(twin)
    s = InferenceState(m.config)
    rng = np.random.default_rng(8)
    toks = [int(t) for t in rng.integers(0, m.config.vocab_size, 48)]
    worst = 0.0
    for pos, tok in enumerate(toks):
        m.forward(s, tok, pos)
        got, exp = s.logits(), ref.forward(tok, pos, 1)
        d = float(np.abs(got - exp).max())
        worst = max(worst, d)
        cos = float(got @ exp / (np.linalg.norm(got) * np.linalg.norm(exp)))
        assert d <= LOGIT_MAX_ABS and cos >= LOGIT_COS, (pos, d, cos)
    # greedy continuation from the last prompt token, compared while the reference's top-2 gap is
    # above the logit tolerance
    ids_ref, gaps, lg = [], [], exp
    ids = []
    tok_g = m.forward_sample(toks[-1], len(toks) - 1)
    for i in range(24):
        top2 = np.sort(lg)[-2:]
        gaps.append(float(top2[1] - top2[0]))
        ids_ref.append(int(np.argmax(lg)))
        ids.append(tok_g)
        lg = ref.forward(ids_ref[-1], len(toks) + i, 1)
        tok_g = m.forward_sample(tok_g, len(toks) + i)
    n_sure = next((i for i, gp in enumerate(gaps) if gp < 2e-3), len(gaps))
    assert n_sure >= 8 and ids[:n_sure] == ids_ref[:n_sure]
    assert m.status() == 0
    m.close()
    print("fp8 worst max-abs logit diff", worst, "greedy compared", n_sure)


@pytest.mark.gpu
def test_fp8_7b_shapes_match_reference_on_twin(gpu):
    """The Mistral-7B architecture cut to 2 layers, fp8: every matvec shape `bench.py --dtype fp8`
    runs (QKV 6144 x 4096 and wo 4096 x 4096 as two 2048-column chunks per row group, gate/up
    28672 x 4096, w2 4096 x 14336 as seven chunks, the 32000-row classifier) against yalm's fp16 CPU
    path on the fp16 twin, teacher-forced, with the north star's logit gate."""
    import oracle
    from yalm_b200 import InferenceState, Model, YALMData, synth
    shape = synth.shape_with("mistral-7b", n_layers=2, dtype="fp8")
    d = synth.scratch_dir(3 * synth.file_bytes(shape))
    fp8 = synth.write_yalm(os.path.join(d, "yalm_mistral-7b_l2_fp8_seed0.yalm"), shape, seed=0)
    twin = synth.expand_fp8_to_fp16(fp8, os.path.join(d, "yalm_mistral-7b_l2_fp8_seed0_twin16.yalm"))
    m = Model(YALMData(fp8)).cuda(0)
    ref = oracle.RefModel(twin)
    s = InferenceState(m.config)
    rng = np.random.default_rng(78)
    toks = [int(t) for t in rng.integers(0, m.config.vocab_size, 20)]
    worst = 0.0
    for pos, tok in enumerate(toks):
        m.forward(s, tok, pos)
        got, exp = s.logits(), ref.forward(tok, pos, 1)
        dmax = float(np.abs(got - exp).max())
        worst = max(worst, dmax)
        cos = float(got @ exp / (np.linalg.norm(got) * np.linalg.norm(exp)))
        assert dmax <= LOGIT_MAX_ABS and cos >= LOGIT_COS, (pos, dmax, cos)
        assert int(np.argmax(got)) == int(np.argmax(exp)) or np.sort(exp)[-1] - np.sort(exp)[-2] < 2e-3, pos
    assert m.status() == 0
    m.close()
    ref.close()
    print("fp8 7B-shape worst max-abs logit diff", worst)


@pytest.mark.gpu
def test_fp8_tensor_core_matvec_matches_reference_on_twin(gpu):
    """The tensor-core fp8 matvec (YB_TUNE=fp8mma=1: weights re-laid at upload into 16-row groups,
    mma.sync with x as fp16 value + remainder columns), off by default, run in a child process (the
    tuning is read once per process) through the 7B-shape check above."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, YB_TUNE="fp8mma=1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu",
                        os.path.abspath(__file__) + "::test_fp8_7b_shapes_match_reference_on_twin"],
                       cwd=root, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-2000:])
