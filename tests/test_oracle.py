"""Pins the CPU oracle: the C restatement against yalm's own CPU path (oracle/_ref) and against the
golden vectors generated from it, plus yalm's known-answer attention test."""
import numpy as np
import pytest

import oracle
from yalm_b200 import Config, YALMData


def test_half_conversions_exhaustive():
    """fp16 <-> fp32 round trip over every non-NaN bit pattern, and rounding against numpy."""
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    f = oracle.h2f(bits)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(f[~nan], ref[~nan])
    assert np.isnan(f[nan]).all()
    back = oracle.f2h(f[~nan])
    assert np.array_equal(back, bits[~nan])
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 1e3, 7e4)])
    assert np.array_equal(oracle.f2h(x), x.astype(np.float16).view(np.uint16))


def test_matmul_bit_exact_vs_reference():
    """The restated fp16 matvec reproduces yalm's AVX2/F16C summation order bit for bit."""
    rng = np.random.default_rng(1)
    for n, d in ((512, 64), (1408, 33), (4096, 17)):
        w = (rng.standard_normal((d, n)) * 0.02).astype(np.float16).view(np.uint16)
        x = rng.standard_normal(n).astype(np.float32)
        ref = np.zeros(d, np.float32)
        oracle.ref_lib().ref_matmul_f16(ref.ctypes.data, x.ctypes.data, w.ctypes.data, n, d)
        assert np.array_equal(oracle.matmul_f16(x, w), ref)


def test_attn_known_answer():
    """yalm's test_attn KAT (src/test.cpp:67-125): GQA 2 q heads / 1 kv head, head_dim 3, seq 4,
    K placed in the 16-tiled layout; one-hot attention picks the matching value row."""
    seq, hd, nh, nkv = 4, 3, 2, 1
    q = np.array([0., 1e4, 0., 0., 0., 1e4], np.float32)
    kb = np.zeros(16 * seq, np.uint16)
    one, mone = np.float16(1).view(np.uint16), np.float16(-1).view(np.uint16)
    kb[0], kb[17], kb[34], kb[48] = one, one, one, mone
    vb = np.array([1, 0, 0, -1, 0, 1, 0, 0, 0, 0, 1, 0], np.float16).view(np.uint16)
    out_c = oracle.mha(q, kb, vb, hd, seq, seq, nh, nkv)
    assert np.allclose(out_c, [0, 1, 0, 0, 0, 1], atol=1e-4)
    out_r = np.zeros(6, np.float32)
    att = np.zeros(nh * seq, np.float32)
    oracle.ref_lib().ref_mha(out_r.ctypes.data, att.ctypes.data, kb.ctypes.data, vb.ctypes.data, q.ctypes.data,
                             hd, seq, seq, nh, nkv)
    assert np.allclose(att.reshape(nh, seq), [[0, 1, 0, 0], [0, 0, 1, 0]], atol=1e-4)
    assert np.allclose(out_r, out_c, atol=1e-6)


def test_positions_ring_buffer():
    """kv_sink / kv_pos / kv_len past the context (src/infer.cpp:489-494)."""
    from yalm_b200.model import positions
    L = oracle.c_lib()
    import ctypes
    for msl in (8, 1024):
        for pos in list(range(0, 3 * msl)) + [10 * msl + 5]:
            a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
            L.yo_positions(pos, msl, ctypes.addressof(a), ctypes.addressof(b), ctypes.addressof(c))
            assert positions(pos, msl) == (a.value, b.value, c.value)
            if pos >= msl:
                assert 2 <= b.value < msl and c.value == msl


def test_restatement_vs_reference_tiny(tiny_yalm):
    """Whole decode steps: C restatement vs yalm's CPU path on the tiny checkpoint."""
    y = YALMData(tiny_yalm)
    c = Config.from_yalm(y)
    ref = oracle.RefModel(tiny_yalm)
    cm = oracle.CModel(y, c)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, c.vocab_size, 24)
    for pos, t in enumerate(toks):
        a = ref.forward(int(t), pos, 1)
        b = cm.forward(int(t), pos, 1)
        assert np.abs(a - b).max() < 2e-3
        cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        assert cos > 0.99999
    for l in range(c.n_layers):
        k1, v1 = ref.read_kv(l, 0, 0, len(toks))
        k2, v2 = cm.read_kv(l, 0, 0, len(toks))
        assert np.abs(oracle.h2f(k1) - oracle.h2f(k2)).max() < 5e-3
        assert np.abs(oracle.h2f(v1) - oracle.h2f(v2)).max() < 5e-3


def test_restatement_vs_reference_gqa4_ring(tmp_path):
    """A second architecture (head_dim 128, 4 query heads per kv head, 2 layers) opened with a
    32-slot context and run to position 80: whole steps past the context, where yalm's CPU path
    writes the ring and re-rotates the sink keys (src/infer.cpp:296-325), agree between the C
    restatement and yalm's own code."""
    from yalm_b200 import synth
    shape = synth.shape_with("tiny", dim=1024, n_heads=8, n_kv_heads=2, head_dim=128, hidden_dim=2048,
                             n_layers=2, vocab_size=1024)
    path = synth.write_yalm(str(tmp_path / "gqa4.yalm"), shape, seed=11)
    ctx = 32
    y = YALMData(path)
    c = Config.from_yalm(y, context=ctx)
    assert c.max_seq_len == ctx and c.n_heads // c.n_kv_heads == 4 and c.head_dim == 128
    ref = oracle.RefModel(path, context=ctx)
    cm = oracle.CModel(y, c)
    rng = np.random.default_rng(17)
    toks = rng.integers(0, c.vocab_size, 80)
    for pos, t in enumerate(toks):
        a = ref.forward(int(t), pos, 1)
        b = cm.forward(int(t), pos, 1)
        assert np.abs(a - b).max() < 2e-3, pos
        assert float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))) > 0.99999, pos
    for l in range(c.n_layers):
        for h in range(c.n_kv_heads):
            k1, v1 = ref.read_kv(l, h, 0, ctx)
            k2, v2 = cm.read_kv(l, h, 0, ctx)
            assert np.abs(oracle.h2f(k1) - oracle.h2f(k2)).max() < 5e-3
            assert np.abs(oracle.h2f(v1) - oracle.h2f(v2)).max() < 5e-3


def test_restatement_vs_reference_gelu(tmp_path):
    """The GELU activation (yalm's default act_type, src/model.cpp:41-48; tanh form, src/infer.cpp:189-191)
    on a 2-layer tiny checkpoint: whole steps of the C restatement against yalm's CPU path."""
    from yalm_b200 import synth
    path = synth.write_yalm(str(tmp_path / "gelu.yalm"), synth.shape_with("tiny", n_layers=2, act_type="gelu"),
                            seed=13)
    y = YALMData(path)
    c = Config.from_yalm(y)
    assert int(c.act) == 0  # GELU
    ref = oracle.RefModel(path)
    cm = oracle.CModel(y, c)
    rng = np.random.default_rng(19)
    for pos, t in enumerate(rng.integers(0, c.vocab_size, 16)):
        a = ref.forward(int(t), pos, 1)
        b = cm.forward(int(t), pos, 1)
        assert np.abs(a - b).max() < 2e-3, pos
        assert float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))) > 0.99999, pos


def test_restatement_vs_golden(tiny_yalm, golden):
    """The C restatement replays the golden run (generated by yalm's own CPU path)."""
    y = YALMData(tiny_yalm)
    c = Config.from_yalm(y)
    import zlib
    for name, crc in zip(golden["weight_crc_names"], golden["weight_crc"]):
        t = y.tensors[str(name)]
        assert zlib.crc32(bytes(y.buf[t.offset:t.offset + min(4096, t.size)])) == int(crc), name
    cm = oracle.CModel(y, c)
    prompt, greedy = golden["prompt"], golden["greedy"]
    steps = list(golden["logit_steps"])
    seq = list(prompt) + list(greedy)
    got_greedy = []
    for step in range(len(prompt) + len(greedy)):
        lg = cm.forward(int(seq[step]), step, 1)
        if step in steps:
            exp = golden["logits"][steps.index(step)]
            assert np.abs(lg - exp).max() < 2e-3, step
        if step >= len(prompt) - 1 and len(got_greedy) < len(greedy):
            got_greedy.append(int(np.argmax(lg)))
    # the restatement follows the teacher-forced stream; its argmax agrees except at recorded near-ties
    gaps = golden["top2_gap"][len(prompt) - 1:len(prompt) - 1 + len(greedy)]
    mism = [i for i, (a, b) in enumerate(zip(got_greedy, greedy)) if a != b]
    assert all(gaps[i] < 2e-3 for i in mism), (mism, gaps[mism] if mism else None)


def test_golden_fixture_regenerates_from_the_reference(tiny_yalm, golden):
    """tests/golden/make_golden.py run again on yalm's CPU path (oracle/_ref) reproduces the
    committed fixture: same prompt, greedy ids, weight CRCs and KV bits, and logits to float
    rounding."""
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    fresh = mg.generate(tiny_yalm)
    for key in ("prompt", "greedy", "logit_steps", "kv_layers", "kv_heads", "weight_crc"):
        assert np.array_equal(fresh[key], golden[key]), key
    assert list(fresh["weight_crc_names"]) == [str(n) for n in golden["weight_crc_names"]]
    assert np.abs(fresh["logits"] - golden["logits"]).max() < 1e-5
    assert np.abs(fresh["top2_gap"] - golden["top2_gap"]).max() < 1e-5
    k_diff = np.count_nonzero(fresh["kv_k"] != golden["kv_k"])
    v_diff = np.count_nonzero(fresh["kv_v"] != golden["kv_v"])
    assert k_diff == 0 and v_diff == 0, (k_diff, v_diff)
