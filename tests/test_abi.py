"""CPU-side checks of the drop-in boundary: the C-ABI library loads without a GPU, exports every
function include/yalm_b200.h declares, and rejects bad configurations before touching CUDA."""
import ctypes
import subprocess

import pytest

from yalm_b200 import _lib, synth
from yalm_b200.codec import YALMData
from yalm_b200.model import Config, Model


def test_library_exports_every_header_symbol():
    names = _lib.header_symbols()
    assert len(names) >= 20
    L = _lib.lib()
    for n in names:
        assert hasattr(L, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # every wrapped signature corresponds to a declared function
    assert set(_lib._SIGS) <= set(names)


def test_library_is_sm100a_only():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    archs = {tok for line in out.splitlines() for tok in line.split(".") if tok.startswith("sm_")}
    assert archs == {"sm_100a"}, archs


def _cfg(**kw):
    c = _lib.yb_config(dim=512, hidden_dim=1408, head_dim=64, n_layers=1, n_heads=8, n_kv_heads=2, vocab_size=64,
                       max_seq_len=64, rotary_dim=64, act=1, n_experts=0, weight_dtype=1, rope_theta=1e6,
                       norm_eps=1e-5, qkv_clip=3e38)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


@pytest.mark.parametrize("kw,code", [({"n_experts": 8}, _lib.YB_E_UNSUPPORTED), ({"weight_dtype": 0}, _lib.YB_E_UNSUPPORTED),
                                     ({"head_dim": 80}, _lib.YB_E_UNSUPPORTED), ({"n_kv_heads": 3}, _lib.YB_E_INVALID),
                                     ({"rotary_dim": 3}, _lib.YB_E_INVALID), ({"dim": 0}, _lib.YB_E_INVALID)])
def test_create_rejects_bad_config_without_gpu(kw, code):
    """Shape/dtype checks happen before any CUDA call and return codes instead of aborting
    (yalm asserts in check_tensor, src/model.cpp:100-117)."""
    w = _lib.yb_weights()
    h = ctypes.c_void_p()
    rc = _lib.lib().yb_create(ctypes.byref(_cfg(**kw)), ctypes.byref(w), 0, 0, 1, ctypes.byref(h))
    assert rc == code
    assert not h.value
    assert _lib.last_error()


def test_tp_config_checks():
    w = _lib.yb_weights()
    h = ctypes.c_void_p()
    rc = _lib.lib().yb_create(ctypes.byref(_cfg()), ctypes.byref(w), 0, 0, 4, ctypes.byref(h))  # 2 kv heads / 4
    assert rc == _lib.YB_E_INVALID


def test_yalm_file_layout_matches_reference_loader(tiny_yalm):
    """The synthetic writer produces files yalm's own loader accepts (oracle/_ref) with the
    metadata Config::from_yalm reads; the Python reader agrees on every tensor."""
    import oracle
    ref = oracle.RefModel(tiny_yalm)
    y = YALMData(tiny_yalm)
    c = Config.from_yalm(y)
    assert (ref.dim, ref.hidden_dim, ref.head_dim, ref.n_layers, ref.n_heads, ref.n_kv_heads, ref.vocab_size,
            ref.max_seq_len, ref.rotary_dim) == (c.dim, c.hidden_dim, c.head_dim, c.n_layers, c.n_heads, c.n_kv_heads,
                                                c.vocab_size, c.max_seq_len, c.rotary_dim)
    assert ref.act_silu == 1 and abs(ref.rope_theta - 1e6) < 1 and abs(ref.norm_eps - 1e-5) < 1e-9
    m = Model(y)  # validates every tensor's dtype and shape
    assert len(m.layers) == c.n_layers
    assert y.tensors["tokenizer.tokens"].dtype == "U8"


def test_yalm_reader_rejects_corrupt_headers(tmp_path):
    p = tmp_path / "bad.yalm"
    p.write_bytes((10 ** 9).to_bytes(8, "little") + b"{}")
    with pytest.raises(ValueError):
        YALMData(str(p))
    import json
    hdr = json.dumps({"__metadata__": {}, "t": {"dtype": "F16", "shape": [4], "data_offsets": [0, 6]}}).encode()
    p.write_bytes(len(hdr).to_bytes(8, "little") + hdr + b"\0" * 8)
    with pytest.raises(ValueError):
        YALMData(str(p))  # 4 x F16 is 8 bytes, offsets say 6


def test_synth_is_deterministic(tmp_path):
    a = synth.write_yalm(str(tmp_path / "a.yalm"), synth.shape_with("tiny", n_layers=1, vocab_size=512), seed=3)
    b = synth.write_yalm(str(tmp_path / "b.yalm"), synth.shape_with("tiny", n_layers=1, vocab_size=512), seed=3)
    assert open(a, "rb").read() == open(b, "rb").read()
    y = YALMData(a)
    w = y.tensors["model.layers.0.mlp.w1.weight"].array(y).view("float16").astype("float64")
    assert abs(w.std() - 0.02) < 0.001 and abs(w.mean()) < 0.001
