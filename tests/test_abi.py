"""CPU-side checks of the drop-in boundary: the C-ABI library loads without a GPU, exports every
function include/yalm_b200.h declares, and rejects bad configurations, NULL handles and impossible
shapes with error codes before touching CUDA."""
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


def test_null_engine_is_an_error_not_a_crash():
    """Every entry point that takes an engine handle returns YB_E_INVALID for NULL (yalm would
    dereference a null Model and crash); the query functions return their neutral value."""
    L = _lib.lib()
    out_i, out_f = ctypes.c_int(), ctypes.c_float()
    toks = (ctypes.c_int * 2)(1, 2)
    calls = {
        "yb_forward": lambda: L.yb_forward(None, 1, 0, 1, None),
        "yb_forward_async": lambda: L.yb_forward_async(None, 1, 0, 0),
        "yb_forward_sample": lambda: L.yb_forward_sample(None, 1, 0, 0.0, 0.0, ctypes.byref(out_i)),
        "yb_forward_prob": lambda: L.yb_forward_prob(None, 1, 0, 1, ctypes.byref(out_f)),
        "yb_prefill": lambda: L.yb_prefill(None, toks, 2, 0, None),
        "yb_sync": lambda: L.yb_sync(None),
        "yb_read_kv": lambda: L.yb_read_kv(None, 0, 0, 0, 1, None, None),
        "yb_clear_status": lambda: L.yb_clear_status(None),
        "yb_tp_export": lambda: L.yb_tp_export(None, None, 0, None),
        "yb_tp_import": lambda: L.yb_tp_import(None, None, 0),
        "yb_profile_kernel": lambda: L.yb_profile_kernel(None, 0, 1, ctypes.byref(out_f)),
    }
    for name, call in calls.items():
        assert call() == _lib.YB_E_INVALID, name
        assert _lib.last_error(), name
    assert L.yb_logits_dev(None) is None
    assert L.yb_stream(None) is None
    assert L.yb_status(None) == 0
    assert L.yb_executor(None) == 0
    L.yb_destroy(None)  # a no-op


def test_kernel_entry_points_check_arguments_before_cuda():
    """The device-pointer and test-hook entry points reject NULL buffers and impossible shapes with
    YB_E_INVALID before any CUDA call (so without a GPU too); a dummy non-NULL address is never
    dereferenced on these paths."""
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    bad = {
        "gemv null y": lambda: L.yb_gemv_dev(None, p, p, 8, 8, None, 0.0, 0, None),
        "gemv cols % 8": lambda: L.yb_gemv_dev(p, p, p, 8, 12, None, 0.0, 0, None),
        "gemv rows 0": lambda: L.yb_gemv_dev(p, p, p, 0, 8, None, 0.0, 0, None),
        "gateup null w": lambda: L.yb_gateup_dev(p, p, None, 8, 8, None, 0.0, 1, None),
        "gateup dim % 8": lambda: L.yb_gateup_dev(p, p, p, 8, 20, None, 0.0, 1, None),
        "qkv odd head_dim": lambda: L.yb_qkv_dev(p, p, p, p, p, p, 1e-5, 64, 2, 1, 31, 30, 16, 0, 0, 0, 3e38, p, None),
        "qkv rotary > head_dim": lambda: L.yb_qkv_dev(p, p, p, p, p, p, 1e-5, 64, 2, 1, 32, 34, 16, 0, 0, 0, 3e38, p, None),
        "qkv kv_pos past the cache": lambda: L.yb_qkv_dev(p, p, p, p, p, p, 1e-5, 64, 2, 1, 32, 32, 16, 16, 16, 0, 3e38, p, None),
        "qkv sink past kv_pos": lambda: L.yb_qkv_dev(p, p, p, p, p, p, 1e-5, 64, 2, 1, 32, 32, 16, 3, 3, 4, 3e38, p, None),
        "qkv null inv_freq": lambda: L.yb_qkv_dev(p, p, p, p, p, p, 1e-5, 64, 2, 1, 32, 32, 16, 0, 0, 0, 3e38, None, None),
        "attention kv_len 0": lambda: L.yb_attention_dev(p, p, p, p, 8, 2, 64, 128, 0, p, None),
        "attention kv_len > cache": lambda: L.yb_attention_dev(p, p, p, p, 8, 2, 64, 128, 129, p, None),
        "attention null scratch": lambda: L.yb_attention_dev(p, p, p, p, 8, 2, 64, 128, 64, None, None),
        "noalloc null q": lambda: L.yb_attention_dev_noalloc(p, None, p, p, 8, 2, 64, 128, 64, None),
        "noalloc kv_len > cache": lambda: L.yb_attention_dev_noalloc(p, p, p, p, 8, 2, 64, 128, 200, None),
        "matmul n % 8": lambda: L.yb_matmul(p, p, p, 12, 4),
        "mha null k": lambda: L.yb_mha(p, None, None, p, p, 64, 4, 8, 8, 2),
        "ffn hidden % 8": lambda: L.yb_ffn(p, p, p, p, p, 12, 8, 1),
        "prefill attention null out": lambda: L.yb_prefill_attention_dev(None, p, p, p, 8, 0, 8, 2, 64, 64, None),
        "prefill gemm bad epilogue": lambda: L.yb_prefill_gemm_dev(p, None, p, p, 128, 256, 64, 99, 256, None),
    }
    for name, call in bad.items():
        assert call() == _lib.YB_E_INVALID, name
        assert _lib.last_error(), name


def test_noalloc_attention_size_limit_checked_on_the_host():
    """The allocation-free attention rejects a shape whose scratch exceeds its fixed device array
    before touching the GPU, naming both sizes; the limit is the header's constant."""
    L = _lib.lib()
    limit = 4 << 20
    p = ctypes.c_void_p(16)
    # 512 heads of 128 over 64 kv heads need more than 4 MiB of cluster records
    assert L.yb_attention_scratch_bytes(512, 64, 128, 4096) > limit
    assert L.yb_attention_scratch_bytes(256, 32, 128, 32768) <= limit
    assert L.yb_attention_scratch_bytes(32, 8, 128, 4096) <= limit
    assert L.yb_attention_scratch_bytes(64, 8, 128, 32768) <= limit
    rc = L.yb_attention_dev_noalloc(p, p, p, p, 512, 64, 128, 4096, 100, None)
    assert rc == _lib.YB_E_INVALID
    msg = _lib.last_error()
    assert "exceeds" in msg and str(limit) in msg
    assert str(L.yb_attention_scratch_bytes(512, 64, 128, 4096)) in msg  # the size the shape needs
    src = open(_lib.HEADER).read()
    assert "#define YB_ATTENTION_NOALLOC_SCRATCH_BYTES (4u << 20)" in src


def test_no_cpu_fallback_without_a_gpu(tiny_yalm):
    """Without a GPU the engine refuses to start (YB_E_CUDA from yb_create) instead of computing
    anywhere else: the product path has no CPU fallback."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; this checks the behaviour without one")
    m = Model(YALMData(tiny_yalm))
    with pytest.raises(_lib.YalmB200Error) as ei:
        m.cuda(0)
    assert ei.value.code == _lib.YB_E_CUDA
