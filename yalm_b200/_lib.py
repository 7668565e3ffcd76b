"""ctypes binding of libyalm_b200.so (the C ABI in include/yalm_b200.h).

Every wrapper raises YalmB200Error with the library's message when an entry point returns a
non-zero code.  The library must have been built (python -m yalm_b200.build); importing this module
never falls back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libyalm_b200.so")
HEADER = os.path.join(ROOT, "include", "yalm_b200.h")

YB_OK = 0
YB_E_INVALID = -1
YB_E_CUDA = -2
YB_E_TIMEOUT = -3
YB_E_UNSUPPORTED = -4
MODE_HYDRATE = 0
MODE_LOGITS = 1


class YalmB200Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"yalm_b200 error {code}: {msg}")
        self.code = code


class yb_config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden_dim", "head_dim", "n_layers", "n_heads", "n_kv_heads",
                                            "vocab_size", "max_seq_len", "rotary_dim", "act", "n_experts",
                                            "weight_dtype")] + \
               [(n, ctypes.c_float) for n in ("rope_theta", "norm_eps", "qkv_clip")]


_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)


class yb_weights(ctypes.Structure):
    _fields_ = [("token_embedding_table", _P), ("rms_final_weight", _P), ("wcls", _P),
                ("rms_att_weight", _PP), ("rms_ffn_weight", _PP), ("wq", _PP), ("wk", _PP), ("wv", _PP),
                ("wo", _PP), ("w1", _PP), ("w2", _PP), ("w3", _PP)]


_lib = None
_I, _F, _S = ctypes.c_int, ctypes.c_float, ctypes.c_size_t

_SIGS = {
    "yb_create": (_I, [ctypes.POINTER(yb_config), ctypes.POINTER(yb_weights), _I, _I, _I, ctypes.POINTER(_P)]),
    "yb_forward": (_I, [_P, _I, _I, _I, _P]),
    "yb_forward_sample": (_I, [_P, _I, _I, ctypes.c_float, ctypes.c_float, _P]),
    "yb_forward_prob": (_I, [_P, _I, _I, _I, _P]),
    "yb_prefill_gemm_dev": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "yb_prefill_attention_dev": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "yb_prefill": (_I, [_P, _P, _I, _I, _P]),
    "yb_forward_async": (_I, [_P, _I, _I, _I]),
    "yb_sync": (_I, [_P]),
    "yb_logits_dev": (_P, [_P]),
    "yb_stream": (_P, [_P]),
    "yb_read_kv": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "yb_status": (ctypes.c_uint, [_P]),
    "yb_executor": (_I, [_P]),
    "yb_trace_read": (_I, [_P, _P, _S, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "yb_clear_status": (_I, [_P]),
    "yb_destroy": (None, [_P]),
    "yb_last_error": (_I, [ctypes.c_char_p, _I]),
    "yb_tp_export": (_I, [_P, _P, _S, ctypes.POINTER(_S)]),
    "yb_tp_import": (_I, [_P, _P, _S]),
    "yb_tp_blob_bytes": (_S, []),
    "yb_tp_shard": (_I, [_P, _I, _I, _P]),
    "yb_matmul": (_I, [_P, _P, _P, _I, _I]),
    "yb_mha": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I]),
    "yb_ffn": (_I, [_P, _P, _P, _P, _P, _I, _I, _I]),
    "yb_gemv_dev": (_I, [_P, _P, _P, _I, _I, _P, _F, _I, _P]),
    "yb_gateup_dev": (_I, [_P, _P, _P, _I, _I, _P, _F, _I, _P]),
    "yb_qkv_dev": (_I, [_P, _P, _P, _P, _P, _P, _F, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P]),
    "yb_attention_dev": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "yb_attention_scratch_bytes": (_S, [_I, _I, _I, _I]),
    "yb_attention_plan_info": (_I, [_I, _I, _I, _I, _P]),
    "yb_attention_dev_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "yb_num_sms": (_I, []),
    "yb_profile_kernel": (_I, [_P, _I, _I, ctypes.POINTER(_F)]),
}


def header_symbols() -> list[str]:
    """Names of the functions declared in include/yalm_b200.h."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(yb_[a-z0-9_]+)\s*\(", src)))


def lib():
    """Loads the library (building it first when absent and a compiler is available)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _build
        _build.build_engine()
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().yb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> int:
    if rc != 0:
        raise YalmB200Error(rc, last_error())
    return rc


def call(name: str, *args):
    return check(getattr(lib(), name)(*args))
