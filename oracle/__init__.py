"""TEST INFRASTRUCTURE ONLY — the CPU oracle for the parity tests and the benchmark's CPU baseline.

Two oracles, both CPU:
  * RefModel — yalm's own CPU decode path (`Model::forward`, `-d cpu`) compiled from the reference
    sources into oracle/_ref/libyalm_ref.so (oracle/Makefile);
  * CModel — the plain-C restatement in oracle/yalm_oracle.c (oracle/_ref/libyalm_oracle.so).
Only tests/, __graft_entry__.smoke() and bench.py's reference / cpu_baseline legs import this
package.  The product (yalm_b200/) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF_LIB = os.path.join(OUT, "libyalm_ref.so")
C_LIB = os.path.join(OUT, "libyalm_oracle.so")
REF_BIN = os.path.join(OUT, "ref_decode")
REF_BIN_GPU = os.path.join(OUT, "ref_decode_gpu")
REF_KERNELS = os.path.join(OUT, "ref_kernels")
YALM_MAIN = os.path.join(OUT, "yalm_main")
YALM_MAIN_B200 = os.path.join(OUT, "yalm_main_b200")


def _reference_root():
    """Where yalm's sources are: $YALM_REF_SRC, else the `reference_path` BASELINE.json names (the
    build container); None where neither exists (the prebuilt oracle/_ref is then used as is)."""
    p = os.environ.get("YALM_REF_SRC")
    if not p:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                p = json.load(f).get("reference_path")
        except (OSError, ValueError):
            p = None
    return p if p and os.path.isfile(os.path.join(p, "src", "model.h")) else None


REF_SRC = _reference_root()

_P, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def build(force: bool = False, gpu: bool = False, b200: bool = False) -> None:
    """Builds the C restatement always, and, when yalm's sources are present, yalm's CPU path; with
    gpu also its CUDA backends (sm_100a) and CLI, with b200 its CLI patched for the -d b200 device
    (needs libyalm_b200.so)."""
    targets = ["oracle"]
    if REF_SRC:
        targets.append("ref")
        if gpu:
            targets.append("ref-gpu")
        if b200:
            targets.append("ref-b200")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REF_SRC or ''}", f"-j{os.cpu_count() or 4}"] + targets, check=True)


def _load(path):
    if not os.path.exists(path):
        build()
    return ctypes.CDLL(path)


_ref = None
_c = None


def ref_lib():
    global _ref
    if _ref is None:
        L = _load(REF_LIB)
        L.ref_open.restype = _P
        L.ref_open.argtypes = [ctypes.c_char_p, _I]
        L.ref_config.argtypes = [_P, _P, _P]
        L.ref_forward.argtypes = [_P, _I, _I, _I, _P]
        L.ref_read_kv.argtypes = [_P, _I, _I, _I, _I, _P, _P]
        L.ref_close.argtypes = [_P]
        L.ref_matmul_f16.argtypes = [_P, _P, _P, _I, _I]
        L.ref_matmul_f32.argtypes = [_P, _P, _P, _I, _I]
        L.ref_mha.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I]
        L.ref_attn.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I]
        L.ref_ffn_f32.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        L.ref_set_threads.argtypes = [_I]
        L.ref_max_threads.restype = _I
        _ref = L
    return _ref


def c_lib():
    global _c
    if _c is None:
        L = _load(C_LIB)
        L.yo_h2f.restype = _F
        L.yo_h2f.argtypes = [ctypes.c_uint16]
        L.yo_f2h.restype = ctypes.c_uint16
        L.yo_f2h.argtypes = [_F]
        L.yo_matmul_f16.argtypes = [_P, _P, _P, _I, _I]
        L.yo_matmul_f32.argtypes = [_P, _P, _P, _I, _I]
        L.yo_rmsnorm.argtypes = [_P, _P, _P, _I, _F]
        L.yo_rope.argtypes = [_P, _I, _I, _I, _F, _I]
        L.yo_attn.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        L.yo_mha.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I]
        L.yo_positions.argtypes = [_I, _I, _P, _P, _P]
        L.yo_model_new.restype = _P
        L.yo_model_new.argtypes = [_P, _P] + [_P] * 12
        L.yo_model_free.argtypes = [_P]
        L.yo_forward.argtypes = [_P, _I, _I, _I, _P]
        L.yo_read_kv.argtypes = [_P, _I, _I, _I, _I, _P, _P]
        L.yo_read_x.argtypes = [_P, _P]
        _c = L
    return _c


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class RefModel:
    """yalm's own Model + InferenceState on the CPU (reference code, via oracle/_ref)."""

    def __init__(self, path: str, context: int = 0, threads: int = 0):
        L = ref_lib()
        if threads:
            L.ref_set_threads(threads)
        self.h = L.ref_open(path.encode(), context)
        if not self.h:
            raise RuntimeError(f"reference loader failed on {path}")
        ci = np.zeros(12, np.int32)
        cf = np.zeros(3, np.float32)
        L.ref_config(self.h, _ptr(ci), _ptr(cf))
        (self.dim, self.hidden_dim, self.head_dim, self.n_layers, self.n_heads, self.n_kv_heads, self.vocab_size,
         self.max_seq_len, self.rotary_dim, self.act_silu, self.n_experts, self.n_experts_active) = [int(v) for v in ci]
        self.rope_theta, self.norm_eps, self.qkv_clip = [float(v) for v in cf]

    def forward(self, token: int, pos: int, mode: int = 1):
        L = ref_lib()
        out = np.zeros(self.vocab_size, np.float32) if mode else None
        L.ref_forward(self.h, token, pos, mode, _ptr(out) if mode else None)
        return out

    def read_kv(self, layer, kvh, slot0, n):
        k = np.zeros((n, self.head_dim), np.uint16)
        v = np.zeros((n, self.head_dim), np.uint16)
        ref_lib().ref_read_kv(self.h, layer, kvh, slot0, n, _ptr(k), _ptr(v))
        return k, v

    def close(self):
        if self.h:
            ref_lib().ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CModel:
    """The C restatement of the same forward pass, built on a yalm_b200.codec.YALMData's tensors."""

    def __init__(self, yalm, config):
        L = c_lib()
        c = config
        self.config = c
        self.yalm = yalm
        ci = np.array([c.dim, c.hidden_dim, c.head_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size,
                       c.max_seq_len, c.rotary_dim, int(c.act)], np.int32)
        cf = np.array([c.rope_theta, c.norm_eps, c.qkv_clip], np.float32)
        t = yalm.tensors

        def addr(name):
            return t[name].address(yalm)

        def arr(key):
            return (ctypes.c_void_p * c.n_layers)(*[addr(f"model.layers.{i}.{key}.weight") for i in range(c.n_layers)])

        self._keep = [arr(k) for k in ("attn.norm", "mlp.norm", "attn.wq", "attn.wk", "attn.wv", "attn.wo", "mlp.w1",
                                       "mlp.w2", "mlp.w3")]
        wcls = addr("model.output.weight") if "model.output.weight" in t else addr("model.embed.weight")
        self.h = L.yo_model_new(_ptr(ci), _ptr(cf), addr("model.embed.weight"), addr("model.norm.weight"), wcls,
                                *[ctypes.cast(a, ctypes.c_void_p) for a in self._keep])

    def forward(self, token: int, pos: int, mode: int = 1):
        out = np.zeros(self.config.vocab_size, np.float32) if mode else None
        c_lib().yo_forward(self.h, token, pos, mode, _ptr(out) if mode else None)
        return out

    def read_kv(self, layer, kvh, slot0, n):
        hd = self.config.head_dim
        k = np.zeros((n, hd), np.uint16)
        v = np.zeros((n, hd), np.uint16)
        c_lib().yo_read_kv(self.h, layer, kvh, slot0, n, _ptr(k), _ptr(v))
        return k, v

    def close(self):
        if self.h:
            c_lib().yo_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- kernel-level oracles
def matmul_f16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """xout = W @ x for fp16 bits W (d, n) — src/infer.cpp:63-100 restated."""
    d, n = w.shape
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint16)
    out = np.zeros(d, np.float32)
    c_lib().yo_matmul_f16(_ptr(out), _ptr(x), _ptr(w), n, d)
    return out


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    out = np.zeros_like(x, dtype=np.float32)
    x = np.ascontiguousarray(x, np.float32)
    weight = np.ascontiguousarray(weight, np.float32)
    c_lib().yo_rmsnorm(_ptr(out), _ptr(x), _ptr(weight), x.size, eps)
    return out


def rope(vec: np.ndarray, head_dim: int, pos: int, theta: float, rotary_dim: int) -> np.ndarray:
    v = np.ascontiguousarray(vec, np.float32).copy()
    c_lib().yo_rope(_ptr(v), v.size, head_dim, pos, theta, rotary_dim)
    return v


def mha(q, kb, vb, head_dim, kv_len, max_seq_len, n_heads, n_kv_heads):
    """Attention over yalm's layouts (kb 16-tiled, vb [kvh][hd][msl]) — src/infer.cpp:394-415."""
    out = np.zeros(n_heads * head_dim, np.float32)
    att = np.zeros(n_heads * max_seq_len, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    kb = np.ascontiguousarray(kb, np.uint16)
    vb = np.ascontiguousarray(vb, np.uint16)
    c_lib().yo_mha(_ptr(out), _ptr(att), _ptr(kb), _ptr(vb), _ptr(q), head_dim, kv_len, max_seq_len, n_heads, n_kv_heads)
    return out


def f2h(x: np.ndarray) -> np.ndarray:
    L = c_lib()
    return np.array([L.yo_f2h(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16).reshape(np.shape(x))


def h2f(h: np.ndarray) -> np.ndarray:
    L = c_lib()
    return np.array([L.yo_h2f(int(v)) for v in np.asarray(h, np.uint16).ravel()], np.float32).reshape(np.shape(h))


def to_ref_kv_layout(k_canon: np.ndarray, v_canon: np.ndarray, max_seq_len: int):
    """[n_kv][slot][hd] canonical K, V -> yalm's 16-tiled K and [n_kv][hd][msl] V (src/model.h:14-17)."""
    n_kv, n, hd = k_canon.shape
    kb = np.zeros((n_kv, hd // 16, max_seq_len, 16), np.uint16)
    vb = np.zeros((n_kv, hd, max_seq_len), np.uint16)
    kb[:, :, :n, :] = k_canon.reshape(n_kv, n, hd // 16, 16).transpose(0, 2, 1, 3)
    vb[:, :, :n] = v_canon.transpose(0, 2, 1)
    return kb.reshape(-1), vb.reshape(-1)
