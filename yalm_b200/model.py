"""Host-side mirror of yalm's model interface on top of the C ABI.

Names and argument meaning follow yalm (src/model.h): `Config.from_yalm`, `Model(yalm, context)`,
`InferenceState(config)` with a host `logits` buffer, and `Model.forward(state, token, pos, mode)`
with `InferenceMode.HYDRATE_KV_CACHE` / `OUTPUT_LOGITS`.  `Model.cuda(device, tp_rank, tp_size)`
plays the part of `Model::cuda()` + `InferenceState::cuda()`: it hands the mmap'd host tensors to
`yb_create`, which uploads them.  Where yalm asserts or aborts on bad input this raises
ValueError / YalmB200Error instead.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass

import numpy as np

from . import _lib
from .codec import YALMData

KV_SINKS = 2  # src/model.h:12


class InferenceMode(enum.IntEnum):  # src/model.h:43-46
    HYDRATE_KV_CACHE = 0
    OUTPUT_LOGITS = 1


class ActivationType(enum.IntEnum):  # src/model.h:19-22
    GELU = 0
    SILU = 1


FLT_MAX = float(np.finfo(np.float32).max)


@dataclass
class Config:
    dim: int = 0
    hidden_dim: int = 0
    head_dim: int = 0
    n_layers: int = 0
    n_heads: int = 0
    n_kv_heads: int = 0
    vocab_size: int = 0
    max_seq_len: int = 0
    rope_theta: float = 0.0
    rotary_dim: int = 0
    norm_eps: float = 1e-5
    act: ActivationType = ActivationType.GELU
    qkv_clip: float = FLT_MAX
    n_experts: int = 0
    n_experts_active: int = 0
    weight_dtype: str = "F16"

    @staticmethod
    def from_yalm(yalm: YALMData, context: int = 0) -> "Config":
        """Config::from_yalm, src/model.cpp:18-71 (metadata values are strings)."""
        m = yalm.metadata
        c = Config()
        c.dim = int(m["dim"])
        c.hidden_dim = int(m["hidden_dim"])
        c.head_dim = int(m["head_dim"])
        c.n_layers = int(m["n_layers"])
        c.n_heads = int(m["n_heads"])
        c.n_kv_heads = int(m["n_kv_heads"])
        c.vocab_size = int(m["vocab_size"])
        c.n_experts = int(m["n_experts"]) if "n_experts" in m else 0
        c.n_experts_active = int(m["n_experts_active"]) if "n_experts_active" in m else 0
        c.max_seq_len = min(int(m["max_seq_len"]), 4096)  # yalm's default cap (model.cpp:30-31)
        if context:
            c.max_seq_len = context
        c.rope_theta = float(m["rope_theta"])
        c.rotary_dim = int(m["rotary_dim"])
        c.norm_eps = float(m.get("norm_eps", "1e-5"))
        c.act = ActivationType.SILU if m.get("act_type", "gelu") == "silu" else ActivationType.GELU
        c.qkv_clip = float(m["qkv_clip"]) if "qkv_clip" in m else FLT_MAX
        dt = m["dtype"]
        if dt == "fp16":
            c.weight_dtype = "F16"
        elif dt == "fp32":
            c.weight_dtype = "F32"
        elif dt == "fp8":
            # convert.py's fp8 is a plain cast to float8_e5m2 (convert.py:160); yalm's runtime stops
            # here (src/model.cpp:61-70), this engine runs it
            c.weight_dtype = "F8_E5M2"
        else:
            raise ValueError(f"unsupported dtype: {dt}")
        return c

    @property
    def weight_bytes(self) -> int:
        return {"F16": 2, "F32": 4, "F8_E5M2": 1}[self.weight_dtype]

    def to_c(self) -> _lib.yb_config:
        return _lib.yb_config(dim=self.dim, hidden_dim=self.hidden_dim, head_dim=self.head_dim,
                              n_layers=self.n_layers, n_heads=self.n_heads, n_kv_heads=self.n_kv_heads,
                              vocab_size=self.vocab_size, max_seq_len=self.max_seq_len, rotary_dim=self.rotary_dim,
                              act=int(self.act), n_experts=self.n_experts,
                              weight_dtype={"F16": 1, "F8_E5M2": 3}.get(self.weight_dtype, 0),
                              rope_theta=self.rope_theta, norm_eps=self.norm_eps, qkv_clip=self.qkv_clip)

    def weight_bytes_per_token(self, tp_size: int = 1) -> int:
        """Algorithmic bytes streamed per decode step on one rank: every matrix once, norms, one
        embedding row and the classifier (not the whole embedding table)."""
        q_dim, kv_dim = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        wb = self.weight_bytes
        per_layer = wb * (q_dim * self.dim + 2 * kv_dim * self.dim + self.dim * q_dim
                          + 3 * self.dim * self.hidden_dim) // tp_size + 2 * self.dim * 4
        return self.n_layers * per_layer + wb * self.vocab_size * self.dim // tp_size + self.dim * 4 + self.dim * wb

    def kv_bytes_per_token(self, kv_len: int, tp_size: int = 1) -> int:
        """KV-cache bytes attention reads per step (K and V, fp16, all layers)."""
        return self.n_layers * 2 * (self.n_kv_heads // tp_size) * self.head_dim * 2 * kv_len


def _check_tensor(yalm: YALMData, name: str, dtype: str, shape):
    """check_tensor / get_tensor, src/model.cpp:100-128 (raises instead of asserting)."""
    t = yalm.tensors.get(name)
    if t is None:
        raise ValueError(f"missing tensor: {name}")
    want = tuple(list(shape) + [0] * (4 - len(shape)))
    if t.dtype != dtype or t.shape != want:
        raise ValueError(f"tensor mismatch for {name}: expected {dtype} {want}, got {t.dtype} {t.shape}")
    return t


class InferenceState:
    """The part of yalm's InferenceState the caller sees: the host logits buffer (model.h:122)."""

    def __init__(self, config: Config):
        self.config = config
        self._logits = np.zeros(config.vocab_size, dtype=np.float32)

    def logits(self) -> np.ndarray:
        return self._logits


class Model:
    """Model(yalm, context) (src/model.cpp:392-435): validates every tensor and keeps host views."""

    def __init__(self, yalm: YALMData, context: int = 0):
        self.yalm = yalm
        self.config = c = Config.from_yalm(yalm, context)
        if c.n_experts > 0:
            raise _lib.YalmB200Error(_lib.YB_E_UNSUPPORTED, "mixture-of-experts checkpoints are not supported")
        dt = c.weight_dtype
        q_dim, kv_dim = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        self.token_embedding_table = _check_tensor(yalm, "model.embed.weight", dt, (c.vocab_size, c.dim))
        self.layers = []
        for i in range(c.n_layers):
            p = f"model.layers.{i}."
            self.layers.append({
                "rms_att": _check_tensor(yalm, p + "attn.norm.weight", "F32", (c.dim,)),
                "rms_ffn": _check_tensor(yalm, p + "mlp.norm.weight", "F32", (c.dim,)),
                "wq": _check_tensor(yalm, p + "attn.wq.weight", dt, (q_dim, c.dim)),
                "wk": _check_tensor(yalm, p + "attn.wk.weight", dt, (kv_dim, c.dim)),
                "wv": _check_tensor(yalm, p + "attn.wv.weight", dt, (kv_dim, c.dim)),
                "wo": _check_tensor(yalm, p + "attn.wo.weight", dt, (c.dim, q_dim)),
                "w1": _check_tensor(yalm, p + "mlp.w1.weight", dt, (c.hidden_dim, c.dim)),
                "w2": _check_tensor(yalm, p + "mlp.w2.weight", dt, (c.dim, c.hidden_dim)),
                "w3": _check_tensor(yalm, p + "mlp.w3.weight", dt, (c.hidden_dim, c.dim)),
            })
        self.rms_final_weight = _check_tensor(yalm, "model.norm.weight", "F32", (c.dim,))
        if "model.output.weight" in yalm.tensors:
            self.wcls = _check_tensor(yalm, "model.output.weight", dt, (c.vocab_size, c.dim))
        else:
            self.wcls = self.token_embedding_table  # tied embeddings (model.cpp:425-428)
        self._engine = None
        self.tp_rank, self.tp_size = 0, 1

    # ------------------------------------------------------------------ device
    def weights_struct(self):
        y = self.yalm
        L = self.config.n_layers

        def arr(key):
            a = (ctypes.c_void_p * L)(*[self.layers[i][key].address(y) for i in range(L)])
            return ctypes.cast(a, ctypes.POINTER(ctypes.c_void_p)), a

        keep = []
        fields = {}
        for key, fname in (("rms_att", "rms_att_weight"), ("rms_ffn", "rms_ffn_weight"), ("wq", "wq"), ("wk", "wk"),
                           ("wv", "wv"), ("wo", "wo"), ("w1", "w1"), ("w2", "w2"), ("w3", "w3")):
            p, a = arr(key)
            keep.append(a)
            fields[fname] = p
        w = _lib.yb_weights(token_embedding_table=self.token_embedding_table.address(y),
                            rms_final_weight=self.rms_final_weight.address(y),
                            wcls=self.wcls.address(y), **fields)
        return w, keep

    def cuda(self, device: int = 0, tp_rank: int = 0, tp_size: int = 1) -> "Model":
        cfg = self.config.to_c()
        w, keep = self.weights_struct()
        h = ctypes.c_void_p()
        _lib.call("yb_create", ctypes.byref(cfg), ctypes.byref(w), device, tp_rank, tp_size, ctypes.byref(h))
        del keep
        self._engine = h
        self.device, self.tp_rank, self.tp_size = device, tp_rank, tp_size
        return self

    @property
    def engine(self):
        if self._engine is None:
            raise _lib.YalmB200Error(_lib.YB_E_INVALID, "model is not on a device; call cuda() first")
        return self._engine

    def tp_join(self, all_gather_bytes) -> None:
        """Joins the tensor-parallel ranks.  all_gather_bytes(bytes) -> list[bytes] in rank order
        (for example built on torch.distributed.all_gather_object)."""
        L = _lib.lib()
        n = L.yb_tp_blob_bytes()
        blob = ctypes.create_string_buffer(n)
        used = ctypes.c_size_t()
        _lib.call("yb_tp_export", self.engine, blob, n, ctypes.byref(used))
        blobs = all_gather_bytes(bytes(blob.raw[:n]))
        if len(blobs) != self.tp_size:
            raise ValueError("expected one blob per rank")
        joined = ctypes.create_string_buffer(b"".join(blobs), n * len(blobs))
        _lib.call("yb_tp_import", self.engine, joined, n)

    def forward(self, s: InferenceState, token: int, pos: int,
                mode: InferenceMode = InferenceMode.OUTPUT_LOGITS) -> None:
        """Model::forward (src/model.cpp:479-494) on the B200 engine."""
        lg = s.logits()
        _lib.call("yb_forward", self.engine, int(token), int(pos), int(mode),
                  lg.ctypes.data if mode == InferenceMode.OUTPUT_LOGITS else None)

    def forward_async(self, token: int, pos: int, mode: InferenceMode = InferenceMode.OUTPUT_LOGITS) -> None:
        _lib.call("yb_forward_async", self.engine, int(token), int(pos), int(mode))

    def prefill(self, tokens, pos0: int = 0, s: InferenceState | None = None) -> None:
        """The prompt loop of yalm's run_completion (src/main.cpp:171-177) in one batched pass:
        tokens at positions pos0.., KV cache filled; with `s` the last token's logits land in
        s.logits()."""
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        lg = s.logits() if s is not None else None
        _lib.call("yb_prefill", self.engine, ids.ctypes.data, int(ids.size), int(pos0),
                  lg.ctypes.data if lg is not None else None)

    def forward_sample(self, token: int, pos: int, temperature: float = 0.0, coin: float = 0.0) -> int:
        """Model::forward + Sampler::sample (src/sampler.cpp:27-64) with the sampler on the device:
        returns the next token id; temperature 0 is greedy, else `coin` plays yalm's
        rand() / RAND_MAX draw."""
        out = ctypes.c_int()
        _lib.call("yb_forward_sample", self.engine, int(token), int(pos), float(temperature), float(coin),
                  ctypes.byref(out))
        return out.value

    def forward_prob(self, token: int, pos: int, target: int) -> float:
        """Model::forward + Sampler::sample_prob(target) (src/sampler.cpp:11-25) on the device."""
        out = ctypes.c_float()
        _lib.call("yb_forward_prob", self.engine, int(token), int(pos), int(target), ctypes.byref(out))
        return out.value

    def sync(self) -> None:
        _lib.call("yb_sync", self.engine)

    def logits_dev_ptr(self) -> int:
        return _lib.lib().yb_logits_dev(self.engine)

    def stream_ptr(self) -> int:
        return _lib.lib().yb_stream(self.engine) or 0

    def read_kv(self, layer: int, kv_head: int, slot0: int, n: int):
        hd = self.config.head_dim
        k = np.zeros((n, hd), dtype=np.uint16)
        v = np.zeros((n, hd), dtype=np.uint16)
        _lib.call("yb_read_kv", self.engine, layer, kv_head, slot0, n, k.ctypes.data, v.ctypes.data)
        return k, v

    def executor(self) -> str:
        return "persistent" if _lib.lib().yb_executor(self.engine) == 1 else "graph"

    def status(self) -> int:
        return int(_lib.lib().yb_status(self.engine))

    def close(self) -> None:
        if self._engine is not None:
            _lib.lib().yb_destroy(self._engine)
            self._engine = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def positions(pos: int, max_seq_len: int):
    """(kv_sink, kv_pos, kv_len) for a step, src/infer.cpp:489-494."""
    kv_sink = KV_SINKS if pos >= max_seq_len else 0
    kv_pos = kv_sink + (pos - kv_sink) % (max_seq_len - kv_sink)
    kv_len = max_seq_len if pos >= max_seq_len else pos + 1
    return kv_sink, kv_pos, kv_len
