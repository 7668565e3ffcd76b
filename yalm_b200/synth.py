"""Seeded synthetic .yalm checkpoints.

A .yalm file is a safetensors container: an 8-byte little-endian header length, a JSON header whose
``__metadata__`` holds string-valued model config keys, and tensor data (yalm convert.py:22-81 for
the keys, convert.py:164-204 and :245 for tensor names and dtypes, src/codec.cpp:97-156 for the
reader).  This module writes files with that exact layout for the architectures in the benchmark
configs: fp16 matrices ~ N(0, std), fp32 norm weights (1.0), an untied classifier and a synthetic
tokenizer vocabulary.  Weight contents depend only on (seed, tensor name), so the same call always
produces the same bytes.
"""
from __future__ import annotations

import json
import os
import zlib
from dataclasses import dataclass, asdict

import numpy as np

@dataclass(frozen=True)
class ModelShape:
    dim: int
    hidden_dim: int
    head_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    max_seq_len: int
    rope_theta: float = 1000000.0
    norm_eps: float = 1e-05
    act_type: str = "silu"
    arch: str = "MistralForCausalLM"
    dtype: str = "fp16"  # metadata dtype: "fp16", or "fp8" (matrices as F8_E5M2, convert.py:160)

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim


# The architectures of the benchmark configs.  `max_seq_len` is the metadata value; yalm caps it at
# 4096 unless a context is given (src/model.cpp:30-34), so the 70B config is opened with context 8192.
SHAPES = {
    "tiny": ModelShape(dim=512, hidden_dim=1408, head_dim=64, n_layers=4, n_heads=8, n_kv_heads=2,
                       vocab_size=4096, max_seq_len=1024),
    "mistral-7b": ModelShape(dim=4096, hidden_dim=14336, head_dim=128, n_layers=32, n_heads=32, n_kv_heads=8,
                             vocab_size=32000, max_seq_len=32768),
    "llama-70b": ModelShape(dim=8192, hidden_dim=28672, head_dim=128, n_layers=80, n_heads=64, n_kv_heads=8,
                            vocab_size=32000, max_seq_len=8192, arch="LlamaForCausalLM"),
}


def shape_with(base: str, **overrides) -> ModelShape:
    d = asdict(SHAPES[base])
    d.update(overrides)
    return ModelShape(**d)


def metadata(shape: ModelShape) -> dict:
    """String-valued metadata exactly as convert.py's Metadata.to_dict (convert.py:58-81)."""
    return {
        "arch": shape.arch,
        "dtype": shape.dtype,
        "dim": str(shape.dim),
        "hidden_dim": str(shape.hidden_dim),
        "head_dim": str(shape.head_dim),
        "n_layers": str(shape.n_layers),
        "n_heads": str(shape.n_heads),
        "n_kv_heads": str(shape.n_kv_heads),
        "vocab_size": str(shape.vocab_size),
        "max_seq_len": str(shape.max_seq_len),
        "bos_token_id": "1",
        "eos_token_id": "2",
        "rope_theta": str(float(shape.rope_theta)),
        "rotary_dim": str(shape.head_dim),
        "norm_eps": str(shape.norm_eps),
        "norm_type": "rmsnorm",
        "act_type": shape.act_type,
    }


def tensor_specs(shape: ModelShape):
    """(name, dtype, shape) in file order, names as convert.py writes them (convert.py:164-204)."""
    s = shape
    W = "F8_E5M2" if s.dtype == "fp8" else "F16"
    out = [("model.embed.weight", W, (s.vocab_size, s.dim))]
    for l in range(s.n_layers):
        p = f"model.layers.{l}."
        out += [
            (p + "attn.norm.weight", "F32", (s.dim,)),
            (p + "attn.wq.weight", W, (s.q_dim, s.dim)),
            (p + "attn.wk.weight", W, (s.kv_dim, s.dim)),
            (p + "attn.wv.weight", W, (s.kv_dim, s.dim)),
            (p + "attn.wo.weight", W, (s.dim, s.q_dim)),
            (p + "mlp.norm.weight", "F32", (s.dim,)),
            (p + "mlp.w1.weight", W, (s.hidden_dim, s.dim)),
            (p + "mlp.w2.weight", W, (s.dim, s.hidden_dim)),
            (p + "mlp.w3.weight", W, (s.hidden_dim, s.dim)),
        ]
    out += [("model.norm.weight", "F32", (s.dim,)), ("model.output.weight", W, (s.vocab_size, s.dim))]
    return out


def vocab_bytes(vocab_size: int) -> bytes:
    """NUL-joined token strings (convert.py:245): specials, 256 byte-fallback pieces, then '~<id>'."""
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    toks += [f"~{i}" for i in range(len(toks), vocab_size)]
    toks = toks[:vocab_size]
    return b"".join(t.encode() + b"\0" for t in toks)


_DTYPE_SIZE = {"F16": 2, "F32": 4, "U8": 1, "F8_E5M2": 1}

# ---------------------------------------------------------------- seeded normal deviates
# Element i of a tensor drawn with (seed, stream) is a deterministic function of those three numbers
# only, so the contents do not depend on the thread count or on the order in which tensors are
# written.  Each element pair takes one splitmix64 output; its two 32-bit halves are the uniforms of
# a Box-Muller transform (float64), each deviate is rounded to float32, scaled by std in float32 and
# rounded to fp16 (round to nearest even).  Pure numpy: the ufuncs release the GIL, so a thread per
# core fills a 7B checkpoint at host memory speed.
_U64 = np.uint64


def _splitmix64(z):
    z = z + _U64(0x9E3779B97F4A7C15)
    z ^= z >> _U64(30)
    z *= _U64(0xBF58476D1CE4E5B9)
    z ^= z >> _U64(27)
    z *= _U64(0x94D049BB133111EB)
    z ^= z >> _U64(31)
    return z


def _stream_key(seed: int, stream: int):
    with np.errstate(over="ignore"):
        return _splitmix64(_U64(seed) * _U64(0x2545F4914F6CDD1D) ^ _splitmix64(_U64(stream) + _U64(0x632BE59BD9B4E019)))


def _normal_f16_pairs(key, p0: int, p1: int, std: float) -> np.ndarray:
    """fp16 bit patterns of elements 2*p0 .. 2*p1 - 1."""
    with np.errstate(over="ignore"):
        r = np.arange(p0, p1, dtype=np.uint64)
        r += key
        r = _splitmix64(r)
    u1 = (r >> _U64(32)).astype(np.float64)  # (0, 1]
    u1 += 1.0
    u1 *= 1.0 / 4294967296.0
    ang = (r & _U64(0xFFFFFFFF)).astype(np.float64)  # 2 pi [0, 1)
    ang *= 6.283185307179586 * (1.0 / 4294967296.0)
    del r
    np.log(u1, out=u1)
    u1 *= -2.0
    np.sqrt(u1, out=u1)
    z = np.empty((p1 - p0, 2), np.float32)
    np.multiply(u1, np.cos(ang), out=z[:, 0], casting="unsafe")
    np.multiply(u1, np.sin(ang), out=z[:, 1], casting="unsafe")
    z *= np.float32(std)
    return z.reshape(-1).astype(np.float16).view(np.uint16)


_CHUNK_PAIRS = 1 << 20


def _threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def fill_normal(out: np.ndarray, seed: int, stream: int, std: float, e5m2: bool = False) -> None:
    """Fills `out` (uint16 fp16 bits, or uint8 E5M2 bytes when e5m2) with std * N(0, 1) deviates of
    (seed, stream).  An E5M2 value is the fp16 value of the same element rounded to nearest even on
    its top byte (e5m2_from_f16_bits)."""
    from concurrent.futures import ThreadPoolExecutor
    n = out.size
    pairs = (n + 1) // 2
    key = _stream_key(seed, stream)

    def work(p0):
        p1 = min(p0 + _CHUNK_PAIRS, pairs)
        e = min(2 * p1, n)
        h = _normal_f16_pairs(key, p0, p1, std)[: e - 2 * p0]
        out[2 * p0:e] = e5m2_from_f16_bits(h) if e5m2 else h

    starts = range(0, pairs, _CHUNK_PAIRS)
    if len(starts) <= 1:
        for p0 in starts:
            work(p0)
        return
    with ThreadPoolExecutor(min(_threads(), len(starts))) as ex:
        list(ex.map(work, starts))


def write_yalm(path: str, shape: ModelShape, seed: int = 0, std: float = 0.02) -> str:
    """Writes a synthetic .yalm checkpoint to `path` and returns it.  Rewrites only when the header
    of an existing file differs (the data is a pure function of the header and seed)."""
    specs = tensor_specs(shape)
    tok = vocab_bytes(shape.vocab_size)
    header = {"__metadata__": dict(metadata(shape), synth_seed=str(seed), synth_std=str(std))}
    off = 0
    for name, dt, shp in specs:
        n = int(np.prod(shp)) * _DTYPE_SIZE[dt]
        header[name] = {"dtype": dt, "shape": list(shp), "data_offsets": [off, off + n]}
        off += n
    header["tokenizer.tokens"] = {"dtype": "U8", "shape": [len(tok)], "data_offsets": [off, off + len(tok)]}
    off += len(tok)
    hjson = json.dumps(header, separators=(",", ":")).encode()
    # pad so tensor data starts on a 256-byte boundary (spaces are valid JSON whitespace)
    pad = (-(8 + len(hjson))) % 256
    hjson += b" " * pad
    data_start = 8 + len(hjson)
    total = data_start + off
    if os.path.exists(path) and os.path.getsize(path) == total:
        with open(path, "rb") as f:
            n = int.from_bytes(f.read(8), "little")
            if f.read(n) == hjson:
                return path
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(len(hjson).to_bytes(8, "little"))
        f.write(hjson)
        f.truncate(total)
    mm = np.memmap(tmp, dtype=np.uint8, mode="r+")
    for name, dt, shp in specs:
        o0, o1 = header[name]["data_offsets"]
        view = mm[data_start + o0: data_start + o1]
        if dt == "F32":
            view.view(np.float32)[:] = 1.0
        elif dt == "F8_E5M2":
            fill_normal(view, seed, zlib.crc32(name.encode()), std, e5m2=True)
        else:
            fill_normal(view.view(np.uint16), seed, zlib.crc32(name.encode()), std)
    o0, _ = header["tokenizer.tokens"]["data_offsets"]
    mm[data_start + o0: data_start + o0 + len(tok)] = np.frombuffer(tok, dtype=np.uint8)
    mm.flush()
    del mm
    os.replace(tmp, path)
    return path


def scratch_dir(nbytes: int) -> str:
    """A directory with room for nbytes: /dev/shm when it has space, else the system temp dir."""
    import shutil
    import tempfile
    for d in ("/dev/shm", tempfile.gettempdir()):
        try:
            if shutil.disk_usage(d).free > nbytes * 1.1 + (1 << 30):
                return d
        except OSError:
            pass
    return tempfile.gettempdir()


def file_bytes(shape: ModelShape) -> int:
    return sum(int(np.prod(s)) * _DTYPE_SIZE[d] for _, d, s in tensor_specs(shape)) + len(vocab_bytes(shape.vocab_size))


def e5m2_from_f16_bits(h: np.ndarray) -> np.ndarray:
    """fp16 bit patterns -> E5M2 bytes, rounding the low byte to nearest even (an E5M2 value is the
    top byte of the fp16 with the same value; torch's float8_e5m2 cast of an fp16-exact value gives
    the same bytes)."""
    h = h.astype(np.uint32)
    lo, up = h & 0xFF, h >> 8
    inc = (lo > 0x80) | ((lo == 0x80) & ((up & 1) == 1))
    nan = (h & 0x7FFF) > 0x7C00
    out = np.where(nan, up | 0x02, up + inc.astype(np.uint32))
    return out.astype(np.uint8)


def expand_fp8_to_fp16(src: str, dst: str) -> str:
    """Writes the fp16 twin of an fp8 (E5M2) .yalm file: same metadata but dtype "fp16", every
    F8_E5M2 tensor as F16 with the identical values (byte << 8).  yalm's own fp16 CPU path on the
    twin computes exactly what an fp8 runtime computes on the original, so it is the oracle for it."""
    with open(src, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
    data = np.memmap(src, dtype=np.uint8, mode="r", offset=8 + n)
    meta = dict(header["__metadata__"], dtype="fp16")
    names = [k for k in header if k != "__metadata__"]
    names.sort(key=lambda k: header[k]["data_offsets"][0])
    out_header = {"__metadata__": meta}
    chunks = []
    off = 0
    for k in names:
        e = header[k]
        a0, a1 = e["data_offsets"]
        raw = np.asarray(data[a0:a1])
        if e["dtype"] == "F8_E5M2":
            raw = (raw.astype(np.uint16) << 8).view(np.uint8)
            dt = "F16"
        else:
            dt = e["dtype"]
        out_header[k] = {"dtype": dt, "shape": e["shape"], "data_offsets": [off, off + raw.size]}
        chunks.append(raw)
        off += raw.size
    hjson = json.dumps(out_header, separators=(",", ":")).encode()
    hjson += b" " * ((-(8 + len(hjson))) % 256)
    tmp = dst + ".tmp"
    with open(tmp, "wb") as f:
        f.write(len(hjson).to_bytes(8, "little"))
        f.write(hjson)
        for c in chunks:
            f.write(c.tobytes())
    os.replace(tmp, dst)
    return dst
