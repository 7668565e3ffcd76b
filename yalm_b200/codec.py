""".yalm checkpoint reader (host side).

Mirrors yalm's YALMData / Tensor (src/codec.h:30-50, src/codec.cpp:39-156): the file is mmap'd,
the 8-byte header length and JSON header are parsed, `__metadata__` becomes `metadata`, and every
other entry becomes a Tensor whose data points into the mapping.  Validation follows
Tensor::from_json: known dtype, at most 4 dimensions, offsets inside the data section, and
numel * dtype size == byte size.  Failures raise ValueError (the C++ reader returns -1).
"""
from __future__ import annotations

import json
import mmap
import os
from dataclasses import dataclass

import numpy as np

# DType, src/codec.h:15-25 (same order), with element sizes (src/codec.cpp:24-37)
DTYPES = {"F32": (0, 4, np.float32), "F16": (1, 2, np.uint16), "BF16": (2, 2, np.uint16),
          "F8_E5M2": (3, 1, np.uint8), "F8_E4M3": (4, 1, np.uint8), "I32": (5, 4, np.int32),
          "I16": (6, 2, np.int16), "I8": (7, 1, np.int8), "U8": (8, 1, np.uint8)}


@dataclass
class Tensor:
    name: str
    dtype: str
    shape: tuple
    offset: int  # absolute byte offset of the data in the file
    size: int    # bytes

    def array(self, data: "YALMData") -> np.ndarray:
        _, _, npdt = DTYPES[self.dtype]
        shp = tuple(s for s in self.shape if s) or (0,)
        return np.frombuffer(data.buf, dtype=npdt, count=self.size // DTYPES[self.dtype][1],
                             offset=self.offset).reshape(shp)

    def address(self, data: "YALMData") -> int:
        return data.base_address + self.offset


class YALMData:
    def __init__(self, path: str):
        self.path = path
        fd = os.open(path, os.O_RDONLY)
        try:
            size = os.fstat(fd).st_size
            if size < 8:
                raise ValueError("file too small")
            self.mm = mmap.mmap(fd, size, mmap.MAP_PRIVATE, mmap.PROT_READ | mmap.PROT_WRITE)
        finally:
            os.close(fd)
        self.size = size
        self.buf = memoryview(self.mm)
        json_size = int.from_bytes(self.mm[:8], "little")
        if json_size == 0 or json_size > size - 8:
            raise ValueError("bad header length")
        header = json.loads(bytes(self.mm[8:8 + json_size]))
        data_start = 8 + json_size
        bytes_size = size - data_start
        self.metadata = {}
        self.tensors: dict[str, Tensor] = {}
        for key, val in header.items():
            if key == "__metadata__":
                self.metadata = val
                continue
            dt = val.get("dtype", "")
            if dt not in DTYPES:
                raise ValueError(f"bad dtype for {key}")
            shape = val["shape"]
            if len(shape) > 4:
                raise ValueError(f"shape exceeds 4 dimensions for {key}")
            numel = 1
            for s in shape:
                if int(s) != s:
                    raise ValueError(f"bad shape for {key}")
                numel *= int(s)
            offs = val["data_offsets"]
            if len(offs) != 2:
                raise ValueError(f"bad offsets for {key}")
            o0, o1 = int(offs[0]), int(offs[1])
            if o0 < 0 or o1 <= o0 or o1 > bytes_size:
                raise ValueError(f"bad offsets for {key}")
            if numel * DTYPES[dt][1] != o1 - o0:
                raise ValueError(f"bad size for {key}")
            shp4 = tuple(list(int(s) for s in shape) + [0] * (4 - len(shape)))
            self.tensors[key] = Tensor(key, dt, shp4, data_start + o0, o1 - o0)
        # a stable address for handing tensor pointers to native code
        self._anchor = np.frombuffer(self.buf, dtype=np.uint8)
        self.base_address = self._anchor.ctypes.data

    def close(self):
        self._anchor = None
        self.buf.release()
        self.mm.close()
