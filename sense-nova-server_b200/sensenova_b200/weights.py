"""The `.snl` weight file (weights.rs:1-120; writer layout convert.rs:318-428).

"SNLQ", u32 version 1, u64 header length, a JSON header {model_name, quant, config,
tensors: {name: {dtype, shape, offset, scales_offset}}}, then tensors at absolute
256-byte aligned offsets. Quantized tensors hold packed quants then f32 scales (one
per 32-element block) in two regions: exactly the layout the kernels read, so the
loader hands the mapped bytes to the library unchanged.
"""
from __future__ import annotations

import json
import mmap
import struct
from pathlib import Path

import numpy as np

from . import ffi
from .config import ModelConfig

MAGIC = b"SNLQ"
VERSION = 1
ALIGN = 256
QBLOCK = 32
DTYPES = {"f32": ffi.SNL_F32, "q8_0": ffi.SNL_Q8_0, "q4_0": ffi.SNL_Q4_0}


def dtype_sizes(dtype: str, rows: int, cols: int) -> tuple[int, int]:
    """DType::sizes (weights.rs:48-55): (quant bytes, scale bytes)."""
    n = rows * cols
    if dtype == "f32":
        return n * 4, 0
    if dtype == "q8_0":
        return n, n // QBLOCK * 4
    if dtype == "q4_0":
        return n // 2, n // QBLOCK * 4
    raise ValueError(f"unknown quantization `{dtype}` (expected q8_0 or q4_0)")


def _align(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


class WeightFile:
    def __init__(self, path: Path, header: dict, mm: mmap.mmap):
        self.path = path
        self.header = header
        self._mm = mm
        self.config = ModelConfig.from_json(header["config"])
        self.quant = header.get("quant", "q8_0")
        self.tensors: dict = header["tensors"]

    @classmethod
    def open(cls, path: str | Path) -> "WeightFile":
        p = Path(path)
        f = open(p, "rb")
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        f.close()
        if len(mm) < 16 or mm[:4] != MAGIC:
            raise ffi.SnlError(-1, f"{p} is not a SenseNova Loop weight file")
        version = struct.unpack_from("<I", mm, 4)[0]
        if version != VERSION:
            raise ffi.SnlError(-1, f"unsupported weight file version {version}; re-run `pull`")
        hlen = struct.unpack_from("<Q", mm, 8)[0]
        header = json.loads(mm[16:16 + hlen])
        wf = cls(p, header, mm)
        wf.config.validate()
        return wf

    def info(self, name: str) -> dict:
        if name not in self.tensors:
            raise ffi.SnlError(-1, f"weight file is missing tensor `{name}`")
        return self.tensors[name]

    def raw(self, name: str):
        """(dtype code, rows, cols, quants as u8, scales as f32 or None): views of the map."""
        t = self.info(name)
        shape = t["shape"]
        rows, cols = (1, shape[0]) if len(shape) == 1 else (shape[0], shape[-1])
        qb, sb = dtype_sizes(t["dtype"], rows, cols)
        q = np.frombuffer(self._mm, dtype=np.uint8, count=qb, offset=t["offset"])
        s = np.frombuffer(self._mm, dtype=np.float32, count=sb // 4, offset=t["scales_offset"]) if sb else None
        return DTYPES[t["dtype"]], rows, cols, q, s


def write_snl(path: str | Path, model_name: str, quant: str, cfg: ModelConfig, tensors: dict) -> None:
    """Write a `.snl` file in the converter's layout (convert.rs:334-428).

    tensors: name -> (dtype str, shape list, quant bytes, scale bytes or b"")."""
    infos = {}
    cursor = 0
    for name in sorted(tensors):  # BTreeMap order (weights.rs:62)
        dtype, shape, q, s = tensors[name]
        rows, cols = (1, shape[0]) if len(shape) == 1 else (shape[0], shape[1])
        qb, sb = dtype_sizes(dtype, rows, cols)
        assert len(q) == qb and len(s) == sb, name
        off = cursor
        cursor = _align(cursor + qb)
        soff = cursor
        cursor = _align(cursor + sb)
        infos[name] = {"dtype": dtype, "shape": list(shape), "offset": off, "scales_offset": soff}
    header = {"model_name": model_name, "quant": quant, "config": cfg.to_json(), "tensors": infos}
    probe = json.dumps(header).encode()
    data_start = _align(16 + len(probe) + 4096)
    for t in infos.values():
        t["offset"] += data_start
        t["scales_offset"] += data_start
    hb = json.dumps(header).encode()
    assert 16 + len(hb) <= data_start
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<IQ", VERSION, len(hb)) + hb)
        end = 0
        for name, (dtype, shape, q, s) in tensors.items():
            t = infos[name]
            f.seek(t["offset"])
            f.write(bytes(q))
            if len(s):
                f.seek(t["scales_offset"])
                f.write(bytes(s))
            end = max(end, t["offset"] + len(q), t["scales_offset"] + len(s))
        f.truncate(_align(end))
