"""Minimal safetensors reader/writer over numpy.

The file layout is the public safetensors format: an 8-byte little-endian header
length, a JSON header mapping tensor names to {dtype, shape, data_offsets}, then
the raw little-endian bytes. The reference reads the same files through its own
mmap loader (src/core/weights.cpp:26-31, 100-122) and converts BF16/F16/F32 to
fp32; here bf16 tensors travel as uint16 bit patterns.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

_NP = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I32": np.int32, "I64": np.int64}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def save(path: str | Path, tensors: dict[str, tuple[str, np.ndarray]], metadata: dict | None = None) -> None:
    """tensors: name -> (dtype tag "F32" | "BF16" | ..., array). BF16 arrays are uint16 bits."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    off = 0
    blobs = []
    for name, (dt, arr) in tensors.items():
        arr = np.ascontiguousarray(arr, dtype=_NP[dt])
        nb = arr.nbytes
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + nb]}
        blobs.append(arr)
        off += nb
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b.tobytes())


def load(path: str | Path) -> dict[str, tuple[str, np.ndarray]]:
    """name -> (dtype tag, array view of the file bytes)."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    (hlen,) = struct.unpack("<Q", bytes(raw[:8]))
    header = json.loads(bytes(raw[8 : 8 + hlen]))
    base = 8 + hlen
    out = {}
    for name, t in header.items():
        if name == "__metadata__":
            continue
        dt = t["dtype"]
        if dt not in _NP:
            raise ValueError(f"unsupported dtype {dt} for {name}")
        b, e = t["data_offsets"]
        arr = np.frombuffer(raw[base + b : base + e], dtype=_NP[dt]).reshape(t["shape"])
        out[name] = (dt, arr)
    return out


def to_f32(entry: tuple[str, np.ndarray]) -> np.ndarray:
    dt, arr = entry
    if dt == "BF16":
        return bf16_bits_to_f32(arr).reshape(arr.shape)
    return np.asarray(arr, dtype=np.float32)


def save_streaming(path: str | Path, entries: list[tuple[str, str, tuple[int, ...]]], produce,
                   metadata: dict | None = None) -> None:
    """Writes tensors one at a time: `entries` lists (name, dtype tag, shape) in file order and
    `produce(name)` returns each array (uint16 bits for BF16) when its turn comes."""
    itemsize = {"F32": 4, "BF16": 2, "F16": 2, "I32": 4, "I64": 8}
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    off = 0
    for name, dt, shape in entries:
        nb = int(np.prod(shape)) * itemsize[dt]
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + nb]}
        off += nb
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for name, dt, shape in entries:
            arr = np.ascontiguousarray(produce(name), dtype=_NP[dt])
            if arr.shape != tuple(shape):
                raise ValueError(f"{name}: produced shape {arr.shape}, declared {shape}")
            f.write(arr.tobytes())
