"""Minimal GGUF v3 writer with the ggml block formats jepa.cpp files use (f32, f16, q8_0, q4_0).

The container format follows the public GGUF v3 layout that jepa.cpp's loader reads through ggml's
`gguf.h` (reference: src/jepa-gguf.cpp:788-907): magic, version, tensor count, KV count, the KV
pairs, the tensor table (name, dims in ggml order ne[0] first, ggml type id, data offset), then the
data section aligned to `general.alignment` (32 by default).

Block formats (reference: docs/quantization.md, scripts/gguf_dequant_selftest.py:1-20):
  q8_0  34-byte block per 32 values: f16 scale d, then 32 int8 q;           value = d * q
  q4_0  18-byte block per 32 values: f16 scale d, then 16 bytes of nibbles;  value = (nibble - 8) * d,
        the low nibbles hold elements 0..15 and the high nibbles elements 16..31.
The quantisers below are written from those formats (scale from the block's extreme value, round to
nearest); dequantisation parity is always judged against the bytes in the file, not the quantiser.
"""
from __future__ import annotations

import struct
from typing import Any

import numpy as np

# ggml type ids (enum ggml_type) and general.file_type values (enum ggml_ftype)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
FTYPE = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 7}
TYPE_OF_FTYPE = {"f32": GGML_F32, "f16": GGML_F16, "q4_0": GGML_Q4_0, "q8_0": GGML_Q8_0}
BLOCK = {GGML_Q4_0: (32, 18), GGML_Q8_0: (32, 34)}

# GGUF value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)


def quantize_q8_0(x: np.ndarray) -> bytes:
    """Row-major f32 values (size a multiple of 32) -> q8_0 blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / 127.0).astype(np.float32)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q4_0(x: np.ndarray) -> bytes:
    """Row-major f32 values (size a multiple of 32) -> q4_0 blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.abs(x).argmax(axis=1)
    vmax = x[np.arange(x.shape[0]), idx]
    d = (vmax / -8.0).astype(np.float32)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.floor(x * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    out = np.empty((x.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.tobytes()


def encode_tensor(x: np.ndarray, ggml_type: int) -> bytes:
    if ggml_type == GGML_F32:
        return np.ascontiguousarray(x, dtype=np.float32).tobytes()
    if ggml_type == GGML_F16:
        return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).tobytes()
    if ggml_type == GGML_Q8_0:
        return quantize_q8_0(x)
    if ggml_type == GGML_Q4_0:
        return quantize_q4_0(x)
    raise ValueError(f"unsupported ggml type {ggml_type}")


def _s(b: bytearray, s: str) -> None:
    e = s.encode("utf-8")
    b += struct.pack("<Q", len(e)) + e


def _val(b: bytearray, v: Any) -> None:
    if isinstance(v, bool):
        b += struct.pack("<I?", _BOOL, v)
    elif isinstance(v, int):
        b += struct.pack("<II", _U32, v) if 0 <= v < 2**32 else struct.pack("<Iq", _I64, v)
    elif isinstance(v, float):
        b += struct.pack("<If", _F32, v)
    elif isinstance(v, str):
        b += struct.pack("<I", _STR)
        _s(b, v)
    elif isinstance(v, (list, tuple)):
        b += struct.pack("<I", _ARR)
        if all(isinstance(e, str) for e in v):
            b += struct.pack("<IQ", _STR, len(v))
            for e in v:
                _s(b, e)
        elif all(isinstance(e, int) and not isinstance(e, bool) for e in v):
            b += struct.pack("<IQ", _U32, len(v)) + struct.pack(f"<{len(v)}I", *v)
        else:
            b += struct.pack("<IQ", _F32, len(v)) + struct.pack(f"<{len(v)}f", *[float(e) for e in v])
    else:
        raise TypeError(type(v))


class GGUFWriter:
    """Collects KV pairs and tensors, then writes one GGUF v3 file.

    Tensors are given in PyTorch row-major shape ([out, in] for a Linear); the file stores the
    ggml dims reversed (ne[0] = the last PyTorch dim), as jepa.cpp's converter does.
    """

    def __init__(self, alignment: int = 32):
        self.kv: list[tuple[str, Any]] = []
        self.tensors: list[tuple[str, tuple[int, ...], int, bytes]] = []
        self.alignment = alignment

    def add_kv(self, key: str, value: Any) -> None:
        self.kv.append((key, value))

    def add_tensor(self, name: str, x: np.ndarray, ggml_type: int = GGML_F32) -> None:
        x = np.asarray(x, dtype=np.float32)
        if ggml_type in BLOCK and x.shape[-1] % BLOCK[ggml_type][0] != 0:
            ggml_type = GGML_F32   # the quantiser keeps such a tensor at its source type
        ne = tuple(int(d) for d in reversed(x.shape))
        self.tensors.append((name, ne, ggml_type, encode_tensor(x, ggml_type)))

    def write(self, path: str) -> None:
        b = bytearray(b"GGUF")
        b += struct.pack("<IQQ", 3, len(self.tensors), len(self.kv))
        for k, v in self.kv:
            _s(b, k)
            _val(b, v)
        off = 0
        offsets = []
        for name, ne, t, data in self.tensors:
            offsets.append(off)
            off += (len(data) + self.alignment - 1) // self.alignment * self.alignment
        for (name, ne, t, data), o in zip(self.tensors, offsets):
            _s(b, name)
            b += struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne) + struct.pack("<IQ", t, o)
        pad = (-len(b)) % self.alignment
        b += b"\0" * pad
        with open(path, "wb") as f:
            f.write(b)
            for (name, ne, t, data), o in zip(self.tensors, offsets):
                f.write(data)
                f.write(b"\0" * ((-len(data)) % self.alignment))
