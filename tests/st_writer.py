"""Writes .safetensors files for the loader tests (8-byte little-endian header
length, JSON header, raw little-endian tensor bytes in header order)."""
from __future__ import annotations

import json
import struct

import numpy as np


def bf16_words(a) -> np.ndarray:
    """fp32 values -> bf16 bit patterns (round to nearest even), as uint16."""
    u = np.ascontiguousarray(np.asarray(a, np.float32)).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(a, np.float32))
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def header_and_data(tensors: dict, metadata: dict | None = None) -> tuple[dict, bytes]:
    """tensors: name -> (safetensors dtype name, numpy array of matching item size)."""
    hdr, blobs, off = {}, [], 0
    if metadata is not None:
        hdr["__metadata__"] = metadata
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        hdr[name] = {"dtype": dt, "shape": list(np.shape(arr)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    return hdr, b"".join(blobs)


def write_raw(path, header_bytes: bytes, data: bytes, length: int | None = None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_bytes) if length is None else length))
        f.write(header_bytes)
        f.write(data)


def write_safetensors(path, tensors: dict, metadata: dict | None = None):
    hdr, data = header_and_data(tensors, metadata)
    h = json.dumps(hdr).encode()
    h += b" " * (-len(h) % 8)  # the format pads the header to 8 bytes
    write_raw(path, h, data)
