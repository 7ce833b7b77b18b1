"""Writes safetensors files for the snapshot tests (the container format the
reference's c/st.h reads: 8-byte little-endian header length, JSON header,
data)."""
import json
import struct

import numpy as np


def bf16_bits(x):
    """float32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def write(path, tensors, metadata=None):
    """tensors: name -> (dtype, array) with dtype in BF16 / F16 / F32 / I8."""
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = metadata
    for name, (dt, a) in tensors.items():
        if dt == "BF16":
            raw = bf16_bits(a).tobytes()
        elif dt == "F16":
            raw = np.ascontiguousarray(a, np.float16).tobytes()
        elif dt == "F32":
            raw = np.ascontiguousarray(a, np.float32).tobytes()
        else:
            raw = np.ascontiguousarray(a, np.int8).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def bf16_value(x):
    """The float32 value a BF16-stored tensor reads back as."""
    return (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)
