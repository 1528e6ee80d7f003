"""Minimal safetensors reader for checkpoint loading (the reference reads the same
format over HTTP range requests: parseSafetensorsHeader / loadTensorFromSafetensors,
src/weights.ts:60-215).

File layout: an 8-byte little-endian header length, a JSON header mapping each tensor
name to {"dtype", "shape", "data_offsets": [begin, end]} (offsets relative to the end
of the header; an optional "__metadata__" entry), then the raw little-endian data.
The file is memory-mapped; tensors are returned as zero-copy numpy views.
"""
from __future__ import annotations

import json
import mmap
import struct
from typing import Dict, Iterator, Tuple

import numpy as np

# dtype name -> (numpy dtype of the raw words, code of vx_load_tensor_typed or None)
DTYPES = {
    "F16": (np.uint16, 0),
    "BF16": (np.uint16, 1),
    "F32": (np.uint32, 2),
    "F64": (np.float64, None),
    "I8": (np.int8, None),
    "I16": (np.int16, None),
    "I32": (np.int32, None),
    "I64": (np.int64, None),
    "U8": (np.uint8, None),
    "U16": (np.uint16, None),
    "U32": (np.uint32, None),
    "BOOL": (np.bool_, None),
}


class SafetensorsFile:
    """Memory-mapped safetensors file: `entries` holds the parsed header."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        if len(self._mm) < 8:
            raise ValueError(f"{path}: not a safetensors file")
        (hlen,) = struct.unpack("<Q", self._mm[:8])
        if 8 + hlen > len(self._mm):
            raise ValueError(f"{path}: header length {hlen} beyond the file")
        header = json.loads(bytes(self._mm[8 : 8 + hlen]).decode("utf-8"))
        self.metadata = header.pop("__metadata__", {})
        self.entries: Dict[str, dict] = header
        self.data_offset = 8 + hlen
        for name, e in self.entries.items():
            if e.get("dtype") not in DTYPES:
                raise ValueError(f"{name}: unsupported dtype {e.get('dtype')}")
            b, end = e["data_offsets"]
            n = int(np.prod(e["shape"])) if e["shape"] else 1
            if end - b != n * np.dtype(DTYPES[e["dtype"]][0]).itemsize or self.data_offset + end > len(self._mm):
                raise ValueError(f"{name}: data offsets {e['data_offsets']} do not match shape {e['shape']}")

    def raw(self, name: str) -> Tuple[np.ndarray, str]:
        """(flat view of the tensor's raw words, dtype name)."""
        e = self.entries[name]
        dt = DTYPES[e["dtype"]][0]
        b, end = e["data_offsets"]
        n = (end - b) // np.dtype(dt).itemsize
        return np.frombuffer(self._mm, dtype=dt, count=n, offset=self.data_offset + b), e["dtype"]

    def names(self) -> Iterator[str]:
        return iter(self.entries.keys())

    def close(self):
        try:
            self._mm.close()
        except BufferError:   # a view is still alive; the map closes with it
            pass
        self._f.close()


def write(path: str, tensors: Dict[str, Tuple[np.ndarray, str]], metadata: dict = None):
    """Write {name: (raw words, dtype name)} as a safetensors file (tests and tools)."""
    header, blobs, off = {}, [], 0
    for name, (arr, dt) in tensors.items():
        a = np.ascontiguousarray(arr)
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
