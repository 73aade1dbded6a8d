"""`.tirs` tensor bundles in numpy, byte-compatible with tabicl-anywhere (src/store.rs:1-11, 282-483).

    bytes 0..8    magic "TIRSBNDL"
    bytes 8..16   u64 little-endian: length of the index in bytes
    index         utf-8 text, one line per tensor:  name dtype offset nbytes dim0 dim1 ...
    data          each tensor starts on a 64-byte boundary (offset counts from the start of the file)
"""
import os
import struct

import numpy as np

MAGIC = b"TIRSBNDL"
DTYPES = {"float32": np.float32, "float16": np.float16, "int32": np.int32, "uint8": np.uint8, "int8": np.int8,
          "float64": np.float64, "int64": np.int64}


class Bundle:
    """A bundle read whole into memory: `b[name]` is the tensor as a numpy array of its stored dtype and shape."""

    def __init__(self, data):
        if isinstance(data, (str, os.PathLike)):
            with open(data, "rb") as f:
                data = f.read()
        self.data = bytes(data)
        if self.data[:8] != MAGIC:
            raise ValueError("not a tabicl-anywhere bundle")
        (n,) = struct.unpack("<Q", self.data[8:16])
        self.entries = {}
        for line in self.data[16:16 + n].decode().splitlines():
            p = line.split(" ")
            name, dtype, off, nb = p[0], p[1], int(p[2]), int(p[3])
            dims = tuple(int(x) for x in p[4:] if x != "")
            if dtype not in DTYPES:
                raise ValueError(f"{line}: unknown tensor type")
            if int(np.prod(dims, dtype=np.int64)) * np.dtype(DTYPES[dtype]).itemsize != nb:
                raise ValueError(f"{line}: shape and length disagree")
            self.entries[name] = (dtype, off, nb, dims)

    def __contains__(self, name):
        return name in self.entries

    def names(self):
        return list(self.entries)

    def raw(self, name):
        dtype, off, nb, dims = self.entries[name]
        return self.data[off:off + nb]

    def __getitem__(self, name):
        dtype, off, nb, dims = self.entries[name]
        return np.frombuffer(self.data, dtype=DTYPES[dtype], count=int(np.prod(dims, dtype=np.int64)), offset=off).reshape(dims)

    def f32(self, name):
        """float32 (float16 widened exactly), flat"""
        return np.asarray(self[name], dtype=np.float32).reshape(-1)


def write(path, tensors):
    """Write `tensors` (name -> numpy array, in order) as a bundle, laid out as store.rs:431-464 does."""
    items = [(k, np.ascontiguousarray(v)) for k, v in tensors.items()]

    def line(k, v, off):
        dims = " ".join(str(x) for x in v.shape)
        return f"{k} {v.dtype.name} {off} {v.nbytes}" + (f" {dims}" if dims else "") + "\n"

    guess = sum(len(line(k, v, 10 ** 15)) for k, v in items) + 16
    pos = (guess + 63) // 64 * 64
    offs = []
    for _, v in items:
        offs.append(pos)
        pos = (pos + v.nbytes + 63) // 64 * 64
    index = "".join(line(k, v, o) for (k, v), o in zip(items, offs)).encode()
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<Q", len(index)) + index)
        for (_, v), o in zip(items, offs):
            f.seek(o)
            f.write(v.astype(v.dtype.newbyteorder("<"), copy=False).tobytes())
        f.truncate(pos)
