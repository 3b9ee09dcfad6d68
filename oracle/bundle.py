"""B2DB bundle files: the exchange format between the oracle, the reference
harness (oracle/ref/harness.cpp) and the golden fixtures under tests/golden.

Layout: b"B2DB", u32 version (1), u32 count, then per entry
  u16 name_len, name (utf-8), u8 dtype, u8 ndim, i64 dims[ndim], u64 nbytes, bytes.
dtype codes: 0 f32, 1 f16, 2 bf16 (u16 payload), 3 q8_0 (34-byte blocks, u8
payload), 4 i64, 5 i32, 6 u8.  Weight dims follow the reference's tensor
metadata order ([out, in] for linears, innermost last).
"""
from __future__ import annotations

import struct
from typing import Dict, Tuple

import numpy as np

F32, F16, BF16, Q8_0, I64, I32, U8 = range(7)
_NP = {F32: np.float32, F16: np.float16, BF16: np.uint16, Q8_0: np.uint8,
       I64: np.int64, I32: np.int32, U8: np.uint8}


class Tensor:
    """A bundle entry: dtype code, logical dims and a flat numpy payload."""

    __slots__ = ("dtype", "dims", "data")

    def __init__(self, dtype: int, dims, data: np.ndarray):
        self.dtype = int(dtype)
        self.dims = tuple(int(d) for d in dims)
        self.data = np.ascontiguousarray(data)

    def array(self) -> np.ndarray:
        if self.dtype in (F32, F16, I64, I32):
            return self.data.reshape(self.dims)
        return self.data


def f32(a) -> Tensor:
    a = np.asarray(a, dtype=np.float32)
    return Tensor(F32, a.shape if a.ndim else (1,), a.reshape(-1))


def i64(a) -> Tensor:
    a = np.asarray(a, dtype=np.int64)
    return Tensor(I64, a.shape if a.ndim else (1,), a.reshape(-1))


def write(path: str, entries: Dict[str, Tensor]) -> None:
    with open(path, "wb") as fh:
        fh.write(b"B2DB")
        fh.write(struct.pack("<II", 1, len(entries)))
        for name in sorted(entries):
            t = entries[name]
            nb = name.encode()
            payload = t.data.tobytes()
            fh.write(struct.pack("<H", len(nb)))
            fh.write(nb)
            fh.write(struct.pack("<BB", t.dtype, len(t.dims)))
            fh.write(struct.pack("<%dq" % len(t.dims), *t.dims))
            fh.write(struct.pack("<Q", len(payload)))
            fh.write(payload)


def read(path: str) -> Dict[str, Tensor]:
    with open(path, "rb") as fh:
        buf = fh.read()
    if buf[:4] != b"B2DB":
        raise ValueError("not a B2DB bundle: %s" % path)
    _, count = struct.unpack_from("<II", buf, 4)
    off = 12
    out: Dict[str, Tensor] = {}
    for _ in range(count):
        (nlen,) = struct.unpack_from("<H", buf, off); off += 2
        name = buf[off:off + nlen].decode(); off += nlen
        dtype, ndim = struct.unpack_from("<BB", buf, off); off += 2
        dims: Tuple[int, ...] = struct.unpack_from("<%dq" % ndim, buf, off); off += 8 * ndim
        (nbytes,) = struct.unpack_from("<Q", buf, off); off += 8
        data = np.frombuffer(buf, dtype=_NP[dtype], count=nbytes // np.dtype(_NP[dtype]).itemsize, offset=off).copy()
        off += nbytes
        out[name] = Tensor(dtype, dims, data)
    return out
