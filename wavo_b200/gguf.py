"""GGUF files on the host: `Gguf` mirrors the reference's reader (src/gguf.rs: `Gguf::open`, `get`,
`optional`, `array`, `tensor`, `Tensor::read`) over the library's native reader, and `write_gguf`
writes a GGUF v3 file (metadata values and F32 / F16 / Q8_0 tensors) in the layout that reader
parses, for tests and benchmarks that need a file. A layer's weights go to the device straight
from the file with `Gpu.linear_from_gguf`."""

from __future__ import annotations

import ctypes
import struct

import numpy as np

from . import _lib as L

TY_F32, TY_F16, TY_Q8_0 = 0, 1, 8
# GGUF value types (the reference's reader, src/gguf.rs:346-363).
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARRAY, U64, I64, F64 = range(13)


class GgufError(RuntimeError):
    pass


def _check(status: int) -> None:
    if status != 0:
        msg = L.lib().wavo_last_error(None)
        raise GgufError(msg.decode() if msg else f"status {status}")


class Gguf:
    """`Gguf::open`: the header is read and checked, tensor data is read when used."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _check(L.lib().wavo_gguf_open(str(path).encode(), ctypes.byref(h)))
        self.h = h
        self.path = str(path)

    def close(self) -> None:
        if L is None or L.lib is None:  # interpreter shutdown: the process releases the file
            return
        if getattr(self, "h", None) is not None and self.h.value:
            L.lib().wavo_gguf_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def names(self) -> list[str]:
        n = L.lib().wavo_gguf_tensor_count(self.h)
        return [L.lib().wavo_gguf_tensor_name(self.h, i).decode() for i in range(n)]

    def dims(self, name: str) -> list[int]:
        buf = (ctypes.c_uint64 * 8)()
        n = L.lib().wavo_gguf_tensor_dims(self.h, name.encode(), buf, 8)
        if n == 0:
            raise GgufError(f"missing tensor {name}")
        return list(buf[:n])

    def tensor(self, name: str, dims=None) -> tuple[int, int]:
        """`Gguf::tensor`: (GGUF type, data bytes) of `name`, which must have exactly the ggml-order
        `dims` when given."""
        ty, nb = ctypes.c_int(), ctypes.c_uint64()
        arr = None if dims is None else (ctypes.c_uint64 * len(dims))(*dims)
        _check(L.lib().wavo_gguf_tensor(self.h, name.encode(), arr, 0 if dims is None else len(dims),
                                        ctypes.byref(ty), ctypes.byref(nb)))
        return ty.value, nb.value

    def read(self, name: str, offset: int = 0, nbytes: int | None = None) -> bytes:
        """`Tensor::read`: the tensor's data bytes from `offset`."""
        if nbytes is None:
            nbytes = self.tensor(name)[1] - offset
        buf = ctypes.create_string_buffer(max(nbytes, 1))
        _check(L.lib().wavo_gguf_read(self.h, name.encode(), offset, buf, nbytes))
        return buf.raw[:nbytes]

    def to_f32(self, name: str) -> np.ndarray:
        """`Tensor::to_f32`."""
        ty, _ = self.tensor(name)
        b = self.read(name)
        if ty == TY_F32:
            return np.frombuffer(b, "<f4").astype(np.float32)
        if ty == TY_F16:
            return np.frombuffer(b, "<f2").astype(np.float32)
        blocks = np.frombuffer(b, np.uint8).reshape(-1, 34)
        d = blocks[:, :2].copy().view("<f2").astype(np.float32)
        return (blocks[:, 2:].view(np.int8).astype(np.float32) * d).ravel()

    def has(self, key: str) -> bool:
        return bool(L.lib().wavo_gguf_has(self.h, key.encode()))

    _RANGES = {"u32": (0, 2**32 - 1), "i32": (-2**31, 2**31 - 1)}

    def get(self, key: str, kind):
        """`Gguf::get::<T>` for T in int, "u32", "i32" (integers that must fit), float, bool, str."""
        k = key.encode()
        if kind is int or kind in self._RANGES:
            v = ctypes.c_int64()
            _check(L.lib().wavo_gguf_get_int(self.h, k, ctypes.byref(v)))
            lo, hi = self._RANGES.get(kind, (-2**63, 2**63 - 1))
            if not lo <= v.value <= hi:
                raise GgufError(f"metadata {key}: {v.value} is not a {kind}")
            return v.value
        if kind is float:
            v = ctypes.c_double()
            _check(L.lib().wavo_gguf_get_float(self.h, k, ctypes.byref(v)))
            return v.value
        if kind is bool:
            v = ctypes.c_int()
            _check(L.lib().wavo_gguf_get_bool(self.h, k, ctypes.byref(v)))
            return bool(v.value)
        p, n = ctypes.c_void_p(), ctypes.c_uint64()
        _check(L.lib().wavo_gguf_get_str(self.h, k, ctypes.byref(p), ctypes.byref(n)))
        return ctypes.string_at(p.value, n.value).decode() if n.value else ""

    def optional(self, key: str, kind):
        """`Gguf::optional`: None when the file has no `key`."""
        return self.get(key, kind) if self.has(key) else None

    def optional_array(self, key: str, kind) -> list:
        """`Gguf::optional_array`: empty when the file has no `key`."""
        return self.array(key, kind) if self.has(key) else []

    def array(self, key: str, kind) -> list:
        """`Gguf::array::<T>` for T in int, "u32", "i32", float, str."""
        item, n = ctypes.c_uint32(), ctypes.c_uint64()
        _check(L.lib().wavo_gguf_array(self.h, key.encode(), ctypes.byref(item), ctypes.byref(n)))
        count = n.value
        cap = max(count, 1)
        if kind is int or kind in self._RANGES:
            out = (ctypes.c_int64 * cap)()
            _check(L.lib().wavo_gguf_array_items(self.h, key.encode(), out, None, None, None, count))
            lo, hi = self._RANGES.get(kind, (-2**63, 2**63 - 1))
            if any(not lo <= x <= hi for x in out[:count]):
                raise GgufError(f"metadata {key}: expected an array of {kind}")
            return list(out[:count])
        if kind is float:
            out = (ctypes.c_double * cap)()
            _check(L.lib().wavo_gguf_array_items(self.h, key.encode(), None, out, None, None, count))
            return list(out[:count])
        ptrs, lens = (ctypes.c_void_p * cap)(), (ctypes.c_uint64 * cap)()
        _check(L.lib().wavo_gguf_array_items(self.h, key.encode(), None, None, ptrs, lens, count))
        return [ctypes.string_at(ptrs[i], lens[i]).decode() if lens[i] else "" for i in range(count)]


# ---- writing ---------------------------------------------------------------------------------

def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


def _value(ty: int, v) -> bytes:
    if ty == STR:
        return _str(v)
    if ty == ARRAY:
        item, items = v
        return struct.pack("<IQ", item, len(items)) + b"".join(_value(item, x) for x in items)
    return struct.pack(_FMT[ty], int(v) if ty == BOOL else v)


def q8_0_blocks(w: np.ndarray) -> bytes:
    """Q8_0 blocks of `w` (a multiple of 32 values): d = max|x| / 127 as f16, q = round(x / d)."""
    x = np.asarray(w, np.float32).reshape(-1, 32)
    d = (np.abs(x).max(axis=1) / 127.0).astype(np.float16)
    df = d.astype(np.float32)
    q = np.where(df[:, None] > 0, np.rint(x / np.where(df > 0, df, 1)[:, None]), 0)
    q = np.clip(q, -127, 127).astype(np.int8)
    return b"".join(d[i].tobytes() + q[i].tobytes() for i in range(len(d)))


def write_gguf(path: str, meta: list[tuple[str, int, object]],
               tensors: list[tuple[str, list[int], int, bytes]], alignment: int = 32) -> None:
    """A GGUF v3 file: `meta` as (key, GGUF value type, value) — an ARRAY value is (item type,
    items) — and `tensors` as (name, ggml-order dims, type, data bytes), each tensor's data at the
    next multiple of `alignment` (recorded as general.alignment when it is not 32)."""
    meta = list(meta)
    if alignment != 32:
        meta.append(("general.alignment", U32, alignment))
    head = bytearray(b"GGUF") + struct.pack("<IQQ", 3, len(tensors), len(meta))
    for key, ty, v in meta:
        head += _str(key) + struct.pack("<I", ty) + _value(ty, v)
    offsets, at = [], 0
    for _, _, _, data in tensors:
        offsets.append(at)
        at += len(data)
        at += -at % alignment
    for (name, dims, ty, _), off in zip(tensors, offsets):
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", ty, off)
    head += b"\0" * (-len(head) % alignment)
    with open(path, "wb") as fh:
        fh.write(head)
        pos = 0
        for (_, _, _, data), off in zip(tensors, offsets):
            fh.write(b"\0" * (off - pos))
            fh.write(data)
            pos = off + len(data)
