"""Writes tests/golden/gguf_sample.gguf: the small GGUF v3 file of the reference's reader test
(src/gguf.rs:382-440 `sample`), byte for byte as that test assembles it: six metadata values (a u32,
a string array, a bool, a negative i32, an i32 array, an f32) and two tensors (an F32 [2, 1] and a
Q8_0 [32]). tests/test_gguf.py checks this library's reader against the reference test's
assertions on it (src/gguf.rs:447-480).

    python tests/golden/make_gguf_sample.py
"""

import os
import struct

import numpy as np


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def sample() -> bytes:
    f = bytearray(b"GGUF")
    f += struct.pack("<IQQ", 3, 2, 6)
    f += _str("a.n") + struct.pack("<II", 4, 7)
    f += _str("a.tokens") + struct.pack("<IIQ", 9, 8, 2) + _str("▁x") + _str("y")
    f += _str("a.flag") + struct.pack("<I", 7) + b"\x01"
    f += _str("a.left") + struct.pack("<Ii", 5, -1)
    f += _str("a.durations") + struct.pack("<IIQ", 9, 5, 3) + struct.pack("<3i", 0, 2, -4)
    f += _str("a.alpha") + struct.pack("<If", 6, 0.97)
    f += _str("w") + struct.pack("<IQQIQ", 2, 2, 1, 0, 0)
    f += _str("q") + struct.pack("<IQIQ", 1, 32, 8, 32)
    f += b"\0" * (-len(f) % 32)
    f += struct.pack("<ff", 1.5, -2.0)
    f += b"\0" * (-len(f) % 32)
    f += np.float16(0.5).tobytes() + bytes((i - 16) & 0xFF for i in range(32))
    return bytes(f)


if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gguf_sample.gguf")
    with open(out, "wb") as fh:
        fh.write(sample())
    print(out, len(sample()), "bytes")
