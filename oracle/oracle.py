"""ctypes wrapper of the CPU oracle (``oracle/libwavo_oracle.so``).

TEST INFRASTRUCTURE ONLY: a restatement of the reference's CPU attention path (vladkens/wavo
src/cpu/ops.rs, src/cpu/gemm.rs, src/cpu/mod.rs) used as the checker of the CUDA kernels and as the
timed CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) import this module; no product code does.
Each function cites the reference function it restates (see wavo_oracle.cpp for file:line).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libwavo_oracle.so")
_lib = None

EPILOGUES = {"bias": 0, "silu": 1, "relu": 2, "residual": 3, "gelu": 4, "gelu_residual": 5, "tanh": 6}
TY_F32, TY_F16, TY_Q8_0 = 0, 1, 8

_f = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t


def build() -> None:
    """Compile the oracle library in place (make)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.wo_random.argtypes = [_f, _sz, ctypes.c_uint32]
        L.wo_to_half.argtypes = [ctypes.c_float]
        L.wo_to_half.restype = ctypes.c_float
        L.wo_to_half_n.argtypes = [_f, _f, _sz]
        L.wo_f16_bits.argtypes = [ctypes.c_float]
        L.wo_f16_bits.restype = ctypes.c_uint16
        L.wo_f16_round_n.argtypes = [_f, _f, _sz]
        for name in ("wo_exp", "wo_silu", "wo_gelu"):
            getattr(L, name).argtypes = [ctypes.c_float]
            getattr(L, name).restype = ctypes.c_float
        L.wo_dot.argtypes = [_f, _f, _sz]
        L.wo_dot.restype = ctypes.c_float
        L.wo_attention.argtypes = [_f, _sz, _f, _sz, _f, _sz, _sz, _sz]
        L.wo_relative_attention.argtypes = [_f, _f, _f, _f, _f, _sz, _sz, _sz]
        L.wo_relative_attention.restype = ctypes.c_int
        L.wo_attend.argtypes = [_f, _f, _sz, _sz, _f, _sz, _sz]
        L.wo_pack_cache.argtypes = [_f, _sz, _sz, _sz, _f, _sz, _sz]
        L.wo_rope.argtypes = [_f, _f, _sz, _sz, _sz, _sz, ctypes.c_int]
        L.wo_rope_table.argtypes = [_sz, _sz, ctypes.c_double, _f]
        L.wo_layer_norm.argtypes = [_f, _f, _f, _f, _sz, _sz, _f, _f, _sz]
        _i = ctypes.POINTER(ctypes.c_int32)
        L.wo_pick.argtypes = [_f, _sz, _i, _sz, _i, _sz, _i, _sz, _sz, _sz, _sz, _sz, ctypes.c_int,
                              _f]
        L.wo_pick.restype = ctypes.c_int
        L.wo_conv_glu.argtypes = [_f, _f, _f, _f, _f, ctypes.c_int, _f, _sz, _sz, _sz]
        L.wo_rel_positions.argtypes = [_sz, ctypes.c_int64, _sz, _f]
        L.wo_pos_rows.argtypes = [_sz]
        L.wo_pos_rows.restype = _sz
        L.wo_linear_new.argtypes = [ctypes.c_int, _sz, _sz, ctypes.c_void_p, _f]
        L.wo_linear_new.restype = ctypes.c_void_p
        L.wo_linear_free.argtypes = [ctypes.c_void_p]
        L.wo_gemm.argtypes = [_f, ctypes.c_void_p, _f, _sz, ctypes.c_int, ctypes.c_float]
        L.wo_gemv.argtypes = [_f, ctypes.c_void_p, _f, ctypes.c_int, ctypes.c_float]
        _d = ctypes.POINTER(ctypes.c_double)
        L.wo_fft.argtypes = [_d, _sz, _d, _d]
        L.wo_log_mel.argtypes = [_f, _sz, _sz, _sz, _f]
        L.wo_mel_features.argtypes = [_f, _sz, _f]
        L.wo_mel_features.restype = _sz
        L.wo_frontend_tables.argtypes = [_d, _f]
        L.wo_subsample.argtypes = [_f, _sz, _sz, _sz, _f, _f, _f, _f, ctypes.c_void_p, _f, _f,
                                   ctypes.c_void_p, ctypes.c_void_p, _f]
        L.wo_subsample.restype = _sz
        L.wo_set_threads.argtypes = [ctypes.c_int]
        L.wo_threads.restype = ctypes.c_int
        L.wo_set_vnni.argtypes = [ctypes.c_int]
        L.wo_vnni.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


def random(n: int, seed: int) -> np.ndarray:
    """The reference tests' xorshift32 values in [-1, 1] (src/gpu/mod.rs:1717-1727)."""
    out = np.empty(n, np.float32)
    lib().wo_random(_p(out), n, seed)
    return out


def to_half(x: np.ndarray) -> np.ndarray:
    """src/cpu/gemm.rs:210-221 `to_half`."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().wo_to_half_n(_p(x), _p(y), x.size)
    return y


def f16_round(x: np.ndarray) -> np.ndarray:
    """`half::f16::from_f32(x).to_f32()` (IEEE round to nearest even)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().wo_f16_round_n(_p(x), _p(y), x.size)
    return y


def exp(x: float) -> float:
    """src/cpu/ops.rs:12-26 (Cephes expf)."""
    return lib().wo_exp(x)


def attention(qk, ld, v, ldv, t, heads, ch) -> np.ndarray:
    """src/cpu/ops.rs:187-221 `attention` -> o [t][ch]."""
    o = np.zeros(t * ch, np.float32)
    lib().wo_attention(_p(qk), ld, _p(v), ldv, _p(o), t, heads, ch)
    return o.reshape(t, ch)


def relative_attention(qkv, pos, u, vb, t, heads, ch) -> np.ndarray:
    """src/cpu/ops.rs:223-273 `relative_attention` over qkv [t][q|k|v] -> o [t][ch]."""
    o = np.zeros(t * ch, np.float32)
    if lib().wo_relative_attention(_p(qkv), _p(pos), _p(u), _p(vb), _p(o), t, heads, ch) != 0:
        raise ValueError("relative_attention needs heads of a multiple of 16 dims")
    return o.reshape(t, ch)


def attend(q, kv, cols, n, heads, hd) -> np.ndarray:
    """src/cpu/ops.rs:300-337 `attend` over a cache [K heads][cols][hd] + [V heads][cols][hd]."""
    o = np.zeros(heads * hd, np.float32)
    lib().wo_attend(_p(q), _p(kv), cols, n, _p(o), heads, hd)
    return o


def pack_cache(kv, rows, d, hd, cache, cols, col) -> None:
    """src/cpu/transformer.rs:209-222 `Decoder::pack` (in place into cache)."""
    lib().wo_pack_cache(_p(kv), rows, d, hd, _p(cache), cols, col)


def rope(qkv, table, rows, heads, hd, rot, neox) -> None:
    """src/cpu/ops.rs:339-355 `rope` (in place)."""
    lib().wo_rope(_p(qkv), _p(table), rows, heads, hd, rot, int(neox))


def layer_norm(x, w, b, rows, cols, table=None, hd=0):
    """src/cpu/ops.rs:65-110 `layer_norm` (eps 1e-5); with a table (row r for row r) also the
    rotated copy yr. Returns y, or (y, yr)."""
    y = np.zeros(rows * cols, np.float32)
    yr = np.zeros(rows * cols, np.float32) if table is not None else None
    lib().wo_layer_norm(_p(np.ascontiguousarray(x, np.float32)), _p(np.ascontiguousarray(w, np.float32)),
                        _p(np.ascontiguousarray(b, np.float32)), _p(y), rows, cols,
                        _p(np.ascontiguousarray(table, np.float32)) if table is not None else None,
                        _p(yr) if yr is not None else None, hd)
    return y if yr is None else (y, yr)


def conv_glu(h, taps, bias, g, beta, layer_norm, t, ch, kernel):
    """src/cpu/ops.rs:133-182 `conv_glu`: h [t][2ch] is updated in place (GLU into its first
    halves); returns y [t][ch]."""
    y = np.zeros(t * ch, np.float32)
    lib().wo_conv_glu(_p(h), _p(np.ascontiguousarray(taps, np.float32)),
                      _p(np.ascontiguousarray(bias, np.float32)), _p(np.ascontiguousarray(g, np.float32)),
                      _p(np.ascontiguousarray(beta, np.float32)), int(layer_norm), _p(y), t, ch, kernel)
    return y


def pick(logits, generated, suppress, begin_suppress, eot, no_timestamps, begin,
         max_initial=50, logprob=True):
    """src/whisper/search.rs:46-59 `pick` (suppression, timestamp rules, argmax): logits (f32,
    edited in place) of one row, the window's generated tokens; returns (token, log-probability)."""
    i32 = lambda a: np.ascontiguousarray(np.asarray(a, np.int32))  # noqa: E731
    gen, sup, bsup = i32(generated), i32(suppress), i32(begin_suppress)
    ip = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))  # noqa: E731
    lp = np.zeros(1, np.float32)
    tok = lib().wo_pick(_p(logits), logits.size, ip(gen), gen.size, ip(sup), sup.size, ip(bsup),
                        bsup.size, eot, no_timestamps, begin, max_initial, int(logprob), _p(lp))
    return int(tok), float(lp[0])


def rope_table(frames, hd, theta) -> np.ndarray:
    """src/gigaam/mod.rs:88-96 `rope`: [frames][hd/2 cos | hd/2 sin]."""
    out = np.empty(frames * hd, np.float32)
    lib().wo_rope_table(frames, hd, float(theta), _p(out))
    return out


def rel_positions(d, first, rows) -> np.ndarray:
    """src/conformer.rs:141-153 `rel_positions`."""
    out = np.empty(rows * d, np.float32)
    lib().wo_rel_positions(d, first, rows, _p(out))
    return out.reshape(rows, d)


def pos_rows(t: int) -> int:
    """src/gpu/mod.rs:1060-1065."""
    return 2 * t + 15


class Linear:
    """src/cpu/gemm.rs:36-75 `Linear` over GGUF bytes (F32 / F16 / Q8_0) and an optional bias."""

    def __init__(self, ty: int, n: int, k: int, data: bytes, bias=None):
        self.n, self.k, self.ty = n, k, ty
        self._buf = ctypes.create_string_buffer(bytes(data), len(data))
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._h = lib().wo_linear_new(ty, n, k, ctypes.cast(self._buf, ctypes.c_void_p),
                                      None if b is None else _p(b))

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.wo_linear_free(self._h)
            self._h = None

    def gemm(self, a: np.ndarray, m: int, c: np.ndarray | None = None, epilogue="bias", alpha=1.0):
        """src/cpu/gemm.rs:125-177 `gemm`: c = epilogue(a·W^T + b); c updated in place."""
        if c is None:
            c = np.zeros(m * self.n, np.float32)
        lib().wo_gemm(_p(a), self._h, _p(c), m, EPILOGUES[epilogue], alpha)
        return c

    def gemv(self, x: np.ndarray, c: np.ndarray | None = None, epilogue="bias", alpha=1.0):
        """src/cpu/gemm.rs:179-208 `gemv`."""
        if c is None:
            c = np.zeros(self.n, np.float32)
        lib().wo_gemv(_p(x), self._h, _p(c), EPILOGUES[epilogue], alpha)
        return c


def set_threads(n: int) -> None:
    lib().wo_set_threads(n)


def threads() -> int:
    return lib().wo_threads()


def set_vnni(mode: int) -> None:
    """-1 detect (the reference's choice), 0 the f16 path, 1/2 the i16 VNNI path."""
    lib().wo_set_vnni(mode)


def vnni() -> int:
    return lib().wo_vnni()


def q8_0_bytes(values: np.ndarray, scale_mode: str = "absmax") -> bytes:
    """GGUF Q8_0 blocks (f16 scale + 32 int8) of float rows, as the reference test builds them
    (src/gpu/mod.rs:1888-1895: d = max|x| / 127 in f32, q = x / d rounded half away from zero,
    saturated as Rust's `as i8`)."""
    v = np.ascontiguousarray(values, np.float32).reshape(-1, 32)
    out = bytearray()
    for blk in v:
        d = np.float32(np.abs(blk).max()) / np.float32(127.0)
        if d != 0:
            y = (blk / d).astype(np.float64)  # f32 quotient, as the reference divides
            q = np.clip(np.sign(y) * np.floor(np.abs(y) + 0.5), -128, 127).astype(np.int8)
        else:
            q = np.zeros(32, np.int8)
        out += np.float16(d).tobytes() + q.tobytes()
    return bytes(out)


# ---- the log-mel frontend (src/parakeet/frontend.rs, src/fft.rs) ----------------------------------

MELS, HOP = 128, 160


def _pd(a: np.ndarray):
    assert a.dtype == np.float64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def fft(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """src/fft.rs `Fft::<f64>::new(n).forward(x)`: the DFT of n real values (re, im)."""
    x = np.ascontiguousarray(x, np.float64)
    re, im = np.empty(x.size), np.empty(x.size)
    lib().wo_fft(_pd(x), x.size, _pd(re), _pd(im))
    return re, im


def log_mel(pcm: np.ndarray, f0: int, f1: int) -> np.ndarray:
    """src/parakeet/frontend.rs:74-108 `Frontend::log_mel`: frames [f0, f1) of 16 kHz pcm."""
    pcm = np.ascontiguousarray(pcm, np.float32)
    out = np.empty((f1 - f0, MELS), np.float32)
    lib().wo_log_mel(_p(pcm), pcm.size, f0, f1, _p(out))
    return out


def mel_features(pcm: np.ndarray) -> np.ndarray:
    """src/parakeet/frontend.rs:50-70 `Frontend::compute`: normalised log-mel [frames][128], empty
    below 3 frames."""
    pcm = np.ascontiguousarray(pcm, np.float32)
    frames = pcm.size // HOP + 1
    out = np.empty((max(frames, 1), MELS), np.float32)
    n = lib().wo_mel_features(_p(pcm), pcm.size, _p(out))
    return out[:n] if n else np.empty((0, MELS), np.float32)


def frontend_tables() -> tuple[np.ndarray, np.ndarray]:
    """The Hann window [512] (f64) and the Slaney filterbank [128][257] (f32)."""
    w, f = np.empty(512), np.empty((MELS, 257), np.float32)
    lib().wo_frontend_tables(_pd(w), _p(f))
    return w, f


def subsample(mel: np.ndarray, valid: int, taps: dict, conv3: "Linear", conv6: "Linear",
              out: "Linear") -> np.ndarray:
    """src/parakeet/cpu.rs:60-98: Parakeet's 8x conv subsampling of mel [frames][128] (valid frames
    of them) into x [t][d]; taps: w0, b0, w2, b2, w5, b5 (3x3 taps [9][ch], biases [ch])."""
    mel = np.ascontiguousarray(mel, np.float32)
    frames = mel.shape[0]
    h = lambda n: (n - 1) // 2 + 1  # noqa: E731
    t = h(h(h(frames - 1)))
    ch = taps["b0"].size
    x = np.zeros((t, out.n), np.float32)
    c = {k: np.ascontiguousarray(v, np.float32) for k, v in taps.items()}
    lib().wo_subsample(_p(mel), frames, valid, ch, _p(c["w0"]), _p(c["b0"]), _p(c["w2"]),
                       _p(c["b2"]), conv3._h, _p(c["w5"]), _p(c["b5"]), conv6._h, out._h, _p(x))
    return x
