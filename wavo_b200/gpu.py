"""Host-side mirror of the reference's GPU backend op interface for the attention path
(vladkens/wavo src/gpu/mod.rs: `Gpu`, `Linear`, `Pass`), over the C ABI of libwavo_cuda.

Device memory comes from torch (CUDA tensors); the context runs on torch's current stream, so the
calls order with the torch work around them. Method names, argument meanings and layouts follow the
reference; errors raise `WavoError` at the call (argument errors) or at `Gpu.sync` (device errors),
as the reference returns `Error::Model` at load and `Error::Gpu`/`Poll` at completion.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L
from ._lib import WavoError, check  # noqa: F401  (re-exported)

EPILOGUES = L.EPILOGUES


def _ptr(t) -> int | None:
    if t is None:
        return None
    assert t.is_cuda, "buffers are CUDA tensors"
    return t.data_ptr()


def _dtype(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.F32
    if t.dtype == torch.float16:
        return L.F16
    raise TypeError(f"unsupported buffer dtype {t.dtype} (float32 or float16)")


def pos_rows(t: int) -> int:
    """src/gpu/mod.rs:1060-1065."""
    return 2 * t + 15


def attend_len(n: int, heads: int, hd: int) -> int:
    """src/gpu/mod.rs:1053-1059 (this build's split size)."""
    return int(L.lib().wavo_attend_len(n, heads, hd))


def device_count() -> int:
    return int(L.lib().wavo_device_count())


class Linear:
    """`Gpu::linear` (src/gpu/mod.rs:758-834): W [rows][k] in a GGUF type, stacked tensors along
    the rows, a bias of 0, rows or rows + dual values."""

    def __init__(self, gpu: "Gpu", ggml_type: int, rows: int, k: int, data: bytes | np.ndarray,
                 bias=None):
        raw = bytes(data) if not isinstance(data, np.ndarray) else data.tobytes()
        self._buf = ctypes.create_string_buffer(raw, len(raw))
        b = None
        if bias is not None and len(bias):
            b = np.ascontiguousarray(bias, np.float32)
        self._bias = b
        h = ctypes.c_void_p()
        check(L.lib().wavo_linear_create(gpu.ctx, ggml_type, rows, k, ctypes.addressof(self._buf),
                                         None if b is None else b.ctypes.data,
                                         0 if b is None else b.size, ctypes.byref(h)), gpu.ctx)
        self.h = h
        self.rows, self.k, self.ty = rows, k, ggml_type
        self.n = (rows + 63) // 64 * 64
        self.cols = rows if rows % 32 == 0 else self.n
        self.dual = int(L.lib().wavo_linear_width(h)) - self.cols
        del self._buf

    @classmethod
    def from_gguf(cls, gpu: "Gpu", gguf, names: list[str], bias=None) -> "Linear":
        """`Gpu::linear(&[Tensor], bias)` with the tensors streamed from a GGUF file
        (`wavo_linear_from_gguf`)."""
        self = cls.__new__(cls)
        b = None
        if bias is not None and len(bias):
            b = np.ascontiguousarray(bias, np.float32)
        self._bias = b
        arr = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        h = ctypes.c_void_p()
        check(L.lib().wavo_linear_from_gguf(gpu.ctx, gguf.h, arr, len(names),
                                            None if b is None else b.ctypes.data,
                                            0 if b is None else b.size, ctypes.byref(h)), gpu.ctx)
        self.h = h
        ty, _ = gguf.tensor(names[0])
        dims = gguf.dims(names[0])
        self.k = int(np.prod(dims)) // dims[-1]
        self.rows = sum(gguf.dims(n)[-1] for n in names)
        self.ty = ty
        self.n = (self.rows + 63) // 64 * 64
        self.cols = self.rows if self.rows % 32 == 0 else self.n
        self.dual = int(L.lib().wavo_linear_width(h)) - self.cols
        return self

    def width(self) -> int:
        """`Linear::width`: output columns including the dual ones."""
        return self.cols + self.dual

    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and h.value and L is not None and L.lib is not None:
            L.lib().wavo_linear_destroy(h)
            self.h = None


class Gpu:
    """`Gpu::new` (src/gpu/mod.rs:461-578): a context on one B200, on torch's current stream."""

    def __init__(self, device: int = 0):
        self.device = device
        self.torch_device = torch.device("cuda", device)
        ctx = ctypes.c_void_p()
        check(L.lib().wavo_create(device, ctypes.byref(ctx)), None)
        self.ctx = ctx
        with torch.cuda.device(device):
            self.use_stream(torch.cuda.current_stream(device))

    def use_stream(self, stream: torch.cuda.Stream) -> None:
        check(L.lib().wavo_set_stream(self.ctx, stream.cuda_stream), self.ctx)

    def close(self) -> None:
        if L is None or L.lib is None:  # interpreter shutdown: the process releases the device
            return
        if getattr(self, "ctx", None) is not None and self.ctx.value:
            L.lib().wavo_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        self.close()

    @property
    def sm_count(self) -> int:
        return int(L.lib().wavo_sm_count(self.ctx))

    def linear(self, ggml_type: int, rows: int, k: int, data, bias=None) -> Linear:
        return Linear(self, ggml_type, rows, k, data, bias)

    def log_mel(self, pcm: torch.Tensor, f0: int, f1: int, mel: torch.Tensor) -> None:
        """`Frontend::log_mel`: frames f0..f1 of the 16 kHz pcm into mel [f1 - f0][128]."""
        check(L.lib().wavo_log_mel(self.ctx, _ptr(pcm), pcm.numel(), f0, f1, _ptr(mel)), self.ctx)

    def mel_features(self, pcm: torch.Tensor, mel: torch.Tensor) -> int:
        """`Frontend::compute`: the normalised features into mel; returns the frames (0 below 3)."""
        n = ctypes.c_uint64()
        check(L.lib().wavo_mel_features(self.ctx, _ptr(pcm), pcm.numel(), _ptr(mel),
                                        ctypes.byref(n)), self.ctx)
        return n.value

    def subsample(self, mel: torch.Tensor, valid: int, taps: dict, conv3: Linear, conv6: Linear,
                  out: Linear, x: torch.Tensor, scratch: torch.Tensor | None = None) -> int:
        """Parakeet's 8x conv subsampling of mel [frames][128] into x [t][d]; taps: device f32
        w0, b0, w2, b2, w5, b5 ([9][ch] taps, [ch] biases). Returns t."""
        frames, ch = mel.shape[0], taps["b0"].numel()
        if scratch is None:
            nbytes = int(L.lib().wavo_subsample_scratch_bytes(frames, ch))
            scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.torch_device)
        base = (scratch.data_ptr() + 255) // 256 * 256
        t = ctypes.c_uint32()
        check(L.lib().wavo_subsample(self.ctx, _ptr(mel), frames, valid, ch, _ptr(taps["w0"]),
                                     _ptr(taps["b0"]), _ptr(taps["w2"]), _ptr(taps["b2"]), conv3.h,
                                     _ptr(taps["w5"]), _ptr(taps["b5"]), conv6.h, out.h, _ptr(x),
                                     base, ctypes.byref(t)), self.ctx)
        self._keep = scratch  # the launches read it until the stream passes them
        return t.value

    def subsample_batch(self, mel: torch.Tensor, frames, valid, taps: dict, conv3: Linear,
                        conv6: Linear, out: Linear, x: torch.Tensor,
                        scratch: torch.Tensor | None = None) -> list[int]:
        """subsample over segments whose mel rows (frames[s] each, valid[s] of them audio) follow
        one another in mel; their output rows follow one another in x. Returns each t_s."""
        n, ch = len(frames), taps["b0"].numel()
        fr = (ctypes.c_uint32 * max(n, 1))(*[int(f) for f in frames])
        va = (ctypes.c_uint32 * max(n, 1))(*[int(v) for v in valid])
        ts = (ctypes.c_uint32 * max(n, 1))()
        if scratch is None:
            nbytes = int(L.lib().wavo_subsample_batch_scratch_bytes(fr, n, ch))
            scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.torch_device)
        base = (scratch.data_ptr() + 255) // 256 * 256
        check(L.lib().wavo_subsample_batch(self.ctx, _ptr(mel), fr, va, n, ch, _ptr(taps["w0"]),
                                           _ptr(taps["b0"]), _ptr(taps["w2"]), _ptr(taps["b2"]),
                                           conv3.h, _ptr(taps["w5"]), _ptr(taps["b5"]), conv6.h,
                                           out.h, _ptr(x), base, ts), self.ctx)
        self._keep = scratch  # the launches read it until the stream passes them
        return list(ts)[:n]

    def linear_from_gguf(self, gguf, names: list[str], bias=None) -> Linear:
        """`Gpu::linear` over GGUF tensors, streamed from the file to the device."""
        return Linear.from_gguf(self, gguf, names, bias)

    def buffer(self, n: int, dtype=torch.float32) -> torch.Tensor:
        """`Gpu::buffer`: zeroed device memory."""
        return torch.zeros(n, dtype=dtype, device=self.torch_device)

    def upload(self, data, dtype=torch.float32) -> torch.Tensor:
        """`Gpu::upload`."""
        return torch.as_tensor(np.ascontiguousarray(data)).to(self.torch_device, dtype)

    def reserve(self, nbytes: int) -> None:
        check(L.lib().wavo_reserve(self.ctx, nbytes), self.ctx)

    def set_q8_gemm(self, mode: int) -> int:
        """How Q8_0 layers' GEMMs read W (L.Q8_AUTO, L.Q8_DEQUANT, L.Q8_PROLOGUE); returns the
        previous mode."""
        return int(L.lib().wavo_set_q8_gemm(self.ctx, mode))

    def sync(self, timeout_ms: int = 60000) -> None:
        """Completion check (src/gpu/mod.rs:969-1003): device errors raise here."""
        check(L.lib().wavo_sync(self.ctx, timeout_ms), self.ctx)

    def pass_(self) -> "Pass":
        return Pass(self)

    # -- graphs ------------------------------------------------------------------------------
    def capture(self, record) -> "Graph":
        """Records `record(Pass)` into a CUDA graph on a side stream and returns it."""
        s = torch.cuda.Stream(self.torch_device)
        s.wait_stream(torch.cuda.current_stream(self.torch_device))
        self.use_stream(s)
        try:
            with torch.cuda.stream(s):
                check(L.lib().wavo_capture_begin(self.ctx), self.ctx)
                try:
                    record(Pass(self))
                finally:
                    g = ctypes.c_void_p()
                    status = L.lib().wavo_capture_end(self.ctx, ctypes.byref(g))
                check(status, self.ctx)
        finally:
            torch.cuda.current_stream(self.torch_device).wait_stream(s)
            self.use_stream(torch.cuda.current_stream(self.torch_device))
        return Graph(self, g)


class Graph:
    def __init__(self, gpu: Gpu, h: ctypes.c_void_p):
        self.gpu, self.h = gpu, h

    def launch(self) -> None:
        check(L.lib().wavo_graph_launch(self.gpu.ctx, self.h), self.gpu.ctx)

    def __del__(self):
        if getattr(self, "h", None) is not None and self.h.value:
            L.lib().wavo_graph_destroy(self.h)
            self.h = None


class Pass:
    """`Pass` (src/gpu/mod.rs:1293-1680): the attention path's ops, enqueued on the context."""

    def __init__(self, gpu: Gpu):
        self.gpu = gpu
        self.ctx = gpu.ctx

    def gemm(self, a: torch.Tensor, l: Linear, c: torch.Tensor, m: int, epilogue="bias",
             alpha: float = 1.0, lda: int = 0, ldc: int = 0) -> None:
        """`Pass::gemm` (src/gpu/mod.rs:1394-1425): c = epilogue(a·W^T + b) for m rows."""
        check(L.lib().wavo_gemm(self.ctx, _ptr(a), _dtype(a), lda, l.h, _ptr(c), _dtype(c), ldc, m,
                                EPILOGUES[epilogue], alpha), self.ctx)

    def gemv(self, a: torch.Tensor, l: Linear, c: torch.Tensor, epilogue="bias", offset: int = 0,
             alpha: float = 1.0) -> None:
        """`Pass::gemv` (src/gpu/mod.rs:1461-1467)."""
        check(L.lib().wavo_gemv(self.ctx, _ptr(a), l.h, _ptr(c), EPILOGUES[epilogue], alpha,
                                offset), self.ctx)

    def gemv_rows(self, a: torch.Tensor, l: Linear, c: torch.Tensor, rows: int, epilogue="bias",
                  alpha: float = 1.0, lda: int = 0, ldc: int = 0) -> None:
        check(L.lib().wavo_gemv_rows(self.ctx, _ptr(a), lda, l.h, _ptr(c), ldc, rows,
                                     EPILOGUES[epilogue], alpha), self.ctx)

    def attention(self, qk: torch.Tensor, v: torch.Tensor | None, pos: torch.Tensor | None,
                  o: torch.Tensor, t: int, heads: int, hd: int) -> None:
        """`Pass::attention` (src/gpu/mod.rs:1556-1605); the scores scratch `s` is not needed."""
        check(L.lib().wavo_attention(self.ctx, _ptr(qk), _ptr(v), _ptr(pos), _ptr(o), t, heads,
                                     hd, _dtype(qk)), self.ctx)

    def attention_varlen(self, qk, v, pos, o, rows: int, seg_start: torch.Tensor,
                         seg_len: torch.Tensor, max_len: int, heads: int, hd: int,
                         pos_t: int = 0) -> None:
        """Attention over independent segments in one launch (int32 device arrays)."""
        assert seg_start.dtype == torch.int32 and seg_len.dtype == torch.int32
        check(L.lib().wavo_attention_varlen(self.ctx, _ptr(qk), _ptr(v), _ptr(pos), _ptr(o), rows,
                                            _ptr(seg_start), _ptr(seg_len), seg_len.numel(),
                                            max_len, pos_t, heads, hd, _dtype(qk), _dtype(o)),
              self.ctx)

    def attention_rope_varlen(self, qkv, o, rows: int, seg_start: torch.Tensor,
                              seg_len: torch.Tensor, max_len: int, heads: int, hd: int,
                              table: torch.Tensor, rot: int, neox: bool, pos: int = 0) -> None:
        """Attention over segments of f16 [q | k | v] rows with rotary positions applied inside the
        kernel (row i of a segment at table row pos + i); the rows are left unrotated."""
        assert seg_start.dtype == torch.int32 and seg_len.dtype == torch.int32
        assert qkv.dtype == torch.float16 and table.dtype == torch.float32
        check(L.lib().wavo_attention_rope_varlen(
            self.ctx, _ptr(qkv), _ptr(o), rows, _ptr(seg_start), _ptr(seg_len), seg_len.numel(),
            max_len, heads, hd, _ptr(table), table.shape[0], pos, rot, int(neox), _dtype(o)),
            self.ctx)

    def layer_norm(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, y: torch.Tensor,
                   rows: int, cols: int, rope=None) -> None:
        """`Pass::layer_norm` (src/gpu/mod.rs:1431-1449): f32 x into y (f32 or f16); rope =
        (table, yr, head_dim[, positions]) also writes the rotary copy yr."""
        table = yr = positions = None
        hd = 0
        if rope is not None:
            table, yr, hd = rope[:3]
            positions = rope[3] if len(rope) > 3 else None
            assert yr.dtype == y.dtype
        check(L.lib().wavo_layer_norm(self.ctx, _ptr(x), _ptr(w), _ptr(b), _ptr(y), _dtype(y), rows,
                                      cols, _ptr(table), _ptr(positions), _ptr(yr), hd), self.ctx)

    def conv_glu(self, h: torch.Tensor, dw_w: torch.Tensor, dw_b: torch.Tensor, kernel: int,
                 n_w: torch.Tensor, n_b: torch.Tensor, layer_norm: bool, y: torch.Tensor, t: int,
                 ch: int, segs=None) -> None:
        """`Pass::conv_glu` (src/gpu/mod.rs:1538-1566); with segs (a Segments) over packed
        segments."""
        norm = L.CONV_LAYER_NORM if layer_norm else L.CONV_AFFINE
        if segs is None:
            check(L.lib().wavo_conv_glu(self.ctx, _ptr(h), _ptr(dw_w), _ptr(dw_b), kernel, _ptr(n_w),
                                        _ptr(n_b), norm, _ptr(y), _dtype(y), t, ch), self.ctx)
        else:
            check(L.lib().wavo_conv_glu_varlen(
                self.ctx, _ptr(h), _ptr(dw_w), _ptr(dw_b), kernel, _ptr(n_w), _ptr(n_b), norm,
                _ptr(y), _dtype(y), t, _ptr(segs.start_t), _ptr(segs.len_t), segs.len_t.numel(),
                segs.max_len, ch), self.ctx)

    def embed_rows(self, l: Linear, positions: torch.Tensor | None, tokens: torch.Tensor,
                   rows: int, pos: int, x: torch.Tensor, ldx: int = 0) -> None:
        """`Pass::embed` (src/gpu/mod.rs:1471-1484) for `rows` token ids (device int32)."""
        assert tokens.dtype == torch.int32
        check(L.lib().wavo_embed_rows(self.ctx, l.h, _ptr(positions), _ptr(tokens), rows, pos,
                                      _ptr(x), ldx), self.ctx)

    def pick(self, logits: torch.Tensor, rows: int, vocab: int, history: torch.Tensor,
             hist_len: torch.Tensor, suppress: torch.Tensor, n_suppress: int,
             begin_suppress: torch.Tensor, n_begin: int, eot: int, no_timestamps: int, begin: int,
             max_initial: int, tokens: torch.Tensor, logprobs: torch.Tensor | None = None) -> None:
        """The greedy pick with Whisper's suppression and timestamp rules (wavo_pick)."""
        check(L.lib().wavo_pick(self.ctx, _ptr(logits), logits.shape[-1], rows, vocab,
                                _ptr(history), _ptr(hist_len), history.shape[-1], _ptr(suppress),
                                n_suppress, _ptr(begin_suppress), n_begin, eot, no_timestamps,
                                begin, max_initial, _ptr(tokens), _ptr(logprobs)), self.ctx)

    def rope(self, table: torch.Tensor, qkv: torch.Tensor, rows: int, pos: int,
             shape: tuple[int, int, int], neox: bool, stride: int = 0) -> None:
        """`Pass::rope` (src/gpu/mod.rs:1630-1649): shape = [heads, hd, rot]."""
        heads, hd, rot = shape
        check(L.lib().wavo_rope(self.ctx, _ptr(table), _ptr(qkv), _dtype(qkv), stride, rows, pos,
                                heads, hd, rot, int(neox)), self.ctx)

    def rope_rows(self, table: torch.Tensor, qkv: torch.Tensor, rows: int,
                  positions: torch.Tensor, shape: tuple[int, int, int], neox: bool,
                  stride: int = 0) -> None:
        """`rope` with each row's table row given (int32 device array)."""
        heads, hd, rot = shape
        assert positions.dtype == torch.int32
        check(L.lib().wavo_rope_rows(self.ctx, _ptr(table), _ptr(qkv), _dtype(qkv), stride, rows,
                                     0, _ptr(positions), heads, hd, rot, int(neox)), self.ctx)

    def pack(self, x: torch.Tensor, src_stride: tuple[int, int], cache: torch.Tensor, rows: int,
             d: int, cols_col: tuple[int, int]) -> None:
        """`Pass::pack` (src/gpu/mod.rs:1507-1522)."""
        src, stride = src_stride
        cols, col = cols_col
        check(L.lib().wavo_pack(self.ctx, _ptr(x), src, stride, _ptr(cache), rows, d, cols, col),
              self.ctx)

    def pack_batch(self, x: torch.Tensor, src_stride: tuple[int, int], x_batch: int,
                   cache: torch.Tensor, cache_batch: int, rows: int, d: int,
                   cols_col: tuple[int, int], batch: int) -> None:
        """`pack` for `batch` segments: segment b's rows at x + b·x_batch floats, its cache at
        cache + b·cache_batch words."""
        src, stride = src_stride
        cols, col = cols_col
        check(L.lib().wavo_pack_batch(self.ctx, _ptr(x), src, stride, x_batch, _ptr(cache),
                                      cache_batch, rows, d, cols, col, batch), self.ctx)

    def attend(self, q: torch.Tensor, kv: torch.Tensor, part: torch.Tensor, o: torch.Tensor,
               n: int, cols: int, heads: int, hd: int) -> None:
        """`Pass::attend` (src/gpu/mod.rs:1485-1505)."""
        check(L.lib().wavo_attend(self.ctx, _ptr(q), _ptr(kv), _ptr(part), _ptr(o), n, cols, heads,
                                  hd), self.ctx)

    def attend_batch(self, q, q_stride: int, kv, kv_stride: int, part, o, o_stride: int, n: int,
                     cols: int, heads: int, hd: int, batch: int) -> None:
        check(L.lib().wavo_attend_batch(self.ctx, _ptr(q), q_stride, _ptr(kv), kv_stride,
                                        _ptr(part), _ptr(o), o_stride, n, cols, heads, hd, batch),
              self.ctx)


def partition_lpt(costs, parts: int) -> list[int]:
    """Longest-processing-time-first assignment of independent items to `parts` devices."""
    c = np.ascontiguousarray(costs, np.uint64)
    out = np.zeros(len(c), np.uint32)
    check(L.lib().wavo_partition_lpt(c.ctypes.data, len(c), parts, out.ctypes.data))
    return out.tolist()
