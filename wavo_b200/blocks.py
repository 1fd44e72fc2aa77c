"""The attention part of the reference's model blocks, over the `Pass` interface: what
src/conformer.rs (`Block::record`, 238-252) and src/transformer.rs (`Encoder::record` 122-131,
`Decoder::record_cross` 243-248, `Decoder::record_step` 254-290) record for attention, with the
layer inputs and the residual stream as the caller's buffers.

Every block runs over independent segments packed one after another (rows `seg_start[z] ..
+ seg_len[z]`); one segment of `rows` rows is the reference's case. Projections write f16
operands that the attention kernel loads directly; the attention writes f16 rows the output
projection reads; the output projection adds into the caller's f32 residual stream
(`Epilogue::Residual(1.0)`, as the reference).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from ._lib import GGML_BF16, GGML_F16, GGML_F32, GGML_Q8_0  # noqa: F401
from .gpu import Gpu, Linear, Pass, pos_rows


def rel_positions(d: int, first: int, rows: int) -> np.ndarray:
    """src/conformer.rs:141-153: the sinusoidal table of relative positions first, first - 1, …
    for `rows` rows of d, in f32: [2k] = sin(pos·d_k), [2k + 1] = cos(pos·d_k)."""
    c = np.float32(-math.log(10000.0)) / np.float32(d)
    div = np.exp(np.arange(0, d, 2, dtype=np.float32) * c).astype(np.float32)
    pos = (first - np.arange(rows)).astype(np.float32)[:, None]
    ang = (pos * div[None, :]).astype(np.float32)
    out = np.empty((rows, d), np.float32)
    out[:, 0::2] = np.sin(ang)
    out[:, 1::2] = np.cos(ang)
    return out


def rope_table(frames: int, hd: int, theta: float) -> np.ndarray:
    """src/gigaam/mod.rs:88-96: per position hd/2 cosines then hd/2 sines, angles in f64."""
    t = np.arange(frames, dtype=np.float64)[:, None]
    inv = theta ** (-2.0 * np.arange(hd // 2, dtype=np.float64) / hd)
    ang = t * inv[None, :]
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)


class Segments:
    """Independent segments packed one after another: device int32 starts and lengths."""

    def __init__(self, lengths, device):
        self.lengths = [int(n) for n in lengths]
        starts = np.concatenate([[0], np.cumsum(self.lengths)[:-1]]).astype(np.int32)
        self.starts = [int(s) for s in starts]
        self.rows = int(sum(self.lengths))
        self.max_len = max(self.lengths) if self.lengths else 0
        self.start_t = torch.tensor(starts, dtype=torch.int32, device=device)
        self.len_t = torch.tensor(self.lengths, dtype=torch.int32, device=device)
        # Each row's position inside its segment (the RoPE table row).
        pos = np.concatenate([np.arange(n, dtype=np.int32) for n in self.lengths]) \
            if self.lengths else np.zeros(0, np.int32)
        self.positions = torch.tensor(pos, dtype=torch.int32, device=device)


class RelPosAttention:
    """Parakeet's relative-position MHSA (src/conformer.rs:174-200, 238-252): one projection
    [q | k | v] whose bias [u | 0 | 0 | v] writes q a second time (the dual outputs), so that it
    produces [q+u | k | v | q+v]; linear_pos over the sinusoidal table; the attention with the
    Transformer-XL terms; the output projection added into the residual stream.

    The projected positions depend only on the position and the layer, so one table of
    pos_rows(t_pos) rows serves every segment of length <= t_pos (the reference projects a table
    of pos_rows(t) rows per segment, src/cpu/conformer.rs:181)."""

    def __init__(self, gpu: Gpu, ty: int, d: int, heads: int, wqkv: bytes, wpos: bytes,
                 wout: bytes, u: np.ndarray, v: np.ndarray, bias_qkv=None, bias_out=None):
        self.gpu, self.d, self.heads, self.hd = gpu, d, heads, d // heads
        bq = np.zeros(3 * d, np.float32) if bias_qkv is None else np.asarray(bias_qkv, np.float32)
        bias = np.concatenate([bq[:d] + np.asarray(u, np.float32).ravel(), bq[d:3 * d],
                               bq[:d] + np.asarray(v, np.float32).ravel()])
        self.qkv = gpu.linear(ty, 3 * d, d, wqkv, bias)
        self.pos = gpu.linear(ty, d, d, wpos, None)
        self.out = gpu.linear(ty, d, d, wout, bias_out)

    def scratch(self, rows: int, t_pos: int):
        dev = self.gpu.torch_device
        return {"qkv": torch.empty(rows, 4 * self.d, dtype=torch.float16, device=dev),
                "p": torch.empty(pos_rows(t_pos), self.d, dtype=torch.float16, device=dev),
                "o": torch.empty(rows, self.d, dtype=torch.float16, device=dev)}

    def record(self, p: Pass, y: torch.Tensor, x: torch.Tensor, segs: Segments,
               table: torch.Tensor, t_pos: int, s: dict, tick=None) -> None:
        """y: the layer input rows (LayerNorm output); x: the f32 residual stream; table: the
        sinusoids of positions t_pos + 15 down to -t_pos (pos_rows(t_pos) rows)."""
        rows = segs.rows
        tick = tick or (lambda name, fn: fn())
        tick("gemm_qkv", lambda: p.gemm(y, self.qkv, s["qkv"], rows, "bias"))
        tick("gemm_pos", lambda: p.gemm(table, self.pos, s["p"], pos_rows(t_pos), "bias"))
        tick("attention", lambda: p.attention_varlen(
            s["qkv"], None, s["p"], s["o"], rows, segs.start_t, segs.len_t, segs.max_len,
            self.heads, self.hd, t_pos))
        tick("gemm_out", lambda: p.gemm(s["o"], self.out, x, rows, "residual", 1.0))


class RotaryAttention:
    """Attention with rotary positions on q and k (BASELINE C3: GigaAM-shaped, RoPE on Q/K with
    NEOX pairs; the reference's ops::rope placement, src/cpu/transformer.rs:104-106) over
    [q | k | v] from one projection."""

    def __init__(self, gpu: Gpu, ty: int, d: int, heads: int, wqkv: bytes, wout: bytes,
                 bias_qkv=None, bias_out=None, theta: float = 10000.0, max_frames: int = 4096,
                 neox: bool = True, fuse_rope: bool = False):
        self.gpu, self.d, self.heads, self.hd = gpu, d, heads, d // heads
        self.neox = neox
        # Rotation inside the attention kernel (wavo_attention_rope_varlen) or as its own pass
        # before it (the default: faster at C3's shapes, 12.5 + 54.3 us against 72.9 us a layer).
        self.fuse_rope = fuse_rope
        self.qkv = gpu.linear(ty, 3 * d, d, wqkv, bias_qkv)
        self.out = gpu.linear(ty, d, d, wout, bias_out)
        self.table = gpu.upload(rope_table(max_frames, self.hd, theta))

    def scratch(self, rows: int):
        dev = self.gpu.torch_device
        return {"qkv": torch.empty(rows, 3 * self.d, dtype=torch.float16, device=dev),
                "o": torch.empty(rows, self.d, dtype=torch.float16, device=dev)}

    def fused(self) -> bool:
        """Whether the rotation runs inside the attention kernel (heads of 16, 32, 48, 64 or 128
        and a rotated half that is a multiple of 8), else as its own pass before it."""
        half = self.hd // 2 if self.neox else self.hd
        return self.fuse_rope and self.hd in (16, 32, 48, 64, 128) and half % 8 == 0

    def record(self, p: Pass, y: torch.Tensor, x: torch.Tensor, segs: Segments, s: dict) -> None:
        rows = segs.rows
        p.gemm(y, self.qkv, s["qkv"], rows, "bias")
        if self.fused():
            p.attention_rope_varlen(s["qkv"], s["o"], rows, segs.start_t, segs.len_t, segs.max_len,
                                    self.heads, self.hd, self.table, self.hd, self.neox)
        else:
            p.rope_rows(self.table, s["qkv"], rows, segs.positions,
                        (self.heads, self.hd, self.hd), self.neox)
            p.attention_varlen(s["qkv"], None, None, s["o"], rows, segs.start_t, segs.len_t,
                               segs.max_len, self.heads, self.hd)
        p.gemm(s["o"], self.out, x, rows, "residual", 1.0)


class EncoderAttention:
    """Whisper's encoder self-attention (src/transformer.rs:122-131): [q | k | v] with biases on
    q and v (none on k, src/transformer.rs:56), attention, output projection."""

    def __init__(self, gpu: Gpu, ty: int, d: int, heads: int, wqkv: bytes, wout: bytes,
                 bias_qkv=None, bias_out=None):
        self.gpu, self.d, self.heads, self.hd = gpu, d, heads, d // heads
        self.qkv = gpu.linear(ty, 3 * d, d, wqkv, bias_qkv)
        self.out = gpu.linear(ty, d, d, wout, bias_out)

    def scratch(self, rows: int):
        dev = self.gpu.torch_device
        return {"qkv": torch.empty(rows, 3 * self.d, dtype=torch.float16, device=dev),
                "o": torch.empty(rows, self.d, dtype=torch.float16, device=dev)}

    def record(self, p: Pass, y: torch.Tensor, x: torch.Tensor, rows: int, s: dict,
               segs: Segments | None = None) -> None:
        p.gemm(y, self.qkv, s["qkv"], rows, "bias")
        if segs is None:
            p.attention(s["qkv"], None, None, s["o"], rows, self.heads, self.hd)
        else:
            p.attention_varlen(s["qkv"], None, None, s["o"], rows, segs.start_t, segs.len_t,
                               segs.max_len, self.heads, self.hd)
        p.gemm(s["o"], self.out, x, rows, "residual", 1.0)


class DecoderAttention:
    """Whisper's decoder attention for a batch of segments (src/transformer.rs:243-290): the
    cross-attention K/V of every segment packed once into F16 caches (`record_cross`), then per
    token: q|k|v of the token, k and v packed into the self cache at the token's position, the
    self attention over positions 0..pos, its output projection into the residual stream; the
    cross query, the cross attention over the encoder frames, its output projection.

    Caches are the reference's layout (src/gpu/mod.rs:1507-1522), one per segment, `cols`
    positions each; the batch of segments runs in one launch per op."""

    def __init__(self, gpu: Gpu, ty: int, d: int, heads: int, context: int, frames: int,
                 batch: int, w: dict, b: dict):
        self.gpu, self.d, self.heads, self.hd = gpu, d, heads, d // heads
        self.context, self.frames, self.batch = context, frames, batch
        self.qkv = gpu.linear(ty, 3 * d, d, w["qkv"], b.get("qkv"))
        self.self_out = gpu.linear(ty, d, d, w["self_out"], b.get("self_out"))
        self.cross_q = gpu.linear(ty, d, d, w["cross_q"], b.get("cross_q"))
        self.cross_kv = gpu.linear(ty, 2 * d, d, w["cross_kv"], b.get("cross_kv"))
        self.cross_out = gpu.linear(ty, d, d, w["cross_out"], b.get("cross_out"))
        dev = gpu.torch_device
        # F16 caches as 32-bit words: own [batch][d][context/…], cross [batch][d · frames].
        self.own = torch.zeros(batch, d * context, dtype=torch.int32, device=dev)
        self.cross = torch.zeros(batch, d * frames, dtype=torch.int32, device=dev)
        self.qkv_buf = torch.empty(batch, 3 * d, dtype=torch.float32, device=dev)
        self.q_buf = torch.empty(batch, d, dtype=torch.float32, device=dev)
        self.att = torch.empty(batch, d, dtype=torch.float32, device=dev)
        from .gpu import attend_len
        self.part = torch.empty(batch * attend_len(max(frames, context), heads, self.hd),
                                dtype=torch.float32, device=dev)

    def record_cross(self, p: Pass, enc: torch.Tensor, chunk: int = 8) -> None:
        """enc: [batch][frames][d] encoder outputs (f32); chunk segments per projection."""
        d, t = self.d, self.frames
        kv = torch.empty(chunk * t, 2 * d, dtype=torch.float32, device=self.gpu.torch_device)
        for b0 in range(0, self.batch, chunk):
            nb = min(chunk, self.batch - b0)
            p.gemm(enc[b0:b0 + nb].reshape(nb * t, d), self.cross_kv, kv, nb * t, "bias")
            p.pack_batch(kv, (0, 2 * d), t * 2 * d, self.cross[b0], d * t, t, d, (t, 0), nb)

    def record_step(self, p: Pass, y_self: torch.Tensor, y_cross: torch.Tensor, x: torch.Tensor,
                    pos: int) -> None:
        """One token per segment at position `pos`: y_self / y_cross are the LayerNorm outputs
        feeding the self and cross projections ([batch][d]); x the residual stream."""
        self.record_self(p, y_self, x, pos)
        self.record_cross_attend(p, y_cross, x)

    def record_self(self, p: Pass, y_self: torch.Tensor, x: torch.Tensor, pos: int) -> None:
        """The self-attention half of a step: q|k|v, k and v into the cache at `pos`, attention
        over 0..pos, the output projection added into x."""
        d, B = self.d, self.batch
        p.gemv_rows(y_self, self.qkv, self.qkv_buf, B, "bias", ldc=3 * d)
        p.pack_batch(self.qkv_buf, (d, 0), 3 * d, self.own, d * self.context, 1, d,
                     (self.context, pos), B)
        p.attend_batch(self.qkv_buf, 3 * d, self.own, d * self.context, self.part, self.att, d,
                       pos + 1, self.context, self.heads, self.hd, B)
        p.gemv_rows(self.att, self.self_out, x, B, "residual", 1.0, ldc=d)

    def record_cross_attend(self, p: Pass, y_cross: torch.Tensor, x: torch.Tensor) -> None:
        """The cross-attention half: the query, attention over the encoder frames, the output
        projection added into x."""
        d, B = self.d, self.batch
        p.gemv_rows(y_cross, self.cross_q, self.q_buf, B, "bias", ldc=d)
        p.attend_batch(self.q_buf, d, self.cross, d * self.frames, self.part, self.att, d,
                       self.frames, self.frames, self.heads, self.hd, B)
        p.gemv_rows(self.att, self.cross_out, x, B, "residual", 1.0, ldc=d)


class ConformerBlock:
    """A whole FastConformer block with relative-position attention (Parakeet; the reference's
    `Block::record`, src/conformer.rs:232-265, CPU `Block::run`, src/cpu/conformer.rs:159-199), over
    packed segments: half-step FFN, MHSA, conv module, half-step FFN, then norm_out. `norms` maps
    "ff1", "attn", "conv", "ff2", "out" to (weight, bias) f32 arrays of d; the conv module's norm is
    a LayerNorm (`conv_norm` (weight, bias), conv_ln=True) or a folded batch norm (per-channel
    scale, shift). Weights are GGUF tensor bytes of `ty`: ff*_1 [f][d], ff*_2 [d][f], pw1 [2d][d],
    pw2 [d][d]; dw [d][kernel] f32 (as the GGUF tensor stores it) with bias dw_b.

    Every GEMM input is f16 (the reference GPU GEMM rounds a to f16); the residual stream x is
    f32; the block output (norm_out) goes to an f32 buffer, as the reference's."""

    def __init__(self, gpu: Gpu, ty: int, d: int, f: int, heads: int, kernel: int, w: dict,
                 norms: dict, conv_ln: bool):
        self.gpu, self.d, self.f, self.heads, self.kernel, self.conv_ln = gpu, d, f, heads, kernel, conv_ln
        up = lambda a: gpu.upload(np.asarray(a, np.float32))  # noqa: E731
        self.norms = {k: (up(wb[0]), up(wb[1])) for k, wb in norms.items()}
        self.ff1 = (gpu.linear(ty, f, d, w["ff1_1"], w.get("ff1_1_b")),
                    gpu.linear(ty, d, f, w["ff1_2"], w.get("ff1_2_b")))
        self.ff2 = (gpu.linear(ty, f, d, w["ff2_1"], w.get("ff2_1_b")),
                    gpu.linear(ty, d, f, w["ff2_2"], w.get("ff2_2_b")))
        self.attn = RelPosAttention(gpu, ty, d, heads, w["qkv"], w["pos"], w["out"], w["u"], w["v"],
                                    w.get("qkv_b"), w.get("out_b"))
        self.pw1 = gpu.linear(ty, 2 * d, d, w["pw1"], w.get("pw1_b"))
        self.pw2 = gpu.linear(ty, d, d, w["pw2"], w.get("pw2_b"))
        self.dw = up(w["dw"])
        self.dw_b = up(w.get("dw_b", np.zeros(d, np.float32)))

    def scratch(self, rows: int, t_pos: int):
        dev = self.gpu.torch_device
        s = self.attn.scratch(rows, t_pos)
        s["y"] = torch.empty(rows, self.d, dtype=torch.float16, device=dev)
        s["h"] = torch.empty(rows, self.f, dtype=torch.float16, device=dev)
        s["pw"] = torch.empty(rows, 2 * self.d, dtype=torch.float32, device=dev)
        return s

    def record(self, p: Pass, x: torch.Tensor, out: torch.Tensor, segs: Segments,
               table: torch.Tensor, t_pos: int, s: dict, tick=None) -> None:
        """x: the f32 block input [rows][d] (updated in place as the residual stream); out: the
        f32 block output norm_out(x); table: the f16 sinusoid rows (pos_rows(t_pos)). tick(name,
        fn) runs each launch (a timer may wrap it)."""
        rows, d = segs.rows, self.d
        y, h = s["y"], s["h"]
        n = self.norms
        tick = tick or (lambda name, fn: fn())
        tick("layer_norm", lambda: p.layer_norm(x, *n["ff1"], y, rows, d))
        tick("gemm_ff1", lambda: p.gemm(y, self.ff1[0], h, rows, "silu"))
        tick("gemm_ff2", lambda: p.gemm(h, self.ff1[1], x, rows, "residual", 0.5))
        tick("layer_norm", lambda: p.layer_norm(x, *n["attn"], y, rows, d))
        self.attn.record(p, y, x, segs, table, t_pos, s, tick)
        tick("layer_norm", lambda: p.layer_norm(x, *n["conv"], y, rows, d))
        tick("gemm_pw1", lambda: p.gemm(y, self.pw1, s["pw"], rows, "bias"))
        tick("conv_glu", lambda: p.conv_glu(s["pw"], self.dw, self.dw_b, self.kernel,
                                            *n["conv_norm"], self.conv_ln, y, rows, d, segs))
        tick("gemm_pw2", lambda: p.gemm(y, self.pw2, x, rows, "residual", 1.0))
        tick("layer_norm", lambda: p.layer_norm(x, *n["ff2"], y, rows, d))
        tick("gemm_ff1", lambda: p.gemm(y, self.ff2[0], h, rows, "silu"))
        tick("gemm_ff2", lambda: p.gemm(h, self.ff2[1], x, rows, "residual", 0.5))
        tick("layer_norm", lambda: p.layer_norm(x, *n["out"], out, rows, d))

    def launches(self) -> int:
        """Kernels the block launches: 5 LayerNorms, 9 GEMMs, the attention and the conv module
        (one kernel with the affine norm, two with the LayerNorm)."""
        return 15 + (2 if self.conv_ln else 1)


class WhisperDecoder:
    """The whole Whisper decoder step for a batch of segments, on the device (the reference's
    `Decoder::record_step`, src/transformer.rs:254-290, with the token picked by `wavo_pick` instead
    of the CPU's search, src/whisper/search.rs:35-123): embed the batch's tokens at the step's
    position, per layer LayerNorm -> self attention -> LayerNorm -> cross attention -> LayerNorm ->
    FFN (GELU), the final LayerNorm, the logits through the tied embedding, the greedy pick with
    the suppression and timestamp rules. The tokens, the generated histories and the logits stay in
    device memory, so a whole decode runs without a host round trip per token (and can be one CUDA
    graph).

    w: "embed" [vocab][d] GGUF bytes of `ty`, "positions" [context][d] f32, "norm" (weight, bias),
    "layers": one dict per layer with the DecoderAttention weights and biases ("qkv", "self_out",
    "cross_q", "cross_kv", "cross_out"; biases under "b"), "fc1" [d_ff][d], "fc2" [d][d_ff] (biases
    "fc1_b", "fc2_b") and the norms "norm_self", "norm_cross", "norm_ffn" as (weight, bias).
    ids: "eot", "no_timestamps", "begin" (the first timestamp), "suppress", "begin_suppress"."""

    def __init__(self, gpu: Gpu, ty: int, d: int, heads: int, d_ff: int, vocab: int,
                 context: int, frames: int, batch: int, w: dict, ids: dict, max_initial: int = 50):
        self.gpu, self.d, self.heads, self.d_ff, self.vocab = gpu, d, heads, d_ff, vocab
        self.context, self.frames, self.batch, self.ids = context, frames, batch, ids
        self.max_initial = max_initial
        dev = gpu.torch_device
        up = lambda a: gpu.upload(np.asarray(a, np.float32))  # noqa: E731
        self.embed = gpu.linear(ty, vocab, d, w["embed"], None)
        self.positions = up(w["positions"])
        self.norm = tuple(up(v) for v in w["norm"])
        self.layers = []
        for lw in w["layers"]:
            att = DecoderAttention(gpu, ty, d, heads, context, frames, batch, lw, lw.get("b", {}))
            self.layers.append({
                "att": att,
                "fc1": gpu.linear(ty, d_ff, d, lw["fc1"], lw.get("fc1_b")),
                "fc2": gpu.linear(ty, d, d_ff, lw["fc2"], lw.get("fc2_b")),
                **{k: tuple(up(v) for v in lw[k]) for k in ("norm_self", "norm_cross", "norm_ffn")},
            })
        self.x = torch.zeros(batch, d, dtype=torch.float32, device=dev)
        self.y = torch.zeros(batch, d, dtype=torch.float32, device=dev)
        self.h = torch.zeros(batch, d_ff, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(batch, self.embed.width(), dtype=torch.float32, device=dev)
        i32 = lambda a: torch.tensor(np.asarray(a, np.int32), dtype=torch.int32, device=dev)  # noqa: E731
        self.suppress = i32(ids.get("suppress", []) or [0])
        self.n_suppress = len(ids.get("suppress", []))
        self.begin_suppress = i32(ids.get("begin_suppress", []) or [0])
        self.n_begin = len(ids.get("begin_suppress", []))
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.history = torch.zeros(batch, context, dtype=torch.int32, device=dev)
        self.hist_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.logprobs = torch.zeros(batch, dtype=torch.float32, device=dev)

    def start(self, last_prompt_tokens) -> None:
        """A new window: each row's last prompt token, empty histories."""
        self.tokens.copy_(torch.as_tensor(np.asarray(last_prompt_tokens, np.int32)))
        self.hist_len.zero_()

    def record_cross(self, p: Pass, enc: torch.Tensor) -> None:
        """The cross-attention caches of every layer from the encoder output [batch][frames][d]."""
        for lay in self.layers:
            lay["att"].record_cross(p, enc)

    # Kernels a step launches: the embedding, per layer 3 LayerNorms + the self attention's 5
    # (q|k|v, pack, attend, combine, output) + the cross attention's 4 + the FFN's 2, then the
    # final LayerNorm, the logits and the pick.
    def launches_per_step(self) -> int:
        return 1 + 14 * len(self.layers) + 3

    def record_step(self, p: Pass, pos: int, tick=None) -> None:
        """The batch's current tokens at position `pos` through the decoder; the picked tokens
        replace them (and are appended to the histories). tick(name, fn) runs each group of
        launches (a timer may wrap it)."""
        d, B = self.d, self.batch
        tick = tick or (lambda name, fn: fn())
        tick("embed", lambda: p.embed_rows(self.embed, self.positions, self.tokens, B, pos, self.x))
        for lay in self.layers:
            tick("layer_norm", lambda: p.layer_norm(self.x, *lay["norm_self"], self.y, B, d))
            tick("self_attention", lambda: lay["att"].record_self(p, self.y, self.x, pos))
            tick("layer_norm", lambda: p.layer_norm(self.x, *lay["norm_cross"], self.y, B, d))
            tick("cross_attention", lambda: lay["att"].record_cross_attend(p, self.y, self.x))
            tick("layer_norm", lambda: p.layer_norm(self.x, *lay["norm_ffn"], self.y, B, d))

            def ffn():
                p.gemv_rows(self.y, lay["fc1"], self.h, B, "gelu", ldc=self.d_ff)
                p.gemv_rows(self.h, lay["fc2"], self.x, B, "residual", 1.0, ldc=d)
            tick("ffn", ffn)
        tick("layer_norm", lambda: p.layer_norm(self.x, *self.norm, self.y, B, d))
        tick("logits", lambda: p.gemv_rows(self.y, self.embed, self.logits, B, "bias",
                                           ldc=self.embed.width()))
        ids = self.ids
        tick("pick", lambda: p.pick(
            self.logits, B, self.vocab, self.history, self.hist_len, self.suppress,
            self.n_suppress, self.begin_suppress, self.n_begin, ids["eot"], ids["no_timestamps"],
            ids["begin"], self.max_initial, self.tokens, self.logprobs))
