"""The model-family attention blocks (wavo_b200.blocks) against the CPU oracle's wiring of the same
layers (src/cpu/conformer.rs:159-186, src/cpu/transformer.rs:94-116, 192-265), within the BASELINE
tolerance (max-abs 2e-3, rel-L2 1e-3), over packed independent segments."""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def check(got, want, max_abs=2e-3, rel_l2=1e-3):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = np.abs(got - want)
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert err.max() <= max_abs and rel <= rel_l2, f"max-abs {err.max():.3g}, rel-L2 {rel:.3g}"


@pytest.fixture(scope="module")
def gpu():
    from wavo_b200.gpu import Gpu
    g = Gpu(0)
    yield g
    g.sync()
    g.close()


def test_rope_rows_restart_per_segment(gpu):
    # Segments packed one after another rotate from their own position 0, as each alone.
    from wavo_b200.blocks import Segments, rope_table
    heads, hd = 3, 48
    lens = [5, 17, 1, 9]
    segs = Segments(lens, "cuda")
    x = O.random(segs.rows * 3 * heads * hd, 41)
    table = rope_table(32, hd, 10000.0)
    want = x.copy().reshape(segs.rows, -1)
    for s, n in zip(segs.starts, lens):
        blk = np.ascontiguousarray(want[s:s + n])
        O.rope(blk, np.ascontiguousarray(table[:n]), n, heads, hd, hd, True)
        want[s:s + n] = blk
    xb = gpu.upload(x)
    gpu.pass_().rope_rows(gpu.upload(table), xb, segs.rows, segs.positions, (heads, hd, hd), True)
    gpu.sync()
    check(xb.cpu().numpy(), want, 2e-6, 1e-6)


def test_bf16_weights(gpu):
    from wavo_b200 import GGML_BF16
    n, k, m = 96, 64, 40
    w = (O.random(n * k, 3) * 0.5).astype(np.float32)
    wb = (w.view(np.uint32) >> 16).astype(np.uint16)
    wf = (wb.astype(np.uint32) << 16).view(np.float32).reshape(n, k)
    lin = gpu.linear(GGML_BF16, n, k, wb.tobytes(), None)
    a = O.random(m * k, 4)
    c = torch.zeros(m, n, device="cuda")
    gpu.pass_().gemm(gpu.upload(a), lin, c, m, "bias")
    gpu.sync()
    want = O.f16_round(a).reshape(m, k).astype(np.float64) @ O.f16_round(wf).T.astype(np.float64)
    check(c.cpu().numpy(), want, 1e-4, 1e-5)


def test_pack_batch_equals_per_segment_pack(gpu):
    d, cols, B = 6, 7, 3
    x = O.random(B * 2 * d, 9)
    out = torch.zeros(B, d * cols, dtype=torch.int32, device="cuda")
    gpu.pass_().pack_batch(gpu.upload(x), (0, 0), 2 * d, out, d * cols, 1, d, (cols, 2), B)
    want = torch.zeros(B, d * cols, dtype=torch.int32, device="cuda")
    for b in range(B):
        gpu.pass_().pack(gpu.upload(x[b * 2 * d:(b + 1) * 2 * d]), (0, 0), want[b], 1, d, (cols, 2))
    gpu.sync()
    assert torch.equal(out, want)


def oracle_linear_gemm(ty, rows, k, data, bias, a, m, c=None, epi="bias"):
    O.set_vnni(0)  # the GPU GEMM's rounding: a and W to f16
    try:
        return O.Linear(ty, rows, k, data, bias).gemm(np.ascontiguousarray(a, np.float32).ravel(),
                                                      m, c, epi, 1.0)
    finally:
        O.set_vnni(-1)


@pytest.mark.parametrize("fuse", [False, True])
def test_rotary_block(gpu, fuse):
    from wavo_b200 import GGML_F16
    from wavo_b200.blocks import RotaryAttention, Segments, rope_table
    d, heads = 96, 2
    hd = d // heads
    lens = [37, 70, 129]
    rng = np.random.default_rng(2)
    wq = (rng.standard_normal((3 * d, d)) * 0.05).astype(np.float16)
    wo = (rng.standard_normal((d, d)) * 0.05).astype(np.float16)
    bq = (rng.standard_normal(3 * d) * 0.05).astype(np.float32)
    blk = RotaryAttention(gpu, GGML_F16, d, heads, wq.tobytes(), wo.tobytes(), bq, None,
                          theta=10000.0, max_frames=256, fuse_rope=fuse)
    assert blk.fused() == fuse
    segs = Segments(lens, "cuda")
    y = rng.standard_normal((segs.rows, d)).astype(np.float32)
    x = torch.ones(segs.rows, d, device="cuda")
    s = blk.scratch(segs.rows)
    blk.record(gpu.pass_(), gpu.upload(y), x, segs, s)
    gpu.sync()
    table = rope_table(256, hd, 10000.0)
    want = np.ones((segs.rows, d), np.float32)
    for st, n in zip(segs.starts, lens):
        qkv = oracle_linear_gemm(O.TY_F16, 3 * d, d, wq.tobytes(), bq, y[st:st + n], n)
        qkv = O.f16_round(qkv)  # the projection's f16 output
        O.rope(qkv, np.ascontiguousarray(table[:n]), n, heads, hd, hd, True)
        qkv = O.f16_round(qkv)  # rotated in place in f16
        o = O.attention(qkv, 3 * d, np.ascontiguousarray(qkv[2 * d:]), 3 * d, n, heads, d)
        w_ = np.ones(n * d, np.float32)
        oracle_linear_gemm(O.TY_F16, d, d, wo.tobytes(), None, o, n, w_, "residual")
        want[st:st + n] = w_.reshape(n, d)
    check(x.cpu().numpy(), want)


def test_relpos_block_q8(gpu):
    # C5-shaped (Q8_0, heads of 128) over packed segments with one shared position table.
    from wavo_b200 import GGML_Q8_0
    from wavo_b200.blocks import RelPosAttention, Segments, rel_positions
    d, heads = 256, 2
    lens = [120, 37, 300]
    rng = np.random.default_rng(4)
    wq = (rng.standard_normal((3 * d, d)) * 0.03).astype(np.float32)
    wp = (rng.standard_normal((d, d)) * 0.03).astype(np.float32)
    wo = (rng.standard_normal((d, d)) * 0.03).astype(np.float32)
    u = (rng.standard_normal(d) * 0.02).astype(np.float32)
    v = (rng.standard_normal(d) * 0.02).astype(np.float32)
    dq, dp, do_ = O.q8_0_bytes(wq), O.q8_0_bytes(wp), O.q8_0_bytes(wo)
    blk = RelPosAttention(gpu, GGML_Q8_0, d, heads, dq, dp, do_, u, v)
    segs = Segments(lens, "cuda")
    t_pos = max(lens)
    table = rel_positions(d, t_pos + 15, 2 * t_pos + 15)
    y = rng.standard_normal((segs.rows, d)).astype(np.float32)
    x = torch.zeros(segs.rows, d, device="cuda")
    s = blk.scratch(segs.rows, t_pos)
    blk.record(gpu.pass_(), gpu.upload(y), x, segs, gpu.upload(table), t_pos, s)
    gpu.sync()
    want = np.zeros((segs.rows, d), np.float32)
    for st, n in zip(segs.starts, lens):
        qkv = oracle_linear_gemm(O.TY_Q8_0, 3 * d, d, dq, None, y[st:st + n], n).reshape(n, 3 * d)
        q = qkv[:, :d]
        quv = O.f16_round(np.concatenate([q + u, qkv[:, d:], q + v], axis=1))
        tab = O.rel_positions(d, n + 15, O.pos_rows(n))
        pos = O.f16_round(oracle_linear_gemm(O.TY_Q8_0, d, d, dp, None, tab, O.pos_rows(n)))
        # The GPU reads [q+u | k | v | q+v] and the positions in f16; the oracle's f32 attention
        # on the same values.
        o = rel_attention_ref(quv.reshape(n, 4 * d), pos.reshape(-1, d), n, heads, d // heads)
        w_ = np.zeros(n * d, np.float32)
        oracle_linear_gemm(O.TY_Q8_0, d, d, do_, None, o.astype(np.float32), n, w_, "residual")
        want[st:st + n] = w_.reshape(n, d)
    check(x.cpu().numpy(), want)


def rel_attention_ref(quv, pos, t, heads, hd):
    d = heads * hd
    i = np.arange(t)[:, None]
    j = np.arange(t)[None, :]
    out = np.zeros((t, d))
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        qu, k, v, qv = (quv[:, s * d:(s + 1) * d][:, sl].astype(np.float64) for s in range(4))
        bd = np.take_along_axis(qv @ pos[:, sl].astype(np.float64).T, j + t + 15 - i, axis=1)
        s_ = (qu @ k.T + bd) / np.sqrt(hd)
        e = np.exp(s_ - s_.max(axis=1, keepdims=True))
        out[:, sl] = (e / e.sum(axis=1, keepdims=True)) @ v
    return out


def test_decoder_steps(gpu):
    # A batch of 3 segments through record_cross and 5 token steps, against the oracle's
    # Decoder::cache / Decoder::step attention path (gemv in f32, f16 caches, f16-rounded q).
    from wavo_b200 import GGML_F16
    from wavo_b200.blocks import DecoderAttention
    d, heads, context, frames, B = 128, 2, 16, 37, 3
    hd = d // heads
    rng = np.random.default_rng(6)
    names = {"qkv": 3 * d, "self_out": d, "cross_q": d, "cross_kv": 2 * d, "cross_out": d}
    w = {k: (rng.standard_normal((r, d)) * 0.05).astype(np.float16) for k, r in names.items()}
    b = {k: (rng.standard_normal(r) * 0.05).astype(np.float32) for k, r in names.items()}
    dec = DecoderAttention(gpu, GGML_F16, d, heads, context, frames, B,
                           {k: v.tobytes() for k, v in w.items()}, b)
    enc = rng.standard_normal((B, frames, d)).astype(np.float32)
    p = gpu.pass_()
    dec.record_cross(p, gpu.upload(enc).reshape(B, frames, d), chunk=2)
    x = torch.zeros(B, d, device="cuda")
    ys = [rng.standard_normal((2, B, d)).astype(np.float32) for _ in range(5)]
    for pos, y in enumerate(ys):
        yb = gpu.upload(y).reshape(2, B, d)
        dec.record_step(p, yb[0], yb[1], x, pos)
    gpu.sync()
    lin = {k: O.Linear(O.TY_F16, names[k], d, w[k].tobytes(), b[k]) for k in names}
    want = np.zeros((B, d), np.float32)
    for s in range(B):
        kv = lin["cross_kv"].gemm(np.ascontiguousarray(enc[s].ravel()), frames)
        cross = np.zeros(frames * 2 * d, np.float32)
        O.pack_cache(kv, frames, d, hd, cross, frames, 0)
        own = np.zeros(context * 2 * d, np.float32)
        xs = np.zeros(d, np.float32)
        for pos, y in enumerate(ys):
            qkv = lin["qkv"].gemv(np.ascontiguousarray(y[0, s]))
            O.pack_cache(np.ascontiguousarray(qkv[d:]), 1, d, hd, own, context, pos)
            att = O.attend(np.ascontiguousarray(qkv[:d]), own, context, pos + 1, heads, hd)
            lin["self_out"].gemv(att, xs, "residual", 1.0)
            q = lin["cross_q"].gemv(np.ascontiguousarray(y[1, s]))
            att = O.attend(q, cross, frames, frames, heads, hd)
            lin["cross_out"].gemv(att, xs, "residual", 1.0)
        want[s] = xs
    check(x.cpu().numpy(), want)
