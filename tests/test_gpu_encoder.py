"""The rest of the encoder block around the attention path, through the C ABI: LayerNorm (with the
rotary copy) and the conv module (Pass::layer_norm, Pass::conv_glu: src/gpu/mod.rs:1431-1449,
1538-1566), restating the reference's own GPU tests (src/gpu/mod.rs:1947-1973 layer_norm_and_rope,
2131-2160 conv_glu: the xorshift inputs, the naive references, 2e-5 · max|want|) and checking against
the CPU oracle (src/cpu/ops.rs:65-110, 133-182); then a whole Parakeet-shaped FastConformer block
over packed segments against the oracle's CPU block (src/cpu/conformer.rs:159-199) at the BASELINE
tolerance (max-abs 2e-3, relative-L2 1e-3).
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    from wavo_b200.gpu import Gpu
    g = Gpu(0)
    yield g
    g.sync()
    g.close()


def assert_close(got, want, tolerance=2e-5):
    """src/gpu/mod.rs:1741-1751: |got - want| <= tolerance · max(1, max|want|)."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    scale = max(1.0, float(np.abs(want).max()))
    err = np.abs(got - want)
    assert err.max() <= tolerance * scale, f"[{int(err.argmax())}] err {err.max():.3g}"


def check(got, want, max_abs=2e-3, rel_l2=1e-3):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = np.abs(got - want)
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert err.max() <= max_abs and rel <= rel_l2, f"max-abs {err.max():.3g}, rel-L2 {rel:.3g}"


def naive_layer_norm(x, g, b):
    """src/gpu/mod.rs:1753-1763."""
    x = x.reshape(-1, g.size).astype(np.float64)
    mean = x.mean(axis=1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=1, keepdims=True)
    return (x - mean) / np.sqrt(var + 1e-5) * g + b


def silu(x):
    return x / (1.0 + np.exp(-x))


@pytest.mark.parametrize("f16", [False, True])
def test_layer_norm_and_rope(gpu, f16):
    # src/gpu/mod.rs:1947-1973: rows 37, cols 192, heads of 48, table rows random(rows·hd, 8).
    rows, cols, hd = 37, 192, 48
    x, g, b = O.random(rows * cols, 5), O.random(cols, 6), O.random(cols, 7)
    rope = O.random(rows * hd, 8)
    y = naive_layer_norm(x, g, b).ravel()
    half = hd // 2
    idx = np.arange(rows * cols)
    t, dd = idx // cols, idx % hd
    cos = rope[t * hd + dd % half]
    sin = rope[t * hd + half + dd % half]
    partner = np.where(dd < half, idx + half, idx - half)
    yr = np.where(dd < half, y * cos - y[partner] * sin, y * cos + y[partner] * sin)
    dt = torch.float16 if f16 else torch.float32
    yb = torch.zeros(rows, cols, dtype=dt, device="cuda")
    yrb = torch.zeros(rows, cols, dtype=dt, device="cuda")
    p = gpu.pass_()
    p.layer_norm(gpu.upload(x), gpu.upload(g), gpu.upload(b), yb, rows, cols,
                 (gpu.upload(rope), yrb, hd))
    gpu.sync()
    tol = 1e-3 if f16 else 2e-5  # f16 outputs: one f16 rounding of values up to max|want|
    assert_close(yb.float().cpu().numpy(), y, tol)
    assert_close(yrb.float().cpu().numpy(), yr, tol)
    # The oracle (the reference's CPU layer_norm with its rope branch) agrees as well.
    oy, oyr = O.layer_norm(x, g, b, rows, cols, rope, hd)
    assert_close(oy, y)
    assert_close(oyr, yr)


def test_layer_norm_positions_and_width(gpu):
    # Packed segments: each row's rotary table row is its position inside its segment.
    rows, cols, hd = 300, 1024, 128
    rng = np.random.default_rng(0)
    x = rng.standard_normal(rows * cols).astype(np.float32) * 3 + 1
    g, b = rng.standard_normal(cols).astype(np.float32), rng.standard_normal(cols).astype(np.float32)
    pos = np.concatenate([np.arange(100), np.arange(200)]).astype(np.int32)
    table = O.rope_table(200, hd, 10000.0).reshape(200, hd)
    y = torch.zeros(rows, cols, device="cuda")
    yr = torch.zeros(rows, cols, device="cuda")
    gpu.pass_().layer_norm(gpu.upload(x), gpu.upload(g), gpu.upload(b), y, rows, cols,
                           (gpu.upload(table), yr, hd, torch.from_numpy(pos).cuda()))
    gpu.sync()
    oy, oyr = O.layer_norm(x, g, b, rows, cols, np.ascontiguousarray(table[pos]), hd)
    assert_close(y.cpu().numpy(), oy)
    assert_close(yr.cpu().numpy(), oyr)


def test_conv_glu(gpu):
    # src/gpu/mod.rs:2131-2160: t 37, ch 192; kernel 5 with LayerNorm, 9 with the affine norm.
    t, ch = 37, 192
    h = O.random(t * 2 * ch, 10)
    g, b = O.random(ch, 13), O.random(ch, 14)
    hh = h.reshape(t, 2 * ch).astype(np.float64)
    glu = hh[:, :ch] / (1.0 + np.exp(-hh[:, ch:]))
    for kernel, ln in [(5, True), (9, False)]:
        w, wb = O.random(ch * kernel, 11), O.random(ch, 12)
        pad = kernel // 2
        dw = np.tile(wb.astype(np.float64), (t, 1))
        wk = w.reshape(ch, kernel).astype(np.float64)
        for r in range(t):
            for k in range(kernel):
                src = r + k - pad
                if 0 <= src < t:
                    dw[r] += wk[:, k] * glu[src]
        want = naive_layer_norm(dw, g, b) if ln else dw * g + b
        want = silu(want)
        y = torch.zeros(t, ch, device="cuda")
        hb = gpu.upload(h)
        gpu.pass_().conv_glu(hb, gpu.upload(w), gpu.upload(wb), kernel, gpu.upload(g),
                             gpu.upload(b), ln, y, t, ch)
        gpu.sync()
        assert_close(y.cpu().numpy(), want)
        assert torch.equal(hb.cpu(), torch.from_numpy(h))  # h is left as it is
        # The oracle's CPU conv_glu (taps transposed to [kernel][ch], as src/cpu/conformer.rs:126).
        oy = O.conv_glu(h.copy(), np.ascontiguousarray(w.reshape(ch, kernel).T), wb, g, b, ln, t,
                        ch, kernel)
        assert_close(oy, want)


@pytest.mark.parametrize("kernel,ln", [(9, True), (31, False), (7, True)])
def test_conv_glu_segments(gpu, kernel, ln):
    # Packed segments: the depthwise conv stops at each segment's ends.
    from wavo_b200.blocks import Segments
    ch, lens = 256, [37, 70, 129, 1]
    rng = np.random.default_rng(kernel)
    segs = Segments(lens, "cuda")
    h = rng.standard_normal(segs.rows * 2 * ch).astype(np.float32)
    w = (rng.standard_normal(ch * kernel) * 0.3).astype(np.float32)
    wb, g, b = (rng.standard_normal(ch).astype(np.float32) for _ in range(3))
    y = torch.zeros(segs.rows, ch, device="cuda")
    gpu.pass_().conv_glu(gpu.upload(h), gpu.upload(w), gpu.upload(wb), kernel, gpu.upload(g),
                         gpu.upload(b), ln, y, segs.rows, ch, segs)
    gpu.sync()
    got = y.cpu().numpy()
    taps = np.ascontiguousarray(w.reshape(ch, kernel).T)
    for st, n in zip(segs.starts, lens):
        want = O.conv_glu(h[st * 2 * ch:(st + n) * 2 * ch].copy(), taps, wb, g, b, ln, n, ch,
                          kernel)
        assert_close(got[st:st + n], want)


def oracle_gemm(ty, rows, k, data, bias, a, m, c=None, epi="bias", alpha=1.0):
    O.set_vnni(0)  # the GPU GEMM's rounding: a and W to f16
    try:
        return O.Linear(ty, rows, k, data, bias).gemm(np.ascontiguousarray(a, np.float32).ravel(),
                                                      m, c, epi, alpha)
    finally:
        O.set_vnni(-1)


@pytest.mark.parametrize("ty,kernel,conv_ln", [(O.TY_Q8_0, 9, False), (O.TY_F16, 31, True)])
def test_conformer_block(gpu, ty, kernel, conv_ln):
    # A Parakeet-shaped FastConformer block (d 256, 2 heads of 128, FFN 1024) over packed segments,
    # against the CPU block run per segment: LN -> FFN/2 -> LN -> rel-pos MHSA -> LN -> pointwise ->
    # GLU -> depthwise -> norm -> SiLU -> pointwise -> LN -> FFN/2 -> norm_out.
    from wavo_b200.blocks import ConformerBlock, Segments, rel_positions
    d, heads, f = 256, 2, 1024
    lens = [120, 37, 300]
    rng = np.random.default_rng(7 + kernel)

    def wt(rows, k, std=0.03):
        w = (rng.standard_normal((rows, k)) * std).astype(np.float32)
        return O.q8_0_bytes(w) if ty == O.TY_Q8_0 else w.astype(np.float16).tobytes()

    w = {"ff1_1": wt(f, d), "ff1_2": wt(d, f), "ff2_1": wt(f, d), "ff2_2": wt(d, f),
         "qkv": wt(3 * d, d), "pos": wt(d, d), "out": wt(d, d), "pw1": wt(2 * d, d),
         "pw2": wt(d, d), "u": (rng.standard_normal(d) * 0.02).astype(np.float32),
         "v": (rng.standard_normal(d) * 0.02).astype(np.float32),
         "dw": (rng.standard_normal((d, kernel)) * 0.2).astype(np.float32),
         "dw_b": (rng.standard_normal(d) * 0.1).astype(np.float32)}
    norm = lambda: (1.0 + rng.standard_normal(d).astype(np.float32) * 0.1,  # noqa: E731
                    rng.standard_normal(d).astype(np.float32) * 0.1)
    norms = {k: norm() for k in ("ff1", "attn", "conv", "ff2", "out", "conv_norm")}
    blk = ConformerBlock(gpu, ty, d, f, heads, kernel, w, norms, conv_ln)
    segs = Segments(lens, "cuda")
    t_pos = max(lens)
    table = rel_positions(d, t_pos + 15, 2 * t_pos + 15)
    x0 = rng.standard_normal((segs.rows, d)).astype(np.float32)
    x = gpu.upload(x0)
    out = torch.zeros(segs.rows, d, device="cuda")
    s = blk.scratch(segs.rows, t_pos)
    blk.record(gpu.pass_(), x, out, segs, gpu.upload(table), t_pos, s)
    gpu.sync()
    got = out.cpu().numpy()
    taps = np.ascontiguousarray(w["dw"].T)
    for st, n in zip(segs.starts, lens):
        xs = x0[st:st + n].ravel().copy()
        y = O.layer_norm(xs, *norms["ff1"], n, d)
        h = oracle_gemm(ty, f, d, w["ff1_1"], None, y, n, epi="silu")
        oracle_gemm(ty, d, f, w["ff1_2"], None, h, n, xs, "residual", 0.5)
        y = O.layer_norm(xs, *norms["attn"], n, d)
        # src/cpu/conformer.rs:177-182: the segment's own position table through linear_pos,
        # relative_attention with u and v (the CPU path, in f32).
        qkv = oracle_gemm(ty, 3 * d, d, w["qkv"], None, y, n)
        tab = O.rel_positions(d, n + 15, O.pos_rows(n))
        pos = oracle_gemm(ty, d, d, w["pos"], None, tab, O.pos_rows(n))
        o = O.relative_attention(qkv, pos, w["u"], w["v"], n, heads, d)
        oracle_gemm(ty, d, d, w["out"], None, o, n, xs, "residual", 1.0)
        y = O.layer_norm(xs, *norms["conv"], n, d)
        hp = oracle_gemm(ty, 2 * d, d, w["pw1"], None, y, n)
        yc = O.conv_glu(hp, taps, w["dw_b"], *norms["conv_norm"], conv_ln, n, d, kernel)
        oracle_gemm(ty, d, d, w["pw2"], None, yc, n, xs, "residual", 1.0)
        y = O.layer_norm(xs, *norms["ff2"], n, d)
        h = oracle_gemm(ty, f, d, w["ff2_1"], None, y, n, epi="silu")
        oracle_gemm(ty, d, f, w["ff2_2"], None, h, n, xs, "residual", 0.5)
        want = O.layer_norm(xs, *norms["out"], n, d)
        check(got[st:st + n], want)
