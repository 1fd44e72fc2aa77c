"""The reference's GPU unit tests (vladkens/wavo src/gpu/mod.rs:1682-2361) restated against the
CUDA path, through the C ABI: same inputs (the xorshift `random`), same naive references, same
tolerances (2e-5 · max|want|; 1e-3 for the kernels that compute with f16 operands, as the
reference's 16×16 f16 tier, src/gpu/mod.rs:2196-2200).
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


def assert_near(got, want, tolerance):
    """src/gpu/mod.rs:1745-1751."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape
    scale = max(1.0, float(np.abs(want).max()))
    err = np.abs(got - want)
    i = int(err.argmax())
    assert err[i] <= tolerance * scale, f"[{i}]: {got[i]} vs {want[i]} (tol {tolerance * scale})"


def half(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def run_out(gpu, init, record):
    """src/gpu/mod.rs:1735-1742: an output buffer that starts as `init`, returned after `record`."""
    out = gpu.upload(np.asarray(init, np.float32))
    record(gpu.pass_(), out)
    gpu.sync()
    return out.cpu().numpy()


def epilogue_ref(e, v, c):
    # src/gpu/mod.rs:1765-1787
    if e == "bias":
        return v
    if e == "silu":
        return v / (1 + np.exp(-v))
    if e == "relu":
        return np.maximum(v, 0)
    if e == "residual":
        return c + 0.5 * v
    z = np.abs(np.sqrt(0.5) * v)
    t = 1 / (1 + 0.3275911 * z)
    p = ((((1.0614054 * t - 1.453152) * t) + 1.4214138) * t - 0.28449674) * t
    g = 0.5 * v * (1 + np.sign(v) * (1 - (p + 0.2548296) * t * np.exp(-z * z)))
    if e == "gelu":
        return g
    if e == "gelu_residual":
        return c + g
    return np.tanh(v)


@pytest.mark.parametrize("ty", [O.TY_F32, O.TY_F16, O.TY_Q8_0])
def test_gemm(gpu, ty):
    # src/gpu/mod.rs:1879-1946. 164 rows: outputs padded to 192 columns come out as epilogue(0);
    # 288 rows (a multiple of 32): 288 columns. Biases: own, none (zeros), and 64 dual outputs.
    for n, cols in [(164, 192), (288, 288)]:
        k = 96
        w = O.random(n * k, 1)
        bias = O.random(n, 2)
        dual = np.concatenate([bias, O.random(64, 5)])
        data = {O.TY_F32: w.tobytes(), O.TY_F16: w.astype(np.float16).tobytes(),
                O.TY_Q8_0: O.q8_0_bytes(w)}[ty]
        if ty == O.TY_Q8_0:
            blocks = np.frombuffer(data, np.uint8).reshape(-1, 34)
            d = blocks[:, :2].copy().view(np.float16).astype(np.float32)
            wf = (blocks[:, 2:].view(np.int8).astype(np.float32) * d).reshape(n, k)
        else:
            wf = np.frombuffer(data, np.float32 if ty == O.TY_F32 else np.float16).astype(
                np.float32).reshape(n, k)
        wf = half(wf).astype(np.float64)
        for b in (bias, np.zeros(0, np.float32), dual):
            width = cols + 64 if len(b) > n else cols
            lin = gpu.linear(ty, n, k, data, b)
            assert lin.width() == width
            for m in (1, 37, 70, 2100):
                a = O.random(m * k, 3)
                ar = half(a).astype(np.float64).reshape(m, k)
                c0 = O.random(m * width + 1, 4)
                dot = ar @ wf.T
                ab = gpu.upload(a)
                for e in O.EPILOGUES:
                    want = c0.astype(np.float64).copy()
                    body = want[: m * width].reshape(m, width)
                    cbody = c0[: m * width].reshape(m, width).astype(np.float64)
                    bb = np.zeros(n) if len(b) == 0 else b[:n].astype(np.float64)
                    v = np.zeros((m, cols))
                    v[:, :n] = dot + bb[None, :]
                    body[:, :cols] = epilogue_ref(e, v, cbody[:, :cols])
                    if width > cols:
                        body[:, cols:] = b[n:][None, :].astype(np.float64) + dot[:, :64]
                    got = run_out(gpu, c0, lambda p, out: p.gemm(ab, lin, out, m, e, 0.5))
                    assert_near(got, want, 2e-5)


def test_gemm_f16_io_and_strides(gpu):
    # The fast path's operand types: f16 a in, f16 c out, c written into a wider row.
    m, k, n = 300, 128, 192
    w = O.random(n * k, 11)
    lin = gpu.linear(O.TY_F16, n, k, w.astype(np.float16).tobytes(), O.random(n, 12))
    a = half(O.random(m * k, 13))
    a16 = gpu.upload(a, torch.float16)
    c = torch.zeros(m, 256, dtype=torch.float16, device="cuda")
    gpu.pass_().gemm(a16, lin, c, m, "bias", ldc=256)
    gpu.sync()
    want = a.reshape(m, k).astype(np.float64) @ half(w).reshape(n, k).T.astype(np.float64) + \
        O.random(n, 12)[None, :]
    got = c.float().cpu().numpy()
    assert_near(got[:, :n], want, 2e-3)
    assert not got[:, n:].any()


ATTENTION_SHAPES = [(37, 48), (100, 48), (100, 56), (5, 36), (70, 52), (100, 64), (40, 80)]


def naive_attention(q, k, v, scale):
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    e = np.exp(s - s.max(axis=1, keepdims=True))
    return (e / e.sum(axis=1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("t,hd", ATTENTION_SHAPES)
def test_attention(gpu, t, hd):
    # src/gpu/mod.rs:2163-2202: qk [t][q | k] and v, values exact in f16, heads 2; tolerance of
    # the f16 tier.
    heads = 2
    d = heads * hd
    tp = (t + 63) // 64 * 64
    qk = half(O.random(tp * 2 * d, 15))
    v = half(O.random(tp * d + 4, 16))
    q2, v2 = qk.reshape(tp, 2 * d), v[: tp * d].reshape(tp, d)
    want = np.zeros((t, d))
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        want[:, sl] = naive_attention(q2[:t, sl], q2[:t, d:][:, sl], v2[:t, sl], 1 / np.sqrt(hd))
    qb, vb = gpu.upload(qk), gpu.upload(v)
    got = run_out(gpu, np.zeros(t * d), lambda p, o: p.attention(qb, vb, None, o, t, heads, hd))
    assert_near(got, want, 1e-3)


def naive_relative(qkv, pos, t, heads, hd):
    d = heads * hd
    x = qkv.reshape(-1, 4 * d)
    p = pos.reshape(-1, d)
    want = np.zeros((t, d))
    i = np.arange(t)[:, None]
    j = np.arange(t)[None, :]
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        qu, k, v, qv = (x[:t, s * d:(s + 1) * d][:, sl].astype(np.float64) for s in range(4))
        ac = qu @ k.T
        bd = np.take_along_axis(qv @ p[:, sl].astype(np.float64).T, j + t + 15 - i, axis=1)
        s = (ac + bd) / np.sqrt(hd)
        e = np.exp(s - s.max(axis=1, keepdims=True))
        want[:, sl] = (e / e.sum(axis=1, keepdims=True)) @ v
    return want


@pytest.mark.parametrize("t,heads,hd", [(5, 2, 40), (37, 2, 40), (100, 3, 128)])
def test_relative_attention(gpu, t, heads, hd):
    # src/gpu/mod.rs:2204-2240: qkv [q+u | k | v | q+v], positions of pos_rows(t) (+64) rows.
    d = heads * hd
    qkv = O.random(((t + 63) // 64 * 64) * 4 * d, 17)
    pos = O.random((O.pos_rows(t) + 64) * d, 18)
    want = naive_relative(qkv, pos, t, heads, hd)
    qb, pb = gpu.upload(qkv), gpu.upload(pos)
    got = run_out(gpu, np.zeros(t * d), lambda p, o: p.attention(qb, None, pb, o, t, heads, hd))
    assert_near(got, want, 1e-3)


def test_attend_and_pack(gpu):
    # src/gpu/mod.rs:2069-2130: rows of K then V into a cache of 4100 positions, one query per
    # head over the first n keys (parts of this build's split size), then the pack layout bits.
    keys = 4100
    for heads, hd in [(2, 40), (3, 36)]:
        d = heads * hd
        kv = O.random(keys * 2 * d, 7)
        q = O.random(d, 8)
        rows = kv.reshape(keys, 2 * d)
        qb, xb = gpu.upload(q), gpu.upload(kv)
        cache = torch.zeros(keys * d, dtype=torch.int32, device="cuda")
        from wavo_b200.gpu import attend_len
        part = gpu.buffer(attend_len(keys, heads, hd))
        for n in (1, 37, 256, 257, 1500, 2049, keys):
            want = np.zeros(d)
            qh = half(q).astype(np.float64)
            for h in range(heads):
                kk = half(rows[:n, h * hd:(h + 1) * hd]).astype(np.float64)
                vv = half(rows[:n, d + h * hd:d + (h + 1) * hd]).astype(np.float64)
                s = kk @ qh[h * hd:(h + 1) * hd] / np.sqrt(hd)
                e = np.exp(s - s.max())
                want[h * hd:(h + 1) * hd] = e @ vv / e.sum()

            def rec(p, o):
                p.pack(xb, (0, 2 * d), cache, keys, d, (keys, 0))
                p.attend(qb, cache, part, o, n, keys, heads, hd)

            assert_near(run_out(gpu, np.zeros(d), rec), want, 2e-5)
    # Rows of K then V (d = 6) from x[3..], 13 floats apart, into a cache of 7 positions; one row
    # at position 4, or 2 rows at 5 and 6.
    x = O.random(3 + 13 * 2, 7)
    xb = gpu.upload(x)

    def h16(v):
        return int(np.float16(v).view(np.uint16))

    for rows_, col in [(1, 4), (2, 5)]:
        y = O.random(7 * 6, 9)
        out = torch.as_tensor(y.view(np.int32).copy()).cuda()
        gpu.pass_().pack(xb, (3, 13), out, rows_, 6, (7, col))
        gpu.sync()
        got = out.cpu().numpy().view(np.uint32)
        want = y.view(np.uint32).copy()
        for j in range(rows_):
            def pair(i):
                return h16(x[3 + 13 * j + 2 * i]) | (h16(x[4 + 13 * j + 2 * i]) << 16)
            for i in range(3):
                want[i * 7 + col + j] = pair(i)
                want[3 * 7 + (col + j) * 3 + i] = pair(3 + i)
        assert np.array_equal(got, want), f"pack {rows_} rows"


@pytest.mark.parametrize("neox", [False, True])
def test_rope(gpu, neox):
    # src/gpu/mod.rs:2298-2330
    rows, heads, hd, rot, pos = 5, 3, 10, 6, 2
    stride = 3 * heads * hd
    x = O.random(rows * stride, 30)
    table = O.random((pos + rows) * rot, 31)
    want = x.copy()
    O.rope(want, np.ascontiguousarray(table[pos * rot:]), rows, heads, hd, rot, neox)
    tb = gpu.upload(table)
    got = run_out(gpu, x, lambda p, xb: p.rope(tb, xb, rows, pos, (heads, hd, rot), neox))
    assert_near(got, want, 2e-5)


@pytest.mark.parametrize("neox,hd,rot", [(True, 48, 48), (False, 64, 32), (True, 128, 64)])
def test_rope_f16_rows(gpu, neox, hd, rot):
    # f16 q|k rows (the projection's output), four pairs a thread: as the oracle's rope on the
    # same f16 values, each result rounded to f16 once.
    rows, heads, pos = 37, 4, 3
    stride = 3 * heads * hd
    x = O.f16_round(O.random(rows * stride, 32))
    table = O.random((pos + rows) * rot, 33)
    want = x.copy()
    O.rope(want, np.ascontiguousarray(table[pos * rot:]), rows, heads, hd, rot, neox)
    xb = torch.from_numpy(x).cuda().half()
    gpu.pass_().rope(gpu.upload(table), xb, rows, pos, (heads, hd, rot), neox)
    gpu.sync()
    got = xb.float().cpu().numpy()
    # Only the q and k sections rotate; v stays bit for bit.
    assert np.array_equal(got.reshape(rows, 3, -1)[:, 2], x.reshape(rows, 3, -1)[:, 2])
    assert_near(got, O.f16_round(want), 1e-3)


@pytest.mark.parametrize("ty", [O.TY_F32, O.TY_F16, O.TY_Q8_0])
def test_gemv(gpu, ty):
    # src/cpu/gemm.rs:616-640 `gemv_matches_dot` and Pass::gemv: one row, W not rounded, f32 sums.
    k, n = 96, 70
    i = np.arange(n * k)
    v = ((i * 7919 % 31) / 8.0 - 15.0 / 8.0).astype(np.float32)
    x = ((np.arange(k) * 31 % 17) / 8.0 - 1.0).astype(np.float32)
    bias = (np.arange(n) / 4.0).astype(np.float32)
    if ty == O.TY_Q8_0:
        data = b"".join(np.float16(0.125).tobytes() + (blk * 8).astype(np.int8).tobytes()
                        for blk in v.reshape(-1, 32))
    elif ty == O.TY_F16:
        data = v.astype(np.float16).tobytes()
    else:
        data = v.tobytes()
    lin = gpu.linear(ty, n, k, data, bias)
    xb = gpu.upload(x)
    want = O.Linear(ty, n, k, data, bias).gemv(x, epilogue="gelu")
    got = run_out(gpu, np.zeros(lin.cols + 3), lambda p, c: p.gemv(xb, lin, c, "gelu", offset=3))
    assert_near(got[3:3 + n], want, 2e-5)


@pytest.mark.parametrize("rows,n,k", [
    (3, 96, 224),         # one ragged tile, k over a cluster of four (k % 64 == 32: zero fill)
    (32, 1280, 1280),     # Whisper's d x d projections: k over a cluster of seven
    (5, 5120, 1280),      # the FFN's first projection: clusters of three
    (32, 1280, 5120),     # the FFN's second: clusters of eight
    (17, 40000, 256),     # many tiles: two or three a CTA, sharing the X chunks
    (3, 80000, 64),       # five tiles a CTA (512 TMEM columns)
    (2, 128, 8192),       # one tile, a long k over eight CTAs: the X slots reused many times
])
@pytest.mark.parametrize("epi", ["bias", "gelu", "residual", "gelu_residual", "silu", "tanh"])
def test_gemv_rows_tc(gpu, rows, n, k, epi):
    # Pass::gemv over a batch of rows (src/gpu/mod.rs:1461-1467) with F16 weights, on the tensor
    # core with every epilogue, against the oracle's gemv of each row (W exact, f32 sums).
    rng = np.random.default_rng(n + k + rows)
    data = (rng.standard_normal(n * k) * 0.05).astype(np.float16).tobytes()
    bias = rng.standard_normal(n).astype(np.float32)
    x = rng.standard_normal(rows * k).astype(np.float32)
    c0 = rng.standard_normal(rows * n).astype(np.float32)
    lin = gpu.linear(O.TY_F16, n, k, data, bias)
    assert lin.cols == n  # c rows of n floats
    ref = O.Linear(O.TY_F16, n, k, data, bias)
    want = c0.reshape(rows, n).copy()
    for r in range(rows):
        ref.gemv(np.ascontiguousarray(x[r * k:(r + 1) * k]), want[r], epi, 0.5)
    xb = gpu.upload(x)
    got = run_out(gpu, c0, lambda p, c: p.gemv_rows(xb, lin, c, rows, epi, 0.5))
    assert_near(got, want, 2e-5)


@pytest.mark.parametrize("m,n,k,dual", [
    (1, 164, 96, 0),        # k % 64 == 32: the last K-step's second half is the TMA's zero fill
    (37, 288, 96, 64),      # dual outputs
    (138, 3072, 1024, 1024),  # C1: the rel-pos layer's [q+u | k | v | q+v] projection
    (300, 1024, 1024, 0),   # three row tiles
    (2100, 1024, 256, 0),   # many row tiles: the persistent tile loop
])
def test_gemm_q8_prologue_matches_dequant(gpu, m, n, k, dual):
    # Q8_0 dequantised in the GEMM's prologue (src/gpu/gemm.wgsl:105-130) against the layer's
    # load-time f16 copy: the converters round q·d to f16 as the load does, so the outputs are
    # bit-identical.
    from wavo_b200 import _lib as L
    w = O.random(n * k, 11) * 0.05
    b = O.random(n + dual, 12)
    lin = gpu.linear(O.TY_Q8_0, n, k, O.q8_0_bytes(w), b)
    width = lin.width()
    a = gpu.upload(O.random(m * k, 13))
    c0 = O.random(m * width, 14)
    outs = {}
    old = gpu.set_q8_gemm(L.Q8_AUTO)
    try:
        for mode in (L.Q8_DEQUANT, L.Q8_PROLOGUE):
            gpu.set_q8_gemm(mode)
            for e in ("bias", "residual", "gelu"):
                outs[mode, e] = run_out(gpu, c0, lambda p, out: p.gemm(a, lin, out, m, e, 0.5))
    finally:
        gpu.set_q8_gemm(old)
    for e in ("bias", "residual", "gelu"):
        np.testing.assert_array_equal(outs[L.Q8_PROLOGUE, e], outs[L.Q8_DEQUANT, e])


@pytest.mark.parametrize("vnni", [0, -1])
def test_gemm_q8_prologue_vs_oracle(gpu, vnni):
    # The C1/C5 projection shape through the prologue path against the CPU oracle's Q8_0 GEMM, in
    # its f16-rounded mode and in the mode the reference picks on this host (i16 VNNI on AVX-VNNI,
    # src/cpu/gemm.rs:129-161), at the model tolerance.
    from wavo_b200 import _lib as L
    m, n, k = 138, 1024, 1024
    rng = np.random.default_rng(5)
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    data = O.q8_0_bytes(w)
    lin = gpu.linear(O.TY_Q8_0, n, k, data, None)
    a = rng.standard_normal(m * k).astype(np.float32)
    old = gpu.set_q8_gemm(L.Q8_PROLOGUE)
    try:
        got = run_out(gpu, np.zeros(m * n, np.float32),
                      lambda p, out: p.gemm(gpu.upload(a), lin, out, m, "bias"))
    finally:
        gpu.set_q8_gemm(old)
    prev = O.vnni()
    O.set_vnni(vnni)
    try:
        want = O.Linear(O.TY_Q8_0, n, k, data, np.zeros(n, np.float32)).gemm(a, m)
    finally:
        O.set_vnni(prev)
    err = np.abs(got - want)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err.max() <= 2e-3 and rel <= 1e-3, f"max-abs {err.max():.3g}, rel-L2 {rel:.3g}"
