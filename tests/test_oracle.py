"""Pins the CPU oracle (a C++ restatement of the reference's CPU attention path) against the
reference's own unit tests: their inputs (the xorshift `random`, the integer-pattern weights), their
naive references and their tolerances.

Reference tests restated here:
- src/cpu/gemm.rs:578-604 `gemm_matches_dot`, 606-614 `halves_round_as_f16`, 616-640
  `gemv_matches_dot`;
- src/gpu/mod.rs:1879-1946 `gemm`, 2069-2130 `attend_and_pack`, 2163-2202 `attention`,
  2204-2240 `relative_attention`, 2298-2330 `rope` (their naive references run here against the
  CPU functions the GPU kernels restate).
"""

import numpy as np
import pytest

from oracle import oracle as O


def assert_near(got, want, tolerance):
    """src/gpu/mod.rs:1745-1751: |got - want| <= tolerance · max(1, max|want|)."""
    got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape
    scale = max(1.0, float(np.abs(want).max()))
    err = np.abs(got - want)
    i = int(err.argmax())
    assert err[i] <= tolerance * scale, f"[{i}]: {got[i]} vs {want[i]} (tol {tolerance * scale})"


def test_random_is_the_reference_xorshift():
    # src/gpu/mod.rs:1717-1727, restated in numpy (u32 wrap-around, f32 arithmetic).
    def ref(n, seed):
        x = np.uint32((seed * 2654435761) % 2**32 | 1)
        out = []
        for _ in range(n):
            x ^= np.uint32((int(x) << 13) % 2**32)
            x ^= np.uint32(int(x) >> 17)
            x ^= np.uint32((int(x) << 5) % 2**32)
            out.append(np.float32(np.float32(x) / np.float32(4294967295.0)) * np.float32(2.0)
                       - np.float32(1.0))
        return np.array(out, np.float32)

    for seed in (1, 7, 15, 17, 31):
        assert np.array_equal(O.random(257, seed), ref(257, seed))


def test_halves_round_as_f16():
    # src/cpu/gemm.rs:606-614: to_half(x) == f16::from_f32(x).to_f32() over normal and subnormal
    # halves of both signs below the f16 maximum. numpy's float16 cast is an independent IEEE
    # round-to-nearest-even implementation; it pins both the oracle's to_half and its f16 rounding.
    b = np.arange(0x30000000, 0x47700000, 4093, dtype=np.uint32)
    x = b.view(np.float32)
    x = np.concatenate([x, -x])
    want = x.astype(np.float16).astype(np.float32)
    assert np.array_equal(O.to_half(x), want)
    assert np.array_equal(O.f16_round(x), want)


def test_exp_is_cephes_within_its_bound():
    # src/cpu/ops.rs:12-26: relative error ~1e-7 against the true exponential.
    xs = np.linspace(-80, 80, 10001, dtype=np.float32)
    got = np.array([O.exp(float(x)) for x in xs], np.float64)
    want = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(got / want - 1)) < 3e-7


def _int_pattern(n, k):
    # The reference's weights exact in every type: (i·7919 % 31)/8 − 15/8.
    i = np.arange(n * k)
    return ((i * 7919 % 31) / 8.0 - 15.0 / 8.0).astype(np.float32)


def _q8_exact(v):
    # Blocks with scale 0.125 and q = v·8 (src/cpu/gemm.rs:583-587).
    out = bytearray()
    for blk in v.reshape(-1, 32):
        out += np.float16(0.125).tobytes() + (blk * 8).astype(np.int8).tobytes()
    return bytes(out)


@pytest.mark.parametrize("vnni", [0, -1])
def test_gemm_matches_dot(vnni):
    # src/cpu/gemm.rs:578-604; vnni 0 forces the f16 tile, -1 lets the CPU choose (the i16 VNNI
    # path for Q8_0 where the CPU has AVX-VNNI or AVX512-VNNI, as the reference does).
    O.set_vnni(vnni)
    try:
        k, n, m = 64, 40, 13
        v = _int_pattern(n, k)
        i = np.arange(m * k)
        a = ((i * 31 % 17) / 8.0 - 1.0).astype(np.float32)
        bias = (np.arange(n) / 4.0).astype(np.float32)
        want = a.reshape(m, k).astype(np.float64) @ v.reshape(n, k).astype(np.float64).T
        for ty, data in [(O.TY_F32, v.tobytes()), (O.TY_F16, v.astype(np.float16).tobytes()),
                         (O.TY_Q8_0, _q8_exact(v))]:
            lin = O.Linear(ty, n, k, data, bias)
            c = np.ones(m * n, np.float32)
            lin.gemm(a, m, c, "residual", 0.5)
            w = 1.0 + 0.5 * (want + bias[None, :])
            assert np.all(np.abs(c.reshape(m, n) - w) <= 1e-4 * np.maximum(np.abs(w), 1.0)), ty
    finally:
        O.set_vnni(-1)


def test_gemv_matches_dot():
    # src/cpu/gemm.rs:616-640: bit-exact against gelu(dot(x, row) + bias).
    k, n = 96, 70
    v = _int_pattern(n, k)
    x = ((np.arange(k) * 31 % 17) / 8.0 - 1.0).astype(np.float32)
    bias = (np.arange(n) / 4.0).astype(np.float32)
    rows = v.reshape(n, k)
    lib = O.lib()
    want = np.array([lib.wo_gelu(lib.wo_dot(O._p(np.ascontiguousarray(x)),
                                            O._p(np.ascontiguousarray(rows[r])), k) + bias[r])
                     for r in range(n)], np.float32)
    for ty, data in [(O.TY_F32, v.tobytes()), (O.TY_Q8_0, _q8_exact(v))]:
        c = O.Linear(ty, n, k, data, bias).gemv(x, epilogue="gelu")
        assert np.array_equal(c, want), ty


def _epilogue(e, v, c):
    # src/gpu/mod.rs:1765-1787 (the test's own silu/gelu/tanh with std exp).
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
def test_gemm_against_the_gpu_tests_reference(ty):
    # src/gpu/mod.rs:1879-1946 on the CPU oracle's f16 path (the GPU's rounding: a and W to f16).
    # The GPU-only padding and dual outputs are checked in the CUDA tests.
    O.set_vnni(0)
    try:
        k = 96
        for n in (164, 288):
            w = O.random(n * k, 1)
            bias = O.random(n, 2)
            data = {O.TY_F32: w.tobytes(), O.TY_F16: w.astype(np.float16).tobytes(),
                    O.TY_Q8_0: O.q8_0_bytes(w)}[ty]
            if ty == O.TY_Q8_0:
                blocks = np.frombuffer(data, np.uint8).reshape(-1, 34)
                d = blocks[:, :2].copy().view(np.float16).astype(np.float32)
                q = blocks[:, 2:].view(np.int8).astype(np.float32)
                wf = (q * d).reshape(n, k)
            else:
                wf = np.frombuffer(data, np.float32 if ty == O.TY_F32 else np.float16).astype(
                    np.float32).reshape(n, k)
            wf = wf.astype(np.float16).astype(np.float64)
            for b in (bias, None):
                lin = O.Linear(ty, n, k, data, b)
                for m in (1, 37, 70, 2100):
                    a = O.random(m * k, 3)
                    ar = a.astype(np.float16).astype(np.float64).reshape(m, k)
                    c0 = O.random(m * n, 4)
                    dot = ar @ wf.T + (0 if b is None else b[None, :].astype(np.float64))
                    for e in O.EPILOGUES:
                        c = c0.copy()
                        lin.gemm(a, m, c, e, 0.5)
                        want = _epilogue(e, dot, c0.reshape(m, n).astype(np.float64))
                        assert_near(c, want, 2e-5)
    finally:
        O.set_vnni(-1)


ATTENTION_SHAPES = [(37, 48), (100, 48), (100, 56), (5, 36), (70, 52), (100, 64), (40, 80)]


def naive_attention(q, k, v, scale):
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    e = np.exp(s - s.max(axis=1, keepdims=True))
    return (e / e.sum(axis=1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("t,hd", ATTENTION_SHAPES)
def test_attention(t, hd):
    # src/gpu/mod.rs:2163-2202: qk [t][q | k], v [t][d], values exact in f16, heads 2.
    heads = 2
    d = heads * hd
    tp = (t + 63) // 64 * 64
    qk = O.f16_round(O.random(tp * 2 * d, 15))
    v = O.f16_round(O.random(tp * d + 4, 16))
    got = O.attention(qk, 2 * d, v, d, t, heads, d)
    q2 = qk.reshape(tp, 2 * d)
    v2 = v[: tp * d].reshape(tp, d)
    for h in range(heads):
        want = naive_attention(q2[:t, h * hd:(h + 1) * hd], q2[:t, d + h * hd:d + (h + 1) * hd],
                               v2[:t, h * hd:(h + 1) * hd], 1 / np.sqrt(hd))
        assert_near(got[:, h * hd:(h + 1) * hd], want, 2e-5)


def naive_relative(qu, qv, k, v, pos, t, scale):
    # score (i, j) = (q+u)_i·k_j + (q+v)_i·pos[j + t + 15 − i]   (src/gpu/mod.rs:2213-2224)
    ac = qu.astype(np.float64) @ k.astype(np.float64).T
    i = np.arange(t)[:, None]
    j = np.arange(t)[None, :]
    bd_full = qv.astype(np.float64) @ pos.astype(np.float64).T
    bd = np.take_along_axis(bd_full, j + t + 15 - i, axis=1)
    s = (ac + bd) * scale
    e = np.exp(s - s.max(axis=1, keepdims=True))
    return (e / e.sum(axis=1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("t,heads,hd", [(5, 2, 48), (37, 2, 48), (100, 3, 128)])
def test_relative_attention(t, heads, hd):
    # src/gpu/mod.rs:2204-2240. The CPU function takes qkv [t][q | k | v] and the biases u, v
    # (src/cpu/ops.rs:228); the GPU test's [q+u | k | v | q+v] rows are formed from them with the
    # same f32 additions. The CPU function needs heads of a multiple of 16 dims (the reference
    # asserts it; src/cpu/conformer.rs:58), so the GPU test's heads of 40 become 48 here.
    d = heads * hd
    qkv = O.random(t * 3 * d, 17)
    pos = O.random((O.pos_rows(t) + 64) * d, 18)
    u, vb = O.random(d, 19), O.random(d, 20)
    got = O.relative_attention(qkv, pos, u, vb, t, heads, d)
    x = qkv.reshape(t, 3 * d)
    p = pos.reshape(-1, d)[: O.pos_rows(t)]
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        q = x[:, sl]
        qu, qv = (q + u[sl]).astype(np.float32), (q + vb[sl]).astype(np.float32)
        want = naive_relative(qu, qv, x[:, d:][:, sl], x[:, 2 * d:][:, sl], p[:, sl], t,
                              1 / np.sqrt(hd))
        assert_near(got[:, sl], want, 2e-5)


def test_attend_and_pack():
    # src/gpu/mod.rs:2069-2130 on the CPU path: rows [K | V] of all heads rounded to f16 into the
    # cache (src/cpu/transformer.rs:209-222), then one query per head (rounded to f16).
    keys = 4100
    for heads, hd in [(2, 40), (3, 36)]:
        d = heads * hd
        kv = O.random(keys * 2 * d, 7)
        q = O.random(d, 8)
        cache = np.zeros(keys * 2 * d, np.float32)
        O.pack_cache(kv, keys, d, hd, cache, keys, 0)
        rows = kv.reshape(keys, 2 * d)
        qh = q.astype(np.float16).astype(np.float64)
        for n in [1, 37, 256, 257, 1500, 2049, keys]:
            got = O.attend(q, cache, keys, n, heads, hd)
            want = np.zeros(d)
            for h in range(heads):
                kk = rows[:n, h * hd:(h + 1) * hd].astype(np.float16).astype(np.float64)
                vv = rows[:n, d + h * hd:d + (h + 1) * hd].astype(np.float16).astype(np.float64)
                s = kk @ qh[h * hd:(h + 1) * hd] / np.sqrt(hd)
                e = np.exp(s - s.max())
                want[h * hd:(h + 1) * hd] = e @ vv / e.sum()
            assert_near(got, want, 2e-5)


def test_relative_attention_rejects_heads_off_16():
    d = 2 * 40
    with pytest.raises(ValueError):
        O.relative_attention(O.random(5 * 3 * d, 1), O.random(O.pos_rows(5) * d, 2),
                             O.random(d, 3), O.random(d, 4), 5, 2, d)


@pytest.mark.parametrize("neox", [False, True])
def test_rope(neox):
    # src/gpu/mod.rs:2298-2330: rows [q | k | v] of 3 heads of 10, the first 6 dims of q's and k's
    # heads rotating, from position 2.
    rows, heads, hd, rot, pos = 5, 3, 10, 6, 2
    stride = 3 * heads * hd
    x = O.random(rows * stride, 30)
    table = O.random((pos + rows) * rot, 31)
    want = x.copy()
    for e in range(x.size):
        r, i = divmod(e, stride)
        dd = i % hd
        if i >= 2 * heads * hd or dd >= rot:
            continue
        t = table[(pos + r) * rot:]
        if neox:
            pair, first, step = dd % (rot // 2), dd < rot // 2, rot // 2
        else:
            pair, first, step = dd // 2, dd % 2 == 0, 1
        c, s = t[pair], t[rot // 2 + pair]
        want[e] = x[e] * c - x[e + step] * s if first else x[e - step] * s + x[e] * c
    got = x.copy()
    O.rope(got, np.ascontiguousarray(table[pos * rot:]), rows, heads, hd, rot, neox)
    assert_near(got, want, 2e-5)


def test_rel_positions_and_rope_table():
    # src/conformer.rs:141-153 and src/gigaam/mod.rs:88-96 in float64 (parity unpinned by any
    # reference test; within f32 rounding of libm).
    d, first, rows = 64, 20, 7
    got = O.rel_positions(d, first, rows)
    k = np.arange(d // 2)
    div = np.exp(2 * k * (-np.log(10000.0) / d))
    pos = (first - np.arange(rows))[:, None]
    assert np.allclose(got[:, 0::2], np.sin(pos * div), atol=2e-5)
    assert np.allclose(got[:, 1::2], np.cos(pos * div), atol=2e-5)
    tab = O.rope_table(9, 48, 10000.0).reshape(9, 48)
    ang = np.arange(9)[:, None] * 10000.0 ** (-2.0 * np.arange(24) / 48)
    assert np.allclose(tab[:, :24], np.cos(ang), atol=1e-7)
    assert np.allclose(tab[:, 24:], np.sin(ang), atol=1e-7)


def test_layer_norm_and_conv_glu_restatements():
    # The oracle's layer_norm (src/cpu/ops.rs:65-110) and conv_glu (133-182) against the naive
    # references of the reference's GPU tests (src/gpu/mod.rs:1753-1763, 1947-1973, 2131-2160) on
    # their inputs, at their tolerance (2e-5 · max(1, max|want|)).
    def close(got, want):
        got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
        assert np.abs(got - want).max() <= 2e-5 * max(1.0, np.abs(want).max())

    def naive_ln(x, g, b):
        x = x.reshape(-1, g.size).astype(np.float64)
        mean = x.mean(axis=1, keepdims=True)
        var = ((x - mean) ** 2).mean(axis=1, keepdims=True)
        return (x - mean) / np.sqrt(var + 1e-5) * g + b

    rows, cols, hd = 37, 192, 48
    x, g, b = O.random(rows * cols, 5), O.random(cols, 6), O.random(cols, 7)
    rope = O.random(rows * hd, 8)
    y = naive_ln(x, g, b).ravel()
    half = hd // 2
    idx = np.arange(rows * cols)
    t, dd = idx // cols, idx % hd
    cos, sin = rope[t * hd + dd % half], rope[t * hd + half + dd % half]
    partner = np.where(dd < half, idx + half, idx - half)
    yr = np.where(dd < half, y * cos - y[partner] * sin, y * cos + y[partner] * sin)
    oy, oyr = O.layer_norm(x, g, b, rows, cols, rope, hd)
    close(oy, y)
    close(oyr, yr)
    close(O.layer_norm(x, g, b, rows, cols), y)

    t, ch = 37, 192
    h = O.random(t * 2 * ch, 10)
    g, b = O.random(ch, 13), O.random(ch, 14)
    hh = h.reshape(t, 2 * ch).astype(np.float64)
    glu = hh[:, :ch] / (1.0 + np.exp(-hh[:, ch:]))
    for kernel, ln in [(5, True), (9, False)]:
        w, wb = O.random(ch * kernel, 11), O.random(ch, 12)
        wk = w.reshape(ch, kernel).astype(np.float64)
        dw = np.tile(wb.astype(np.float64), (t, 1))
        for r in range(t):
            for k in range(kernel):
                if 0 <= r + k - kernel // 2 < t:
                    dw[r] += wk[:, k] * glu[r + k - kernel // 2]
        want = naive_ln(dw, g, b) if ln else dw * g + b
        want = want / (1.0 + np.exp(-want))
        hc = h.copy()
        got = O.conv_glu(hc, np.ascontiguousarray(wk.T.astype(np.float32)), wb, g, b, ln, t, ch,
                         kernel)
        close(got, want)
        # The CPU conv_glu leaves the GLU in h's first halves (src/cpu/ops.rs:146-156).
        close(hc.reshape(t, 2 * ch)[:, :ch], glu)


def test_pick_restates_reference_rules():
    # src/whisper/search.rs:180-225 (tests): a vocabulary of 20 (text 0..10, EOT 10,
    # <|notimestamps|> 12, timestamps 13..20); with all logits equal, which tokens the timestamp
    # rules leave open, and the scripted greedy decode T, 3, T + 4, EOT.
    T = 13

    def rules(generated):
        lg = np.zeros(20, np.float32)
        O.pick(lg, generated, [], [], 10, 12, T)
        return list(np.isfinite(lg))

    allowed = lambda s: [i in s for i in range(20)]  # noqa: E731
    assert rules([]) == allowed(range(T, 20))
    assert rules([T, 3, T + 2]) == allowed(range(T + 2, 20))
    assert rules([T, 3, T + 2, T + 2]) == allowed(range(0, 12))
    assert rules([T + 1, 3]) == allowed(range(T + 2, 20))

    one_hot = lambda i: np.array([5.0 if j == i else 0.0 for j in range(20)], np.float32)  # noqa: E731
    gen, lps = [], []
    for logits in (one_hot(T), one_hot(3), one_hot(T + 4), one_hot(10)):
        tok, lp = O.pick(logits, gen, [11], [1, 10], 10, 12, T)
        lps.append(lp)
        if tok == 10:
            break
        gen.append(tok)
    assert gen == [T, 3, T + 4]
    assert -1.0 < float(np.mean(lps)) < 0.0


# ---- the log-mel frontend ----------------------------------------------------------------------

def test_fft_matches_a_dft():
    # src/fft.rs:150-175 `matches_a_dft` (f64, tolerance 1e-10), and numpy's FFT besides.
    for n in (320, 360, 400, 512, 15):
        x = np.array([((i * 7919 % 1000) / 500.0 - 1.0) * 0.3 for i in range(n)])
        re, im = O.fft(x)
        k = np.arange(n)
        phase = 2 * np.pi * ((k[:, None] * k[None, :]) % n) / n
        assert np.abs(re - (x[None, :] * np.cos(phase)).sum(1)).max() < 1e-10
        assert np.abs(im + (x[None, :] * np.sin(phase)).sum(1)).max() < 1e-10
        ref = np.fft.fft(x)
        assert np.abs(re - ref.real).max() < 1e-10 and np.abs(im - ref.imag).max() < 1e-10


def test_frontend_short_input():
    # src/parakeet/frontend.rs:143-150 `short_input`.
    assert O.mel_features(np.full(319, 0.1, np.float32)).size == 0
    mel = O.mel_features(np.full(320, 0.1, np.float32))
    assert mel.shape == (3, O.MELS) and np.isfinite(mel).all()


def test_frontend_frame_ranges():
    # src/parakeet/frontend.rs:152-161 `frame_ranges`: a range of frames equals those frames of the
    # whole audio, at the edges too.
    pcm = (np.sin(np.arange(16000, dtype=np.float32) * np.float32(0.01)) * np.float32(0.5)).astype(np.float32)
    whole = O.log_mel(pcm, 0, 101)
    for a, b in ((0, 1), (0, 7), (3, 40), (95, 101), (100, 101)):
        np.testing.assert_array_equal(O.log_mel(pcm, a, b), whole[a:b])


def test_frontend_filterbank_and_window():
    # librosa's Slaney mel filters peak at 2 / (f[m+2] - f[m]) and partition the band: each bin of
    # 0-8 kHz lies under at most two filters; the window is a symmetric Hann of 400 centred in 512.
    w, f = O.frontend_tables()
    assert (w[:56] == 0).all() and (w[456:] == 0).all() and w[56] == 0.0
    np.testing.assert_allclose(w[56:456], w[56:456][::-1], atol=1e-15)
    assert ((f > 0).sum(axis=0) <= 2).all() and (f >= 0).all()
    assert f.shape == (128, 257) and (f.sum(axis=1) > 0).all()


def _subsample_numpy(mel, valid, tp, w3, b3, w6, b6, wo, bo):
    """Parakeet's subsampling written again with numpy (the same convolutions, a different code)
    to check the oracle's restatement; the GEMMs here are f64 on the f16-rounded operands."""
    h = lambda n: (n - 1) // 2 + 1  # noqa: E731
    frames, ch = mel.shape[0], tp["b0"].size
    t1, f1 = h(valid), 64
    f2, t2, t, f = 32, h(h(frames)), h(h(h(frames - 1))), 16
    m = np.zeros((valid + 2, 130), np.float64)
    m[1:valid + 1, 1:129] = mel[:valid]
    c0 = np.zeros((t1 + 2, f1 + 2, ch))
    for r in range(t1):
        for c in range(f1):
            acc = tp["b0"].astype(np.float64).copy()
            for tap in range(9):
                tm, fm = 2 * r + tap // 3, 2 * c + tap % 3
                v = m[tm, fm] if tm < valid + 2 else 0.0
                acc += tp["w0"][tap] * v
            c0[r + 1, c + 1] = np.maximum(acc, 0)
    a = np.zeros((t2, f2, ch))
    for k in range(min(t2, h(t1))):
        for fo in range(f2):
            acc = tp["b2"].astype(np.float64).copy()
            for tap in range(9):
                acc += tp["w2"][tap] * c0[2 * k + tap // 3, 2 * fo + tap % 3]
            a[k, fo] = acc
    half_ = lambda x: x.astype(np.float16).astype(np.float64)  # noqa: E731
    b = np.maximum(half_(a.reshape(-1, ch)) @ half_(w3).T + b3, 0).reshape(t2, f2, ch)
    bp = np.zeros((t2 + 2, f2 + 2, ch))
    bp[1:t2 + 1, 1:f2 + 1] = b
    y = np.zeros((t, f, ch))
    for k in range(t):
        for fo in range(f):
            acc = tp["b5"].astype(np.float64).copy()
            for tap in range(9):
                acc += tp["w5"][tap] * bp[2 * k + tap // 3, 2 * fo + tap % 3]
            y[k, fo] = acc
    y = np.maximum(half_(y.reshape(-1, ch)) @ half_(w6).T + b6, 0).reshape(t, f, ch)
    flat = y.transpose(0, 2, 1).reshape(t, ch * f)
    return half_(flat) @ half_(wo).T + bo


def subsample_case(frames, valid, ch, d, seed):
    rng = np.random.default_rng(seed)
    mel = rng.standard_normal((frames, 128)).astype(np.float32)
    tp = {k: (rng.standard_normal((9, ch)) * 0.3).astype(np.float32) for k in ("w0", "w2", "w5")}
    tp.update({k: (rng.standard_normal(ch) * 0.1).astype(np.float32) for k in ("b0", "b2", "b5")})
    w3, w6 = (rng.standard_normal((2, ch, ch)) * 0.1).astype(np.float32)
    wo = (rng.standard_normal((d, 16 * ch)) * 0.05).astype(np.float32)
    b3, b6, bo = (rng.standard_normal((3, max(ch, d))) * 0.1).astype(np.float32)
    b3, b6, bo = b3[:ch].copy(), b6[:ch].copy(), bo[:d].copy()
    return mel, tp, w3, b3, w6, b6, wo, bo


@pytest.mark.parametrize("frames,valid", [(97, 97), (97, 60), (33, 33)])
def test_subsample_restatement(frames, valid):
    ch, d = 32, 64
    mel, tp, w3, b3, w6, b6, wo, bo = subsample_case(frames, valid, ch, d, frames + valid)
    O.set_vnni(0)
    try:
        l3 = O.Linear(O.TY_F16, ch, ch, w3.astype(np.float16).tobytes(), b3)
        l6 = O.Linear(O.TY_F16, ch, ch, w6.astype(np.float16).tobytes(), b6)
        lo = O.Linear(O.TY_F16, d, 16 * ch, wo.astype(np.float16).tobytes(), bo)
        got = O.subsample(mel, valid, tp, l3, l6, lo)
    finally:
        O.set_vnni(-1)
    want = _subsample_numpy(mel, valid, tp, w3.astype(np.float16).astype(np.float32), b3,
                            w6.astype(np.float16).astype(np.float32), b6,
                            wo.astype(np.float16).astype(np.float32), bo)
    h = lambda n: (n - 1) // 2 + 1  # noqa: E731
    assert got.shape == (h(h(h(frames - 1))), d)
    err = np.abs(got - want).max() / max(1.0, np.abs(want).max())
    assert err < 2e-3, err
