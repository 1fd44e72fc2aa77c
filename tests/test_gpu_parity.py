"""Parity of the CUDA path with the CPU oracle (the reference's src/cpu attention path restated) at
the BASELINE.json configurations' shapes, within the BASELINE tolerance: max-abs error 2e-3 and
relative-L2 error 1e-3.

Level (i): identical attention inputs (the f16 values the kernel reads) into the oracle's f32
attention. Level (ii): a whole attention layer — projection, attention, output projection with its
residual — against the oracle's f16-rounded GEMM and f32 attention (src/cpu/gemm.rs, ops.rs).
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-3, 1e-3


def check(got, want, max_abs=MAX_ABS, rel_l2=REL_L2):
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


def f16(x):
    return np.ascontiguousarray(np.asarray(x, np.float32).astype(np.float16).astype(np.float32))


def qkv_like(rng, t, ch, sections, std=0.7):
    """Activations shaped like projection outputs of N(0,1) rows through N(0, 0.02) weights."""
    return (rng.standard_normal((t, sections * ch)) * std).astype(np.float32)


@pytest.mark.parametrize("t,heads,hd", [(1500, 20, 64), (1000, 20, 64), (750, 16, 48),
                                         (300, 4, 128), (129, 2, 64)])
def test_plain_attention_level_i(gpu, t, heads, hd):
    # C2 (Whisper turbo encoder; 7 CTAs of 224 rows a head), 1000 rows (CTAs of 144 rows: one live
    # row group in the second tile), C3 (GigaAM heads of 48), and tile edges; f16 operands straight
    # from a [t][q | k | v] f16 buffer (the fast path).
    rng = np.random.default_rng(t + hd)
    ch = heads * hd
    x = f16(qkv_like(rng, t, ch, 3))
    want = O.attention(x.ravel(), 3 * ch, np.ascontiguousarray(x.ravel()[2 * ch:]), 3 * ch, t,
                       heads, ch)
    xb = torch.from_numpy(x).cuda().half()
    o = torch.zeros(t, ch, dtype=torch.float16, device="cuda")
    gpu.pass_().attention(xb, None, None, o, t, heads, hd)
    gpu.sync()
    check(o.float().cpu().numpy(), want)


def grid(rng, shape, step, bound):
    """Values on a grid of `step` (a power of two) within (-bound, bound): sums of such values stay
    exact in f16 and f32, so that the GPU's f16 operands and the oracle's f32 operands agree."""
    x = np.clip(rng.standard_normal(shape) * bound / 3, -bound + step, bound - step)
    return (np.round(x / step) * step).astype(np.float32)


def rel_inputs(rng, t, heads, hd, pos_rows):
    """q, k, v, u, v_bias and a position table on which q+u and q+v are exact in f16: the GPU's
    [q+u | k | v | q+v] rows and the oracle's own sums of q [q | k | v] with u and v are the same
    values (level (i))."""
    ch = heads * hd
    q = grid(rng, (t, ch), 2.0 ** -8, 4.0)
    kv = f16(qkv_like(rng, t, ch, 2))
    u = grid(rng, ch, 2.0 ** -8, 0.25)
    vb = grid(rng, ch, 2.0 ** -8, 0.25)
    pos = f16(rng.standard_normal((pos_rows, ch)) * 0.5)
    qkv = np.ascontiguousarray(np.concatenate([q, kv], axis=1))
    quv = np.ascontiguousarray(np.concatenate([q + u, kv, q + vb], axis=1))
    assert np.array_equal(f16(quv), quv)
    return qkv, quv, u, vb, pos


@pytest.mark.parametrize("t", [138, 300, 64, 1])
def test_relative_attention_level_i(gpu, t):
    # C1 / C5 shapes, 8 heads of 128, positions pos_rows(t), against the oracle's
    # relative_attention (src/cpu/ops.rs:223-273) on identical values; f32 and f16 operand rows.
    heads, hd = 8, 128
    ch = heads * hd
    rng = np.random.default_rng(t)
    qkv, quv, u, vb, pos = rel_inputs(rng, t, heads, hd, O.pos_rows(t))
    want = O.relative_attention(qkv.ravel(), pos.ravel(), u, vb, t, heads, ch)
    for dtype in (torch.float32, torch.float16):
        xb = torch.from_numpy(quv).cuda().to(dtype)
        pb = torch.from_numpy(pos).cuda().to(dtype)
        o = torch.zeros(t, ch, dtype=dtype, device="cuda")
        gpu.pass_().attention(xb, None, pb, o, t, heads, hd)
        gpu.sync()
        check(o.float().cpu().numpy(), want)


def test_relative_attention_matches_the_cpu_oracle(gpu):
    # The oracle's own relative_attention (src/cpu/ops.rs:223-273) on qkv [q | k | v], u and v:
    # the GPU gets [q+u | k | v | q+v] as the reference's dual-bias projection writes it.
    t, heads, hd = 138, 8, 128
    ch = heads * hd
    rng = np.random.default_rng(7)
    qkv = qkv_like(rng, t, ch, 3)
    u = (rng.standard_normal(ch) * 0.02).astype(np.float32)
    vb = (rng.standard_normal(ch) * 0.02).astype(np.float32)
    pos = (rng.standard_normal((O.pos_rows(t), ch)) * 0.5).astype(np.float32)
    want = O.relative_attention(qkv.ravel(), pos.ravel(), u, vb, t, heads, ch)
    q = qkv[:, :ch]
    quv = np.ascontiguousarray(np.concatenate([q + u, qkv[:, ch:], q + vb], axis=1))
    o = torch.zeros(t, ch, device="cuda")
    gpu.pass_().attention(torch.from_numpy(quv).cuda(), None, torch.from_numpy(pos).cuda(), o, t,
                          heads, hd)
    gpu.sync()
    check(o.cpu().numpy(), want)


def test_varlen_segments(gpu):
    # Independent segments in one launch equal each segment alone through the oracle (plain and
    # relative, the relative ones sharing one position table); rows between segments (gaps of 5)
    # are left as they were.
    rng = np.random.default_rng(3)
    lens = [200, 37, 129, 300, 1, 256]
    gap = 5
    starts = np.cumsum([0] + [n + gap for n in lens[:-1]]).astype(np.int32)
    rows = int(starts[-1] + lens[-1] + gap)
    for rel in (False, True):
        heads, hd = (8, 128) if rel else (4, 64)
        ch = heads * hd
        pos_t = max(lens)
        if rel:
            qkv, x, u, vb, pos = rel_inputs(rng, rows, heads, hd, O.pos_rows(pos_t))
        else:
            x = f16(qkv_like(rng, rows, ch, 3))
            pos = None
        xb = torch.from_numpy(x).cuda().half()
        pb = torch.from_numpy(pos).cuda().half() if rel else None
        o = torch.full((rows, ch), 7.0, dtype=torch.float16, device="cuda")
        gpu.pass_().attention_varlen(xb, None, pb, o, rows, torch.from_numpy(starts).cuda(),
                                     torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                     max(lens), heads, hd, pos_t)
        gpu.sync()
        got = o.float().cpu().numpy()
        for s, n in zip(starts, lens):
            if rel:
                # The shared table: row r is position pos_t + 15 - r; this segment's rows r' =
                # r - (pos_t - n) give its own pos_rows(n) table.
                p = np.ascontiguousarray(pos[pos_t - n: pos_t - n + O.pos_rows(n)])
                want = O.relative_attention(np.ascontiguousarray(qkv[s:s + n]).ravel(), p.ravel(),
                                            u, vb, n, heads, ch)
            else:
                seg = x[s:s + n]
                want = O.attention(np.ascontiguousarray(seg.ravel()), 3 * ch,
                                   np.ascontiguousarray(seg.ravel()[2 * ch:]), 3 * ch, n, heads, ch)
            check(got[s:s + n], want)
        inside = np.zeros(rows, dtype=bool)
        for s, n in zip(starts, lens):
            inside[s:s + n] = True
        assert np.all(got[~inside] == 7.0), "rows outside the segments were written"


@pytest.mark.parametrize("ty", [O.TY_F16, O.TY_Q8_0])
def test_layer_level_ii(gpu, ty):
    # A Whisper-shaped layer (C2 weights f16) and a Parakeet-shaped one (C5 weights Q8_0): the
    # oracle's GEMM rounds a and W to f16 (its f16 path, as the reference GPU GEMM).
    from wavo_b200 import GGML_F16, GGML_Q8_0
    O.set_vnni(0)
    try:
        rng = np.random.default_rng(11)
        t, heads, hd = (1500, 20, 64) if ty == O.TY_F16 else (300, 8, 128)
        d = heads * hd
        y = rng.standard_normal((t, d)).astype(np.float32)
        wq = (rng.standard_normal((3 * d, d)) * 0.02).astype(np.float32)
        wo = (rng.standard_normal((d, d)) * 0.02).astype(np.float32)
        bq = np.concatenate([rng.standard_normal(d) * 0.02, np.zeros(d),
                             rng.standard_normal(d) * 0.02]).astype(np.float32)
        bo = (rng.standard_normal(d) * 0.02).astype(np.float32)
        if ty == O.TY_F16:
            dq, do_, gty = wq.astype(np.float16).tobytes(), wo.astype(np.float16).tobytes(), GGML_F16
        else:
            dq, do_, gty = O.q8_0_bytes(wq), O.q8_0_bytes(wo), GGML_Q8_0
        lq, lo = gpu.linear(gty, 3 * d, d, dq, bq), gpu.linear(gty, d, d, do_, bo)
        yb = torch.from_numpy(y).cuda()
        qkv = torch.zeros(t, 3 * d, dtype=torch.float16, device="cuda")
        o = torch.zeros(t, d, dtype=torch.float16, device="cuda")
        x = torch.ones(t, d, device="cuda")
        p = gpu.pass_()
        p.gemm(yb, lq, qkv, t, "bias")
        p.attention(qkv, None, None, o, t, heads, hd)
        p.gemm(o, lo, x, t, "residual", 1.0)
        gpu.sync()
        ref_qkv = O.Linear(ty, 3 * d, d, dq, bq).gemm(y.ravel(), t)
        r16 = f16(ref_qkv)
        ref_o = O.attention(r16, 3 * d, np.ascontiguousarray(r16[2 * d:]), 3 * d, t, heads, d)
        want = np.ones(t * d, np.float32)
        O.Linear(ty, d, d, do_, bo).gemm(np.ascontiguousarray(ref_o.ravel()), t, want, "residual",
                                         1.0)
        check(x.cpu().numpy(), want)
    finally:
        O.set_vnni(-1)


@pytest.mark.parametrize("hd,heads,neox,lens,pos", [
    (48, 4, True, [37, 129, 300], 0),     # C3's heads (GigaAM: 16 x 48, NEOX, base 10000)
    (64, 3, True, [200, 5], 0),
    (64, 2, False, [70, 129], 7),        # adjacent pairs, table rows from 7
    (128, 2, True, [150, 64], 0),
    (16, 2, True, [33], 0),
    (32, 2, False, [50, 257], 0),
])
def test_rotary_attention_fused(gpu, hd, heads, neox, lens, pos):
    # Rotary positions inside the attention kernel against the oracle's rope (src/cpu/ops.rs:339-355)
    # then attention (ops.rs:184-221) per segment; the rows in memory stay unrotated.
    from wavo_b200 import _lib as L
    from wavo_b200.blocks import Segments, rope_table
    d = heads * hd
    rng = np.random.default_rng(hd + heads + len(lens))
    segs = Segments(lens, "cuda")
    x = f16(qkv_like(rng, segs.rows, d, 3))
    table = rope_table(pos + max(lens), hd, 10000.0)
    qkv = torch.from_numpy(x).to("cuda", torch.float16)
    before = qkv.clone()
    o = torch.zeros(segs.rows, d, dtype=torch.float32, device="cuda")
    gpu.pass_().attention_rope_varlen(qkv, o, segs.rows, segs.start_t, segs.len_t, segs.max_len,
                                      heads, hd, torch.from_numpy(table).cuda(), hd, neox, pos)
    gpu.sync()
    assert torch.equal(qkv, before)
    got = o.cpu().numpy()
    for st, n in zip(segs.starts, lens):
        q = np.ascontiguousarray(x[st:st + n].copy())
        O.rope(q, np.ascontiguousarray(table[pos:pos + n]), n, heads, hd, hd, neox)
        q = f16(q)  # the kernel rotates the f16 tiles and rounds the result to f16
        q = q.ravel()
        want = O.attention(q, 3 * d, np.ascontiguousarray(q[2 * d:]), 3 * d, n, heads, d)
        check(got[st:st + n], want)
    # Shapes the kernel cannot rotate in its tiles are refused, not computed another way.
    lib = L.lib()
    st = lib.wavo_attention_rope_varlen(gpu.ctx, qkv.data_ptr(), o.data_ptr(), segs.rows,
                                        segs.start_t.data_ptr(), segs.len_t.data_ptr(), len(lens),
                                        segs.max_len, heads, hd, table.ctypes.data, 1, pos, hd,
                                        int(neox), L.F32)
    assert st == L.EINVAL  # a table shorter than the segments
