"""Parity at the shapes the bench times, against the CPU oracle (the reference's src/cpu path
restated), within the BASELINE tolerance (max-abs 2e-3, relative-L2 1e-3):

- C5: a Parakeet rel-pos attention layer at its own width (d 1024, 8 heads of 128) with GGUF
  Q8_0 weights of the bench's distribution, over segments of C5's seeded lengths packed into one
  varlen launch, against the oracle's layer (Q8_0 GEMM, relative_attention, output GEMM) in both
  of the reference's GEMM paths: the i16 VNNI path it takes on CPUs with AVX-VNNI
  (src/cpu/gemm.rs:129-161) and its f16-rounded f32 path (gemm.rs:163);
- C4: decoder attention of a batch of 32 segments, 20 heads of 64, over the 1500-frame cross
  cache and over self caches of 448 positions at steps 0, 127 and 223, against the oracle's
  attend (src/cpu/ops.rs:300-337), through wavo_attend_batch and wavo_attend_batch_noalloc.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-3, 1e-3


def errors(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return (float(np.abs(got - want).max()),
            float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)))


def check(got, want, what=""):
    err, rel = errors(got, want)
    assert err <= MAX_ABS and rel <= REL_L2, f"{what}: max-abs {err:.3g}, rel-L2 {rel:.3g}"


@pytest.fixture(scope="module")
def gpu():
    from wavo_b200.gpu import Gpu
    g = Gpu(0)
    yield g
    g.sync()
    g.close()


def q8_0_weights(rng, rows, k):
    """GGUF Q8_0 bytes as the bench draws them: int8 ~U[-127,127], f16 scale ~|N(0,0.02)|/127."""
    nb = rows * k // 32
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * 0.02 / 127).astype(np.float16)
    out = np.empty((nb, 34), np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def c5_lengths():
    """Segments of C5's seeded list (400 x U[120,300], seed 5000): its first six, plus its
    shortest and longest."""
    lens = np.random.default_rng(5000).integers(120, 301, size=400).tolist()
    return lens[:6] + [min(lens), max(lens)]


@pytest.fixture(scope="module")
def c5_layer(gpu):
    from wavo_b200 import GGML_Q8_0
    from wavo_b200.blocks import RelPosAttention, Segments, rel_positions
    d, heads = 1024, 8
    rng = np.random.default_rng(5001)
    wq, wp, wo = q8_0_weights(rng, 3 * d, d), q8_0_weights(rng, d, d), q8_0_weights(rng, d, d)
    u = rng.standard_normal(d, dtype=np.float32) * 0.02
    v = rng.standard_normal(d, dtype=np.float32) * 0.02
    lens = c5_lengths()
    blk = RelPosAttention(gpu, GGML_Q8_0, d, heads, wq, wp, wo, u, v)
    segs = Segments(lens, "cuda")
    t_pos = max(lens)
    table = rel_positions(d, t_pos + 15, 2 * t_pos + 15)
    y = rng.standard_normal((segs.rows, d), dtype=np.float32)
    x = torch.zeros(segs.rows, d, device="cuda")  # the layer's output alone: the strictest check
    s = blk.scratch(segs.rows, t_pos)
    blk.record(gpu.pass_(), gpu.upload(y), x, segs, gpu.upload(table), t_pos, s)
    gpu.sync()
    return dict(d=d, heads=heads, wq=wq, wp=wp, wo=wo, u=u, v=v, lens=lens, starts=segs.starts,
                y=y, got=x.cpu().numpy())


@pytest.mark.parametrize("vnni", [1, 0], ids=["i16-vnni", "f16"])
def test_relpos_layer_c5_width_q8(c5_layer, vnni):
    L = c5_layer
    d, heads = L["d"], L["heads"]
    O.set_vnni(vnni)
    try:
        lq = O.Linear(O.TY_Q8_0, 3 * d, d, L["wq"])
        lp = O.Linear(O.TY_Q8_0, d, d, L["wp"])
        lo = O.Linear(O.TY_Q8_0, d, d, L["wo"])
        for st, n in zip(L["starts"], L["lens"]):
            # src/cpu/conformer.rs:169-186: qkv, the segment's own position table through
            # linear_pos, relative_attention with u and v, the output projection into x.
            y = np.ascontiguousarray(L["y"][st:st + n]).ravel()
            qkv = lq.gemm(y, n)
            tab = O.rel_positions(d, n + 15, O.pos_rows(n))
            pos = lp.gemm(np.ascontiguousarray(tab.ravel()), O.pos_rows(n))
            o = O.relative_attention(qkv, pos, L["u"], L["v"], n, heads, d)
            want = np.zeros(n * d, np.float32)
            lo.gemm(np.ascontiguousarray(o.ravel()), n, want, "residual", 1.0)
            check(L["got"][st:st + n], want, f"segment of {n} frames")
    finally:
        O.set_vnni(-1)


# ---- C4: decoder attention at the bench's shape ------------------------------------------------

D4, H4, HD4, B4 = 1280, 20, 64, 32


def _caches(gpu, n_pos, cols, seed):
    """B4 caches of `cols` positions whose first n_pos hold K/V rows ~N(0,1) (f32), packed on the
    GPU in the reference's layout (wavo_pack_batch) and on the host in the oracle's."""
    rng = np.random.default_rng(seed)
    words = D4 * cols
    cache = torch.zeros(B4, words, dtype=torch.int32, device="cuda")
    host = []
    for b in range(B4):
        kv = rng.standard_normal((n_pos, 2 * D4), dtype=np.float32)
        xb = gpu.upload(kv)
        gpu.pass_().pack_batch(xb, (0, 2 * D4), 0, cache[b], 0, n_pos, D4, (cols, 0), 1)
        oc = np.zeros(cols * 2 * D4, np.float32)
        O.pack_cache(np.ascontiguousarray(kv.ravel()), n_pos, D4, HD4, oc, cols, 0)
        host.append(oc)
    gpu.sync()
    return cache, host


@pytest.fixture(scope="module")
def c4_cross(gpu):
    return _caches(gpu, 1500, 1500, 4001)


@pytest.fixture(scope="module")
def c4_self(gpu):
    # The self cache at step 223 holds 224 positions of its 448; earlier steps read a prefix.
    return _caches(gpu, 224, 448, 4002)


def _attend_both(gpu, cache, n, cols, seed):
    """The batch through wavo_attend_batch and wavo_attend_batch_noalloc, and q."""
    from wavo_b200 import _lib
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B4, D4), dtype=np.float32)
    qb = gpu.upload(q)
    part = torch.empty(B4 * _lib.lib().wavo_attend_len(n, H4, HD4) + 1, device="cuda")
    o = torch.full((B4, D4), float("nan"), device="cuda")
    gpu.pass_().attend_batch(qb, D4, cache, D4 * cols, part, o, D4, n, cols, H4, HD4, B4)
    o2 = torch.full((B4, D4), float("nan"), device="cuda")
    stream = torch.cuda.current_stream()
    _lib.check(_lib.lib().wavo_attend_batch_noalloc(
        qb.data_ptr(), D4, cache.data_ptr(), D4 * cols, o2.data_ptr(), D4, n, cols, H4, HD4, B4,
        ctypes.c_void_p(stream.cuda_stream)), None)
    gpu.sync()
    torch.cuda.synchronize()
    return q, o.cpu().numpy(), o2.cpu().numpy()


def test_attend_batch_c4_cross(gpu, c4_cross):
    # 1500 keys: two 1024-key parts a head, combined.
    cache, host = c4_cross
    q, got, got2 = _attend_both(gpu, cache, 1500, 1500, 7)
    for b in range(B4):
        want = O.attend(np.ascontiguousarray(q[b]), host[b], 1500, 1500, H4, HD4)
        check(got[b], want, f"segment {b}")
        check(got2[b], want, f"segment {b} (no-alloc)")


@pytest.mark.parametrize("step", [0, 127, 223])
def test_attend_batch_c4_self(gpu, c4_self, step):
    # step + 1 keys of a 448-position cache: one part a head (the four-group path up to 256 keys).
    cache, host = c4_self
    n = step + 1
    q, got, got2 = _attend_both(gpu, cache, n, 448, 100 + step)
    for b in range(B4):
        want = O.attend(np.ascontiguousarray(q[b]), host[b], 448, n, H4, HD4)
        check(got[b], want, f"segment {b}")
        check(got2[b], want, f"segment {b} (no-alloc)")
