"""Weights streamed from a GGUF file to the device (`wavo_linear_from_gguf`, the reference's
`Gpu::linear` over file tensors, src/gpu/mod.rs:758-827): the same layer, bit for bit, as
`wavo_linear_create` on the same bytes, for F32 / F16 / Q8_0, stacked tensors, biases with dual
outputs, and a layer larger than one streamed piece."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from wavo_b200 import _lib as L
from wavo_b200 import gguf as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    from wavo_b200.gpu import Gpu
    g = Gpu(0)
    yield g
    g.sync()
    g.close()


def _bytes(ty, w):
    if ty == G.TY_F32:
        return w.astype(np.float32).tobytes()
    if ty == G.TY_F16:
        return w.astype(np.float16).tobytes()
    return G.q8_0_blocks(w)


def _same(got, want):
    """The GEMM outputs (deterministic) bit for bit; the gemv's last (the CUDA-core form for F32 and
    Q8_0 weights adds its k-splits with atomics, in no fixed order) to f32 rounding."""
    for g_, w_ in zip(got[:-1], want[:-1]):
        np.testing.assert_array_equal(g_, w_)
    np.testing.assert_allclose(got[-1], want[-1], rtol=0, atol=1e-6 * max(1.0, np.abs(want[-1]).max()))


def _outputs(gpu, lin, m, a, a_rows):
    outs = []
    for e in ("bias", "gelu"):
        c = torch.zeros(m * lin.width(), device="cuda")
        gpu.pass_().gemm(a, lin, c, m, e)
        outs.append(c)
    c = torch.zeros(a_rows * lin.cols, device="cuda")
    gpu.pass_().gemv_rows(a, lin, c, a_rows, "bias")
    outs.append(c)
    gpu.sync()
    return [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("ty", [G.TY_F32, G.TY_F16, G.TY_Q8_0])
def test_linear_from_gguf_equals_create(gpu, tmp_path, ty):
    rng = np.random.default_rng(ty + 1)
    k, parts = 256, [96, 96, 70]
    ws = [(rng.standard_normal((r, k)) * 0.05).astype(np.float32) for r in parts]
    datas = [_bytes(ty, w) for w in ws]
    rows = sum(parts)
    bias = rng.standard_normal(rows + 64).astype(np.float32)  # 64 dual outputs
    path = str(tmp_path / "layer.gguf")
    G.write_gguf(path, [("general.architecture", G.STR, "test")],
                 [(f"blk.0.{n}.weight", [k, r], ty, d) for n, r, d in zip("qkv", parts, datas)])
    g = G.Gguf(path)
    names = [f"blk.0.{n}.weight" for n in "qkv"]
    a_from = gpu.linear_from_gguf(g, names, bias)
    a_create = gpu.linear(ty, rows, k, b"".join(datas), bias)
    assert (a_from.cols, a_from.dual, a_from.width()) == (a_create.cols, a_create.dual,
                                                          a_create.width())
    x = gpu.upload(O.random(300 * k, 7))
    for m, r in ((37, 5), (300, 32)):
        _same(_outputs(gpu, a_from, m, x, r), _outputs(gpu, a_create, m, x, r))
    if ty == G.TY_Q8_0:
        old = gpu.set_q8_gemm(L.Q8_PROLOGUE)
        try:
            _same(_outputs(gpu, a_from, 300, x, 32), _outputs(gpu, a_create, 300, x, 32))
        finally:
            gpu.set_q8_gemm(old)
    # Against the oracle's CPU layer on the file's own values (the reference's tolerance).
    want = O.Linear(ty, rows, k, b"".join(datas), bias[:rows]).gemv(
        np.ascontiguousarray(O.random(300 * k, 7)[:k]))[:rows]
    got = _outputs(gpu, a_from, 1, x, 1)[2][:rows]
    assert np.abs(got - want).max() <= 2e-5 * max(1.0, np.abs(want).max())
    g.close()


def test_linear_from_gguf_streams_many_pieces(gpu, tmp_path):
    # 8192 x 1024 Q8_0 weights: 8.9 MB of blocks, more than two of the streamed pieces.
    rng = np.random.default_rng(5)
    n, k = 8192, 1024
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    data = G.q8_0_blocks(w)
    path = str(tmp_path / "big.gguf")
    G.write_gguf(path, [], [("w", [k, n], G.TY_Q8_0, data)], alignment=64)
    g = G.Gguf(path)
    a_from = gpu.linear_from_gguf(g, ["w"])
    a_create = gpu.linear(G.TY_Q8_0, n, k, data)
    x = gpu.upload(O.random(64 * k, 9))
    _same(_outputs(gpu, a_from, 64, x, 8), _outputs(gpu, a_create, 64, x, 8))
    g.close()


def test_linear_from_gguf_rejects(gpu, tmp_path):
    path = str(tmp_path / "bad.gguf")
    G.write_gguf(path, [], [("a", [64, 8], G.TY_F16, bytes(64 * 8 * 2)),
                            ("b", [32, 8], G.TY_F16, bytes(32 * 8 * 2)),
                            ("c", [48, 8], G.TY_F32, bytes(48 * 8 * 4))])
    g = G.Gguf(path)
    from wavo_b200._lib import WavoError
    with pytest.raises(WavoError, match="differ"):
        gpu.linear_from_gguf(g, ["a", "b"])
    with pytest.raises(WavoError, match="k % 32"):
        gpu.linear_from_gguf(g, ["c"])
    with pytest.raises(WavoError, match="missing tensor"):
        gpu.linear_from_gguf(g, ["zz"])
    g.close()
