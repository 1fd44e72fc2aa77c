"""wavo_attend_batch_noalloc (no reference counterpart): the decoder attention with its split
partials in the library's fixed device array, against wavo_attend_batch with a caller-provided
`part` buffer (the entry point of Pass::attend, src/gpu/mod.rs:1485-1505) and against the CPU
oracle's attend (src/cpu/ops.rs:300-337), through the C ABI. Collected last so that it also runs
after every other GPU test in one process."""

import ctypes

import numpy as np
import pytest
import torch

from wavo_b200 import _lib as L


def oracle_cache(kv_words: np.ndarray, d: int, cols: int, heads: int, hd: int) -> np.ndarray:
    """The cache of one segment in the oracle's layout ([K heads][cols][hd] then the same for V,
    f32) from the GPU layout (f16 pairs in 32-bit words: K transposed, pair i of position j at
    word i·cols + j, then V by position at word d/2·cols + j·d/2 + i)."""
    h = kv_words.view(np.float16).astype(np.float32)
    k = h[:d * cols].reshape(d // 2, cols, 2).transpose(1, 0, 2).reshape(cols, d)
    v = h[d * cols:2 * d * cols].reshape(cols, d)
    to_heads = lambda m: m.reshape(cols, heads, hd).transpose(1, 0, 2).ravel()  # noqa: E731
    return np.ascontiguousarray(np.concatenate([to_heads(k), to_heads(v)]))


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def test_noalloc_rejects_oversize_partials():
    # Checked before any CUDA call: batch·heads·splits·(hd+2) above the fixed array is an error
    # with a reason, not a launch.
    lib = L.lib()
    n, heads, hd = 3000, 20, 64          # 3 splits of 1024 keys: 20·3·66 = 3960 floats a segment
    batch = L.WAVO_ATTEND_NOALLOC_PART_FLOATS // (heads * 3 * (hd + 2)) + 1
    st = lib.wavo_attend_batch_noalloc(1, 0, 1, 0, 1, 0, n, n, heads, hd, batch, None)
    assert st == L.EINVAL
    msg = lib.wavo_last_error(None).decode()
    assert "split the batch" in msg and str(L.WAVO_ATTEND_NOALLOC_PART_FLOATS) in msg


@pytest.mark.gpu
@pytest.mark.parametrize("n,cols,heads,hd,batch", [
    (1500, 1500, 20, 64, 4),    # Whisper cross attention over 1500 frames: 2 splits
    (2900, 3000, 6, 64, 3),     # 3 splits, the last ragged
    (37, 448, 20, 64, 5),       # one split: the output is written directly, no partials
])
def test_noalloc_matches_attend_batch(n, cols, heads, hd, batch):
    lib = L.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = ctypes.c_void_p()
    L.check(lib.wavo_create(0, ctypes.byref(ctx)), None)
    try:
        stream = torch.cuda.current_stream(dev)
        L.check(lib.wavo_set_stream(ctx, stream.cuda_stream), ctx)
        d = heads * hd
        words = d * cols                                   # one F16 cache: K^T then V, 32-bit words
        g = torch.Generator(device="cpu").manual_seed(n + cols + batch)
        part = torch.empty(batch * lib.wavo_attend_len(n, heads, hd) + 1, device=dev)
        for call in range(2):                              # two calls in a row, new inputs each
            kv = (torch.randn(batch, 2 * words, generator=g) * 0.5).half().to(dev)
            kv = kv.view(torch.int32)
            q = torch.randn(batch, d + 16, generator=g).to(dev)   # q_stride ≠ d
            want = torch.full((batch, d + 8), float("nan"), device=dev)
            got = torch.full((batch, d + 8), float("nan"), device=dev)
            L.check(lib.wavo_attend_batch(ctx, _ptr(q), d + 16, _ptr(kv), words, _ptr(part),
                                          _ptr(want), d + 8, n, cols, heads, hd, batch), ctx)
            L.check(lib.wavo_attend_batch_noalloc(_ptr(q), d + 16, _ptr(kv), words, _ptr(got),
                                                  d + 8, n, cols, heads, hd, batch,
                                                  stream.cuda_stream), None)
            L.check(lib.wavo_sync(ctx, 60000), ctx)
            torch.cuda.synchronize(dev)
            w = want[:, :d].cpu().numpy()
            o = got[:, :d].cpu().numpy()
            assert np.isfinite(w).all() and np.isfinite(o).all(), f"call {call}"
            assert np.abs(o - w).max() <= 2e-5, f"call {call}: {np.abs(o - w).max():.3g}"
            # And the oracle, within the BASELINE tolerance (max-abs 2e-3, relative-L2 1e-3).
            from oracle import oracle as O
            kv_h = kv.cpu().numpy()
            q_h = q.cpu().numpy()
            for b in range(batch):
                ref = O.attend(np.ascontiguousarray(q_h[b, :d]),
                               oracle_cache(kv_h[b], d, cols, heads, hd), cols, n, heads, hd)
                err = np.abs(o[b] - ref).max()
                rel = np.linalg.norm(o[b] - ref) / np.linalg.norm(ref)
                assert err <= 2e-3 and rel <= 1e-3, f"call {call} segment {b}: {err:.3g} {rel:.3g}"
            # The padding between rows is not written.
            assert torch.isnan(got[:, d:]).all(), f"call {call}"
    finally:
        lib.wavo_destroy(ctx)
