"""The GGUF reader (src/gguf.rs) through the C ABI, on the CPU: the reference's own reader test on
its sample file (src/gguf.rs:382-490, restated as tests/golden/gguf_sample.gguf by
tests/golden/make_gguf_sample.py), then files written by `wavo_b200.gguf.write_gguf`."""

import os

import numpy as np
import pytest

from wavo_b200 import gguf as G

SAMPLE = os.path.join(os.path.dirname(__file__), "golden", "gguf_sample.gguf")


def test_golden_sample_is_the_reference_test_file():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_gguf_sample", os.path.join(os.path.dirname(__file__), "golden", "make_gguf_sample.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with open(SAMPLE, "rb") as fh:
        assert fh.read() == mod.sample()


def test_reads_metadata_and_tensors():
    # src/gguf.rs:447-480 `reads_metadata_and_tensors`, assertion for assertion.
    g = G.Gguf(SAMPLE)
    assert g.get("a.n", "u32") == 7
    assert g.get("a.n", "i32") == 7
    with pytest.raises(G.GgufError):
        g.get("missing", "u32")
    with pytest.raises(G.GgufError):
        g.get("a.n", str)
    assert g.array("a.tokens", str) == ["▁x", "y"]
    assert g.get("a.flag", bool) is True
    assert g.optional("a.flag", bool) is True
    assert g.optional("missing", bool) is None
    with pytest.raises(G.GgufError):
        g.optional("a.flag", str)
    assert g.get("a.left", "i32") == -1
    with pytest.raises(G.GgufError):
        g.get("a.left", "u32")
    assert g.array("a.durations", "i32") == [0, 2, -4]
    with pytest.raises(G.GgufError):
        g.array("a.durations", "u32")
    assert g.optional_array("a.durations", "i32") == [0, 2, -4]
    assert g.optional_array("missing", "i32") == []
    with pytest.raises(G.GgufError):
        g.optional_array("a.durations", "u32")
    assert np.float32(g.get("a.alpha", float)) == np.float32(0.97)

    g.tensor("w", [2, 1])
    assert g.to_f32("w").tolist() == [1.5, -2.0]
    with pytest.raises(G.GgufError):
        g.tensor("w", [1, 2])

    ty, nbytes = g.tensor("q", [32])
    assert ty == G.TY_Q8_0 and nbytes == 34
    assert g.to_f32("q").tolist() == [(i - 16) * 0.5 for i in range(32)]
    # Tensor::read in pieces of 16: (0, 16), (16, 16), (32, 2).
    whole = g.read("q")
    assert g.read("q", 0, 16) + g.read("q", 16, 16) + g.read("q", 32, 2) == whole
    with pytest.raises(G.GgufError):
        g.read("q", 32, 3)
    assert g.names() == ["w", "q"]


def test_rejects_truncated_files(tmp_path):
    # src/gguf.rs:483-489 `rejects_truncated_files`.
    with open(SAMPLE, "rb") as fh:
        data = fh.read()
    p = tmp_path / "cut.gguf"
    p.write_bytes(data[:-1])
    with pytest.raises(G.GgufError, match="out of file bounds"):
        G.Gguf(str(p))
    for cut in (3, 10, 40, 200):
        p.write_bytes(data[:cut])
        with pytest.raises(G.GgufError):
            G.Gguf(str(p))


def test_rejects_other_files(tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(G.GgufError, match="not a GGUF file"):
        G.Gguf(str(p))
    with open(SAMPLE, "rb") as fh:
        data = bytearray(fh.read())
    data[4] = 2  # version 2
    p.write_bytes(bytes(data))
    with pytest.raises(G.GgufError, match="version 2"):
        G.Gguf(str(p))
    with pytest.raises(G.GgufError, match="cannot open"):
        G.Gguf(str(tmp_path / "none.gguf"))


def test_written_files_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    w32 = rng.standard_normal(96 * 64).astype(np.float32)
    w16 = rng.standard_normal(70 * 64).astype(np.float16)
    wq = rng.standard_normal(40 * 128).astype(np.float32)
    meta = [("general.architecture", G.STR, "whisper"), ("x.count", G.U64, 2**40 + 3),
            ("x.small", G.I8, -5), ("x.scale", G.F64, 0.125), ("x.ok", G.BOOL, False),
            ("x.names", G.ARRAY, (G.STR, ["a", "bé", ""])), ("x.ids", G.ARRAY, (G.U16, [1, 65535])),
            ("x.nested", G.ARRAY, (G.ARRAY, [(G.I32, [1, 2]), (G.I32, [])]))]
    tensors = [("t.f32", [64, 96], G.TY_F32, w32.tobytes()), ("t.f16", [64, 70], G.TY_F16, w16.tobytes()),
               ("t.q8", [128, 40], G.TY_Q8_0, G.q8_0_blocks(wq))]
    for align in (32, 64, 256):
        p = str(tmp_path / f"r{align}.gguf")
        G.write_gguf(p, meta, tensors, alignment=align)
        g = G.Gguf(p)
        assert g.get("general.architecture", str) == "whisper"
        assert g.get("x.count", int) == 2**40 + 3 and g.get("x.small", int) == -5
        assert g.get("x.scale", float) == 0.125 and g.get("x.ok", bool) is False
        assert g.array("x.names", str) == ["a", "bé", ""] and g.array("x.ids", int) == [1, 65535]
        with pytest.raises(G.GgufError):
            g.array("x.nested", int)
        assert g.dims("t.f32") == [64, 96] and g.tensor("t.f16") == (G.TY_F16, 70 * 64 * 2)
        assert np.array_equal(g.to_f32("t.f32"), w32)
        assert np.array_equal(g.to_f32("t.f16"), w16.astype(np.float32))
        assert g.tensor("t.q8") == (G.TY_Q8_0, 40 * 128 // 32 * 34)
        assert np.abs(g.to_f32("t.q8") - wq).max() <= np.abs(wq).max() / 127
        g.close()


def test_large_reads_in_parallel_parts_and_clean_exit(tmp_path):
    # A tensor over 1 MiB is read as several ranges by the library's reader threads; the bytes must
    # be the file's, and a process that used them must still exit on its own.
    import subprocess
    import sys
    rng = np.random.default_rng(3)
    w = rng.standard_normal(3 * 2**20 // 4 + 17 * 32).astype(np.float32)
    p = str(tmp_path / "big.gguf")
    G.write_gguf(p, [], [("big", [32, w.size // 32], G.TY_F32, w.tobytes())])
    g = G.Gguf(p)
    assert g.read("big") == w.tobytes()
    assert g.read("big", 1000, 2_500_000) == w.tobytes()[1000:2_501_000]
    g.close()
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from wavo_b200 import gguf as G\n"
            "g = G.Gguf(%r)\n"
            "assert len(g.read('big')) == %d\n") % (os.path.dirname(os.path.dirname(__file__)), p,
                                                    w.size * 4)
    r = subprocess.run([sys.executable, "-c", code], timeout=120)
    assert r.returncode == 0
