"""CPU checks of the C ABI: the library loads, exports every entry point include/wavo_cuda.h
declares, validates arguments without a GPU, and partitions segments deterministically."""

import ctypes
import subprocess

import numpy as np
import pytest
import torch

from wavo_b200 import _lib as L


def test_library_exports_every_header_symbol():
    lib = L.lib()
    declared = L.header_symbols()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", L.SO], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported
    assert sorted(L.SIGNATURES) == declared


def test_build_targets_sm100a_only():
    from wavo_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert build.up_to_date(), "libwavo_cuda.so is older than its sources"


def test_null_context_is_rejected():
    lib = L.lib()
    assert lib.wavo_sync(None, 0) == L.EINVAL
    assert lib.wavo_gemm(None, None, 0, 0, None, None, 0, 0, 1, 0, 1.0) == L.EINVAL
    assert lib.wavo_attention(None, None, None, None, None, 1, 1, 64, 0) == L.EINVAL
    assert lib.wavo_attend(None, None, None, None, None, 1, 1, 1, 64) == L.EINVAL
    assert lib.wavo_pack(None, None, 0, 0, None, 1, 2, 1, 0) == L.EINVAL


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU path")
def test_create_without_a_gpu_fails_cleanly():
    lib = L.lib()
    ctx = ctypes.c_void_p()
    st = lib.wavo_create(0, ctypes.byref(ctx))
    assert st in (L.EUNSUPPORTED, L.ECUDA)
    assert not ctx.value
    assert lib.wavo_last_error(None)


def test_pos_rows_and_attend_len():
    lib = L.lib()
    for t in (1, 138, 1500):
        assert lib.wavo_pos_rows(t) == 2 * t + 15
    # one split of 1024 keys per (head), hd + 2 floats each
    assert lib.wavo_attend_len(1500, 20, 64) == 2 * 20 * 66
    assert lib.wavo_attend_len(224, 20, 64) == 1 * 20 * 66


def lpt_reference(costs, parts):
    order = sorted(range(len(costs)), key=lambda i: -costs[i])
    load = [0] * parts
    out = [0] * len(costs)
    for i in order:
        p = min(range(parts), key=lambda j: (load[j], j))
        out[i] = p
        load[p] += costs[i]
    return out


@pytest.mark.parametrize("parts", [1, 2, 4, 8])
def test_partition_lpt(parts):
    from wavo_b200.gpu import partition_lpt
    rng = np.random.default_rng(5)
    lens = rng.integers(120, 301, 400)
    costs = [int(24 * (6 * t * t * 1024 + 10 * t * 1024 * 1024)) for t in lens]
    got = partition_lpt(costs, parts)
    assert got == lpt_reference(costs, parts)
    loads = np.zeros(parts)
    for c, p in zip(costs, got):
        loads[p] += c
    assert loads.max() / loads.mean() < 1.02


def test_context_free_errors_are_per_thread():
    # Two threads fail context-free calls (argument errors, returned before any CUDA call) with
    # different messages and read wavo_last_error(NULL) many times: each thread reads its own
    # message, never the other thread's or a freed one.
    import threading

    lib = L.lib()
    bad = {}

    def worker(tag, heads):
        for _ in range(2000):
            # hd 3 is odd: rejected with the thread's own head count in the message.
            st = lib.wavo_attend_batch_noalloc(1, 0, 1, 0, 1, 0, 10, 10, heads, 3, 1, None)
            msg = lib.wavo_last_error(None).decode()
            if st != L.EINVAL or f"heads {heads} of 3" not in msg:
                bad[tag] = msg
                return

    ts = [threading.Thread(target=worker, args=(i, h)) for i, h in enumerate((7, 11))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not bad, bad
