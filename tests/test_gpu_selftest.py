"""Device building blocks the kernels rest on, through the C ABI:

- the bounded mbarrier wait: a wait that nothing ends gives up after its limit, the kernel
  returns, wavo_sync reports WAVO_EDEVICE (the reference surfaces device failures at completion,
  src/gpu/mod.rs:969-1003) and the context keeps working;
- the FMA-pipe 2^x of the softmax against exact values: relative error at most 7.8e-6 over the
  inputs the softmax gives it ([-125, 8]).
"""

import numpy as np
import pytest
import torch

from wavo_b200 import _lib as L

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    from wavo_b200.gpu import Gpu
    g = Gpu(0)
    yield g
    g.sync()
    g.close()


def test_wait_timeout_reaches_sync_and_the_context_recovers(gpu):
    lib = L.lib()
    # ~50 us at the B200's clocks: the wait gives up, the kernel returns.
    L.check(lib.wavo_selftest_wait_timeout(gpu.ctx, 100_000), gpu.ctx)
    st = lib.wavo_sync(gpu.ctx, 10_000)
    assert st == L.EDEVICE, L.STATUS.get(st, st)
    msg = lib.wavo_last_error(gpu.ctx).decode()
    assert "bounded wait gave up" in msg and "softmax" in msg, msg
    # The error word was cleared and the context still runs work.
    x = torch.linspace(-3, 3, 4096, device="cuda")
    y = torch.empty_like(x)
    L.check(lib.wavo_selftest_exp2(gpu.ctx, x.data_ptr(), y.data_ptr(), x.numel()), gpu.ctx)
    gpu.sync()
    np.testing.assert_allclose(y.cpu().numpy(), np.exp2(x.cpu().numpy()), rtol=1e-5)
    # Out-of-range limits are argument errors.
    assert lib.wavo_selftest_wait_timeout(gpu.ctx, 0) == L.EINVAL


def test_exp2_polynomial_error_bound(gpu):
    lib = L.lib()
    x = np.linspace(-125.0, 8.0, 20_000_001, dtype=np.float64).astype(np.float32)
    # The points where the rounding to n = round(x) switches, and values just either side.
    half = (np.arange(-125, 8) + 0.5).astype(np.float32)
    x = np.concatenate([x, half, np.nextafter(half, np.float32(-np.inf)),
                        np.nextafter(half, np.float32(np.inf))])
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    L.check(lib.wavo_selftest_exp2(gpu.ctx, xd.data_ptr(), yd.data_ptr(), x.size), gpu.ctx)
    gpu.sync()
    y = yd.cpu().numpy().astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(y - want) / want
    assert rel.max() <= 7.8e-6, f"max relative error {rel.max():.3g} at x = {x[rel.argmax()]}"
    # Below the range the polynomial saturates at 2^-125.
    lo = torch.tensor([-126.0, -200.0, -1e30], device="cuda")
    out = torch.empty_like(lo)
    L.check(lib.wavo_selftest_exp2(gpu.ctx, lo.data_ptr(), out.data_ptr(), 3), gpu.ctx)
    gpu.sync()
    np.testing.assert_allclose(out.cpu().numpy(), np.full(3, 2.0 ** -125), rtol=1e-5)
