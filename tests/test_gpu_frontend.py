"""The Parakeet log-mel frontend on the device (src/parakeet/frontend.rs) through the C ABI, against
the oracle's restatement of the reference (CPU): the log-mel of every frame, frame ranges, the
normalised features, short and silent inputs; the reference's tolerance (max-abs 2e-3, rel-L2
1e-3), and the measured error is far below it (the spectrum is the reference's bit for bit)."""

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


def speech_like(seconds: float, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    n = int(seconds * 16000)
    t = np.arange(n) / 16000.0
    x = 0.05 * rng.standard_normal(n)
    for f in (180.0, 440.0, 1250.0, 3300.0):
        x += 0.2 * np.sin(2 * np.pi * f * t + rng.uniform(0, 6)) * (0.5 + 0.5 * np.sin(2 * np.pi * 1.3 * t))
    return x.astype(np.float32)


def close(got, want):
    err = np.abs(got.astype(np.float64) - want)
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert err.max() <= 2e-3 and rel <= 1e-3, (err.max(), rel)
    return err.max()


def gpu_log_mel(gpu, pcm, f0, f1):
    p = torch.from_numpy(pcm).cuda()
    mel = torch.zeros(f1 - f0, 128, device="cuda")
    gpu.log_mel(p, f0, f1, mel)
    gpu.sync()
    return mel.cpu().numpy()


@pytest.mark.parametrize("seconds", [1.0, 7.3])
def test_log_mel_matches_oracle(gpu, seconds):
    pcm = speech_like(seconds, 1)
    frames = pcm.size // 160 + 1
    got = gpu_log_mel(gpu, pcm, 0, frames)
    want = O.log_mel(pcm, 0, frames)
    assert close(got, want) < 1e-4
    # The spectrum is the reference's: the log-mel agrees but for the last bit of ln.
    assert (got == want).mean() > 0.5


def test_log_mel_frame_ranges(gpu):
    # src/parakeet/frontend.rs:152-161 `frame_ranges` on the device.
    pcm = (np.sin(np.arange(16000, dtype=np.float32) * np.float32(0.01)) * np.float32(0.5)).astype(np.float32)
    whole = gpu_log_mel(gpu, pcm, 0, 101)
    close(whole, O.log_mel(pcm, 0, 101))
    for a, b in ((0, 1), (0, 7), (3, 40), (95, 101), (100, 101)):
        np.testing.assert_array_equal(gpu_log_mel(gpu, pcm, a, b), whole[a:b])


@pytest.mark.parametrize("seconds,seed", [(0.02, 2), (3.0, 3), (75.0, 4)])
def test_mel_features_match_oracle(gpu, seconds, seed):
    pcm = speech_like(seconds, seed)
    want = O.mel_features(pcm)
    mel = torch.zeros(pcm.size // 160 + 1, 128, device="cuda")
    n = gpu.mel_features(torch.from_numpy(pcm).cuda(), mel)
    gpu.sync()
    assert n == want.shape[0]
    got = mel.cpu().numpy()[:n]
    close(got, want)
    assert (got[-1] == 0).all()


def test_mel_features_short_and_silent(gpu):
    # src/parakeet/frontend.rs:143-150 `short_input`, and silence (zero variance).
    mel = torch.full((8, 128), 7.0, device="cuda")
    assert gpu.mel_features(torch.full((319,), 0.1, device="cuda"), mel) == 0
    gpu.sync()
    assert (mel.cpu().numpy() == 7.0).all()  # nothing written
    assert gpu.mel_features(torch.full((320,), 0.1, device="cuda"), mel) == 3
    gpu.sync()
    got = mel.cpu().numpy()[:3]
    assert np.isfinite(got).all()
    close(got, O.mel_features(np.full(320, 0.1, np.float32)))
    silent = np.zeros(16000, np.float32)
    mel = torch.zeros(101, 128, device="cuda")
    assert gpu.mel_features(torch.from_numpy(silent).cuda(), mel) == 101
    gpu.sync()
    np.testing.assert_array_equal(mel.cpu().numpy(), O.mel_features(silent))


@pytest.mark.parametrize("frames,valid,seed", [(801, 801, 1), (801, 520, 2), (97, 97, 3)])
def test_subsample_matches_oracle(gpu, frames, valid, seed):
    # Parakeet's 8x conv subsampling (src/parakeet/cpu.rs:60-174) at its width (256 channels),
    # F16 pointwise and output weights, against the oracle's CPU restatement (its f16 GEMM path).
    ch, d = 256, 512
    rng = np.random.default_rng(seed)
    mel = rng.standard_normal((frames, 128)).astype(np.float32)
    taps = {k: (rng.standard_normal((9, ch)) * 0.3).astype(np.float32) for k in ("w0", "w2", "w5")}
    taps.update({k: (rng.standard_normal(ch) * 0.1).astype(np.float32) for k in ("b0", "b2", "b5")})
    w3 = (rng.standard_normal((ch, ch)) * 0.06).astype(np.float16)
    w6 = (rng.standard_normal((ch, ch)) * 0.06).astype(np.float16)
    wo = (rng.standard_normal((d, 16 * ch)) * 0.02).astype(np.float16)
    b3, b6 = (rng.standard_normal((2, ch)) * 0.1).astype(np.float32)
    bo = (rng.standard_normal(d) * 0.1).astype(np.float32)
    O.set_vnni(0)
    try:
        want = O.subsample(mel, valid, taps,
                           O.Linear(O.TY_F16, ch, ch, w3.tobytes(), b3),
                           O.Linear(O.TY_F16, ch, ch, w6.tobytes(), b6),
                           O.Linear(O.TY_F16, d, 16 * ch, wo.tobytes(), bo))
    finally:
        O.set_vnni(-1)
    l3 = gpu.linear(O.TY_F16, ch, ch, w3.tobytes(), b3)
    l6 = gpu.linear(O.TY_F16, ch, ch, w6.tobytes(), b6)
    lo = gpu.linear(O.TY_F16, d, 16 * ch, wo.tobytes(), bo)
    dt = {k: torch.from_numpy(v).cuda() for k, v in taps.items()}
    x = torch.zeros(want.shape[0], d, device="cuda")
    t = gpu.subsample(torch.from_numpy(mel).cuda(), valid, dt, l3, l6, lo, x)
    gpu.sync()
    assert t == want.shape[0]
    got = x.cpu().numpy()
    err = np.abs(got - want).max() / max(1.0, np.abs(want).max())
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 2e-3 and rel <= 1e-3, (err, rel)


def test_subsample_batch_matches_each_segment(gpu):
    # wavo_subsample_batch over ragged segments (padding rows in some, a 2-frame one, one longer
    # than the rest) against the oracle segment by segment, and against wavo_subsample per segment
    # (conv6 and the output projection run over every segment's rows at once there).
    ch, d = 256, 384
    rng = np.random.default_rng(11)
    frames = [801, 97, 2, 333, 1201, 64]
    valid = [801, 60, 2, 333, 1000, 64]
    mels = [rng.standard_normal((f, 128)).astype(np.float32) for f in frames]
    taps = {k: (rng.standard_normal((9, ch)) * 0.3).astype(np.float32) for k in ("w0", "w2", "w5")}
    taps.update({k: (rng.standard_normal(ch) * 0.1).astype(np.float32) for k in ("b0", "b2", "b5")})
    w3 = (rng.standard_normal((ch, ch)) * 0.06).astype(np.float16)
    w6 = (rng.standard_normal((ch, ch)) * 0.06).astype(np.float16)
    wo = (rng.standard_normal((d, 16 * ch)) * 0.02).astype(np.float16)
    b3, b6 = (rng.standard_normal((2, ch)) * 0.1).astype(np.float32)
    bo = (rng.standard_normal(d) * 0.1).astype(np.float32)
    O.set_vnni(0)
    try:
        wants = [O.subsample(m, v, taps, O.Linear(O.TY_F16, ch, ch, w3.tobytes(), b3),
                             O.Linear(O.TY_F16, ch, ch, w6.tobytes(), b6),
                             O.Linear(O.TY_F16, d, 16 * ch, wo.tobytes(), bo))
                 for m, v in zip(mels, valid)]
    finally:
        O.set_vnni(-1)
    l3 = gpu.linear(O.TY_F16, ch, ch, w3.tobytes(), b3)
    l6 = gpu.linear(O.TY_F16, ch, ch, w6.tobytes(), b6)
    lo = gpu.linear(O.TY_F16, d, 16 * ch, wo.tobytes(), bo)
    dt = {k: torch.from_numpy(v).cuda() for k, v in taps.items()}
    rows = sum(w.shape[0] for w in wants)
    x = torch.full((rows, d), float("nan"), device="cuda")
    ts = gpu.subsample_batch(torch.from_numpy(np.concatenate(mels)).cuda(), frames, valid, dt,
                             l3, l6, lo, x)
    gpu.sync()
    assert ts == [w.shape[0] for w in wants]
    got = x.cpu().numpy()
    r = 0
    for m, v, want in zip(mels, valid, wants):
        part = got[r:r + want.shape[0]]
        err = np.abs(part - want).max() / max(1.0, np.abs(want).max())
        rel = np.linalg.norm(part - want) / np.linalg.norm(want)
        assert err <= 2e-3 and rel <= 1e-3, (err, rel)
        one = torch.zeros(want.shape[0], d, device="cuda")
        gpu.subsample(torch.from_numpy(m).cuda(), v, dt, l3, l6, lo, one)
        gpu.sync()
        np.testing.assert_allclose(part, one.cpu().numpy(), rtol=0, atol=1e-5 * max(1.0, np.abs(want).max()))
        r += want.shape[0]


def test_subsample_batch_rejects_bad_segments(gpu):
    from wavo_b200 import _lib as L
    ch = 256
    rng = np.random.default_rng(12)
    taps = {k: torch.from_numpy((rng.standard_normal((9, ch)) * 0.3).astype(np.float32)).cuda()
            for k in ("w0", "w2", "w5")}
    taps.update({k: torch.zeros(ch, device="cuda") for k in ("b0", "b2", "b5")})
    w = np.zeros((ch, ch), np.float16)
    l3 = gpu.linear(O.TY_F16, ch, ch, w.tobytes(), np.zeros(ch, np.float32))
    lo = gpu.linear(O.TY_F16, 64, 16 * ch, np.zeros((64, 16 * ch), np.float16).tobytes(),
                    np.zeros(64, np.float32))
    mel = torch.zeros(200, 128, device="cuda")
    x = torch.zeros(64, 64, device="cuda")
    scratch = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    for frames, valid in (([100, 1], [100, 1]), ([100, 100], [100, 0]), ([100, 50], [100, 51])):
        with pytest.raises(L.WavoError):
            gpu.subsample_batch(mel, frames, valid, taps, l3, l3, lo, x, scratch)
    assert gpu.subsample_batch(mel, [], [], taps, l3, l3, lo, x, scratch) == []
