"""The Whisper decoder step's ends on the device, through the C ABI: the token embedding of a batch
(Pass::embed, src/gpu/mod.rs:1471-1484) and the greedy pick with the suppression lists and the
timestamp rules (src/whisper/search.rs:46-123, which the reference runs on the CPU), checked
against the reference's own search tests (search.rs:180-225) and the CPU oracle's `pick`; then a
whole greedy decode of a small Whisper-shaped decoder kept on the device against the oracle's CPU
decoder step (src/cpu/transformer.rs:226-262) and search.
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


def gpu_pick(gpu, logits, histories, suppress, begin_suppress, eot, no_ts, begin,
             max_initial=50, tokens=None):
    """One wavo_pick launch over the rows of `logits` with their histories; returns (tokens,
    logprobs, the edited logits, histories, lengths)."""
    rows, vocab = logits.shape
    hmax = max(8, max(len(h) for h in histories) + 1)
    hist = np.zeros((rows, hmax), np.int32)
    for r, h in enumerate(histories):
        hist[r, :len(h)] = h
    lg = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    hb = torch.from_numpy(hist).cuda()
    hl = torch.tensor([len(h) for h in histories], dtype=torch.int32, device="cuda")
    i32 = lambda a: torch.tensor(np.asarray(list(a) or [0], np.int32), device="cuda")  # noqa: E731
    tok = torch.tensor(np.zeros(rows, np.int32) if tokens is None else tokens, dtype=torch.int32,
                       device="cuda")
    lp = torch.zeros(rows, device="cuda")
    gpu.pass_().pick(lg, rows, vocab, hb, hl, i32(suppress), len(suppress), i32(begin_suppress),
                     len(begin_suppress), eot, no_ts, begin, max_initial, tok, lp)
    gpu.sync()
    return (tok.cpu().numpy(), lp.cpu().numpy(), lg.cpu().numpy(), hb.cpu().numpy(),
            hl.cpu().numpy())


def test_pick_reference_rules(gpu):
    # search.rs:190-208: vocabulary 20 (text 0..10, EOT 10, <|notimestamps|> 12, timestamps
    # 13..20), all logits equal; which tokens the rules leave open, four histories in one launch.
    T = 13
    hists = [[], [T, 3, T + 2], [T, 3, T + 2, T + 2], [T + 1, 3]]
    want = [range(T, 20), range(T + 2, 20), range(0, 12), range(T + 2, 20)]
    _, _, lg, _, _ = gpu_pick(gpu, np.zeros((4, 20), np.float32), hists, [], [], 10, 12, T)
    for r in range(4):
        assert list(np.isfinite(lg[r])) == [i in want[r] for i in range(20)], r


def test_pick_scripted_decode(gpu):
    # search.rs:210-225: one-hot logits that script T, 3, T + 4, EOT; the row then stays finished.
    T = 13
    one_hot = lambda i: np.array([[5.0 if j == i else 0.0 for j in range(20)]], np.float32)  # noqa: E731
    rows, hmax = 1, 8
    hist = torch.zeros(rows, hmax, dtype=torch.int32, device="cuda")
    hl = torch.zeros(rows, dtype=torch.int32, device="cuda")
    tok = torch.tensor([7], dtype=torch.int32, device="cuda")  # the prompt's last token
    lp = torch.zeros(rows, device="cuda")
    sup = torch.tensor([11], dtype=torch.int32, device="cuda")
    bsup = torch.tensor([1, 10], dtype=torch.int32, device="cuda")
    picks, lps = [], []
    for i in (T, 3, T + 4, 10, 3):
        lg = torch.from_numpy(one_hot(i)).cuda()
        gpu.pass_().pick(lg, rows, 20, hist, hl, sup, 1, bsup, 2, 10, 12, T, 50, tok, lp)
        gpu.sync()
        picks.append(int(tok[0]))
        lps.append(float(lp[0]))
    assert picks == [T, 3, T + 4, 10, 10]
    assert int(hl[0]) == 3 and hist[0, :3].tolist() == [T, 3, T + 4]
    assert -1.0 < np.mean(lps[:4]) < 0.0


@pytest.mark.parametrize("vocab,eot,no_ts,begin,rows,hmax", [
    (3000, 2500, 2503, 2504, 24, 7),         # one CTA a row
    (51866, 50257, 50364, 50365, 32, 200),   # Whisper large-v3's ids: seven CTAs a row
])
def test_pick_matches_oracle(gpu, vocab, eot, no_ts, begin, rows, hmax):
    # Random logits at a Whisper-like split (text, EOT, <|notimestamps|>, timestamps) and random
    # histories: the same token, log-probability and edited logits as the oracle's pick.
    rng = np.random.default_rng(3)
    hists = []
    for r in range(rows):
        n = int(rng.integers(0, hmax))
        p_ts = 0.0 if r % 4 == 1 else 0.5  # some histories without a timestamp
        h = [int(rng.integers(begin, vocab)) if rng.random() < p_ts else int(rng.integers(0, eot))
             for _ in range(n)]
        hists.append(h)
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    logits[::3, begin:] += 4.0  # rows where the timestamps' mass wins
    suppress, bsup = [2501, 2502, 17, 400], [220, eot]
    tok, lp, lg, hist, hl = gpu_pick(gpu, logits, hists, suppress, bsup, eot, no_ts, begin)
    for r in range(rows):
        ol = logits[r].copy()
        t, l = O.pick(ol, hists[r], suppress, bsup, eot, no_ts, begin)
        assert tok[r] == t, (r, tok[r], t)
        assert abs(lp[r] - l) <= 1e-5 * max(1.0, abs(l)), (r, lp[r], l)
        np.testing.assert_array_equal(np.isfinite(lg[r]), np.isfinite(ol))
        want_h = hists[r] + ([t] if t != eot else [])
        assert hl[r] == len(want_h) and list(hist[r, :hl[r]]) == want_h


@pytest.mark.parametrize("ty", [O.TY_F16, O.TY_Q8_0, O.TY_F32])
def test_embed_rows(gpu, ty):
    rng = np.random.default_rng(9)
    vocab, d, rows, pos = 300, 128, 5, 7
    w = (rng.standard_normal((vocab, d)) * 0.5).astype(np.float32)
    data = {O.TY_F16: w.astype(np.float16).tobytes(), O.TY_F32: w.tobytes(),
            O.TY_Q8_0: O.q8_0_bytes(w)}[ty]
    if ty == O.TY_Q8_0:
        blocks = np.frombuffer(data, np.uint8).reshape(-1, 34)
        dd = blocks[:, :2].copy().view(np.float16).astype(np.float32)
        wf = (blocks[:, 2:].view(np.int8).astype(np.float32) * dd).reshape(vocab, d)
    else:
        wf = np.frombuffer(data, np.float32 if ty == O.TY_F32 else np.float16).astype(
            np.float32).reshape(vocab, d)
    bias = rng.standard_normal(vocab).astype(np.float32)[:vocab]
    lin = gpu.linear(ty, vocab, d, data, None)
    positions = rng.standard_normal((16, d)).astype(np.float32)
    toks = np.array([0, 299, 17, 17, 150], np.int32)
    x = torch.zeros(rows, d, device="cuda")
    gpu.pass_().embed_rows(lin, gpu.upload(positions), torch.from_numpy(toks).cuda(), rows, pos, x)
    gpu.sync()
    np.testing.assert_allclose(x.cpu().numpy(), wf[toks] + positions[pos], rtol=1e-6, atol=1e-6)
    del bias


def test_greedy_decode_on_device(gpu):
    # A small Whisper-shaped decoder (2 layers, d 128, 2 heads, FFN 256, vocabulary 700 with EOT,
    # <|notimestamps|> and 150 timestamps) over 3 segments' encoder outputs: 10 greedy steps with
    # tokens, histories and logits kept on the device, against the oracle's CPU decoder step
    # (gemv in f32, f16 caches, LayerNorm, attend) and search, segment by segment.
    from wavo_b200 import GGML_F16
    from wavo_b200.blocks import WhisperDecoder
    d, heads, d_ff, vocab, context, frames, B, L = 128, 2, 256, 700, 32, 37, 3, 2
    hd = d // heads
    eot, no_ts, begin = 540, 545, 550
    ids = {"eot": eot, "no_timestamps": no_ts, "begin": begin, "suppress": [541, 542, 3],
           "begin_suppress": [220, eot]}
    rng = np.random.default_rng(11)
    f16 = lambda r, c, s: (rng.standard_normal((r, c)) * s).astype(np.float16)  # noqa: E731
    vec = lambda n, s: (rng.standard_normal(n) * s).astype(np.float32)  # noqa: E731
    norm = lambda: (1.0 + vec(d, 0.1), vec(d, 0.1))  # noqa: E731
    embed = f16(vocab, d, 0.3)
    layers = []
    for _ in range(L):
        lw = {"qkv": f16(3 * d, d, 0.08), "self_out": f16(d, d, 0.08), "cross_q": f16(d, d, 0.08),
              "cross_kv": f16(2 * d, d, 0.08), "cross_out": f16(d, d, 0.08),
              "fc1": f16(d_ff, d, 0.08), "fc2": f16(d, d_ff, 0.08)}
        lw["b"] = {"qkv": vec(3 * d, 0.05), "self_out": vec(d, 0.05), "cross_q": vec(d, 0.05),
                   "cross_kv": vec(2 * d, 0.05), "cross_out": vec(d, 0.05)}
        lw["fc1_b"], lw["fc2_b"] = vec(d_ff, 0.05), vec(d, 0.05)
        lw["norm_self"], lw["norm_cross"], lw["norm_ffn"] = norm(), norm(), norm()
        layers.append(lw)
    positions = vec(context * d, 0.3).reshape(context, d)
    final = norm()
    wb = {"embed": embed.tobytes(), "positions": positions, "norm": final,
          "layers": [{**{k: (v.tobytes() if isinstance(v, np.ndarray) and v.dtype == np.float16
                             else v) for k, v in lw.items()}} for lw in layers]}
    dec = WhisperDecoder(gpu, GGML_F16, d, heads, d_ff, vocab, context, frames, B, wb, ids)
    enc = rng.standard_normal((B, frames, d)).astype(np.float32)
    prompt_last = [500, 501, 502]
    steps = 10
    p = gpu.pass_()
    dec.record_cross(p, gpu.upload(enc).reshape(B, frames, d))
    dec.start(prompt_last)
    for pos in range(steps):
        dec.record_step(p, pos)
    gpu.sync()
    hist = dec.history.cpu().numpy()
    hl = dec.hist_len.cpu().numpy()
    toks = dec.tokens.cpu().numpy()

    # The oracle, one segment at a time.
    lin = lambda w, b=None: O.Linear(O.TY_F16, w.shape[0], w.shape[1], w.tobytes(), b)  # noqa: E731
    E = lin(embed)
    ow = [{k: lin(lw[k], lw["b"].get(k) if k in lw["b"] else lw.get(k + "_b"))
           for k in ("qkv", "self_out", "cross_q", "cross_kv", "cross_out", "fc1", "fc2")}
          for lw in layers]
    ef = embed.astype(np.float32)
    for s in range(B):
        cross = []
        for l in range(L):
            kv = ow[l]["cross_kv"].gemm(np.ascontiguousarray(enc[s].ravel()), frames)
            c = np.zeros(frames * 2 * d, np.float32)
            O.pack_cache(kv, frames, d, hd, c, frames, 0)
            cross.append(c)
        own = [np.zeros(context * 2 * d, np.float32) for _ in range(L)]
        token, gen = prompt_last[s], []
        for pos in range(steps):
            if token == eot:
                break
            x = (ef[token] + positions[pos]).astype(np.float32)
            for l in range(L):
                lw, w = layers[l], ow[l]
                y = O.layer_norm(x, *lw["norm_self"], 1, d)
                qkv = w["qkv"].gemv(y)
                O.pack_cache(np.ascontiguousarray(qkv[d:]), 1, d, hd, own[l], context, pos)
                att = O.attend(np.ascontiguousarray(qkv[:d]), own[l], context, pos + 1, heads, hd)
                w["self_out"].gemv(att, x, "residual", 1.0)
                y = O.layer_norm(x, *lw["norm_cross"], 1, d)
                att = O.attend(w["cross_q"].gemv(y), cross[l], frames, frames, heads, hd)
                w["cross_out"].gemv(att, x, "residual", 1.0)
                y = O.layer_norm(x, *lw["norm_ffn"], 1, d)
                w["fc2"].gemv(w["fc1"].gemv(y, None, "gelu"), x, "residual", 1.0)
            y = O.layer_norm(x, *final, 1, d)
            logits = E.gemv(y)[:vocab].copy()
            token, _ = O.pick(logits, gen, ids["suppress"], ids["begin_suppress"], eot, no_ts,
                              begin)
            if token != eot:
                gen.append(token)
        assert list(hist[s, :hl[s]]) == gen, (s, list(hist[s, :hl[s]]), gen)
        assert (toks[s] == eot) == (token == eot)
