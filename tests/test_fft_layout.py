"""The register-phase FFT of log_mel_kernel (wavo_b200/csrc/frontend.cu), checked at the index level
against the reference's radix-2 Stockham FFT (src/fft.rs:131-143: stage `size` computes output i
from inputs 2i and 2i + 1 into positions i and i + 256 with the twiddle of index
i / (512 / size) · (512 / size)). The kernel's three register layouts, its per-lane twiddle rows
and its exchange swizzle are restated here from the kernel's formulas; every butterfly of every
stage must take the reference's inputs and twiddle and write the reference's outputs, and every
quarter-warp's 16-byte accesses of each layout must fall in distinct bank groups."""

N = 512


def rotr(x, k):
    k %= 9
    return ((x >> k) | (x << (9 - k))) & (N - 1)


def phys(L):  # fe_phys
    return L ^ (((L >> 4) ^ (L >> 3)) & 7)


LAYOUTS = {  # (lane, register) -> label
    "A": lambda l, r: (l << 4) | r,                                # stages 0-3
    "B": lambda l, r: (l & 15) | (r << 4) | ((l >> 4) << 8),       # stages 4-7
    "C": lambda l, r: (r & 7) | (l << 3) | ((r >> 3) << 8),        # stage 8
}


def twiddle_index(t, L0):  # the label's low t bits · 2^(8 - t)
    return (L0 & ((1 << t) - 1)) << (8 - t)


def twl_rows():
    """The host's per-lane twiddle table [23][32] (indices into the 256 twiddles)."""
    twl = [[None] * 32 for _ in range(23)]
    for l in range(32):
        for t in range(4, 8):
            for rl in range(1 << (t - 4)):
                twl[(1 << (t - 4)) - 1 + rl][l] = twiddle_index(t, (l & 15) | (rl << 4))
        for r0 in range(8):
            twl[15 + r0][l] = twiddle_index(8, r0 | (l << 3))
    return twl


def reference_stage(t):
    size, out = 2 << t, []
    for i in range(N // 2):
        out.append((2 * i, 2 * i + 1, i, i + N // 2, i // (N // size) * (N // size)))
    return sorted(out)


def kernel_stage(t, twl):
    lay = LAYOUTS["A" if t < 4 else "B" if t < 8 else "C"]
    bit = t if t < 4 else t - 4 if t < 8 else 3
    out = []
    for l in range(32):
        for r0 in range(16):
            if (r0 >> bit) & 1:
                continue
            L0, L1 = lay(l, r0), lay(l, r0 | (1 << bit))
            if t < 4:
                idx = (r0 & ((1 << t) - 1)) << (8 - t)  # the same for every lane
            elif t < 8:
                idx = twl[(1 << bit) - 1 + (r0 & ((1 << bit) - 1))][l]
            else:
                idx = twl[15 + r0][l]
            out.append((rotr(L0, t), rotr(L1, t), rotr(L0, t + 1), rotr(L1, t + 1), idx))
    return sorted(out)


def test_layouts_are_permutations():
    for name, f in LAYOUTS.items():
        assert sorted(f(l, r) for l in range(32) for r in range(16)) == list(range(N)), name
    assert sorted(phys(L) for L in range(N)) == list(range(N))


def test_every_stage_is_the_references():
    twl = twl_rows()
    assert all(v is not None for row in twl for v in row)
    for t in range(9):
        assert kernel_stage(t, twl) == reference_stage(t), t


def test_first_stage_order_and_final_bins():
    # Label L starts at position L, which holds sample bitrev9(L) (the reference's first-stage
    # order: even samples before odd ones at every level), computed by the kernel as
    # bitrev4(r) · 32 + bitrev5(lane); after nine stages label L is at position (bin) L.
    starts = [0]
    while len(starts) < N:
        starts = [2 * v for v in starts] + [2 * v + 1 for v in starts]
    rev = lambda x, b: int(format(x, f"0{b}b")[::-1], 2)  # noqa: E731
    for l in range(32):
        for r in range(16):
            L = (l << 4) | r
            assert starts[L] == (rev(r, 4) << 5) | rev(l, 5)
    assert all(rotr(L, 9) == L for L in range(N))


def test_exchanges_are_free_of_bank_conflicts():
    for name, f in LAYOUTS.items():
        for r in range(16):
            for q in range(4):
                groups = {phys(f(l, r)) % 8 for l in range(8 * q, 8 * q + 8)}
                assert len(groups) == 8, (name, r, q)
