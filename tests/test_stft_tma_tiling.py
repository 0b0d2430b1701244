"""CPU check of the output tiling of stft_tma_kernel (spectral_stft_tma.cuh).

The kernel writes a complex64 (C, F, S) output, F = 1025, in tiles of 8
columns: bin rows R = c*F + k are split by R mod 4 into classes whose rows
share the 32-byte phase d = (R * o_rs) mod 4, one TMA box of 256 rows x 8
columns per class and tile, whose columns start d elements before the tile
(the last d columns of a tile are carried to the next tile's box by the
thread that computed them); values go out by plain stores at the first tile
of a run (shifted classes), after a run's last tile (carried columns), for
bin 1024, and for the whole last tile of a channel.  This test replays the
same decisions as the kernel, thread by thread, with symbolic values
(c, k, s) and checks that every output element is written exactly once with
its own value, that every staging slot a box reads was written in the same
tile, that no staging slot is written twice, and that every box lies inside
its tensor map (rows of its class, columns [0, S + d)) and needs no clipping.
"""
import pytest

F, W, Q, ROWS = 1025, 8, 4, 256


def thread_bins(t):
    """Bins of thread t of a transform group: butterfly j = 4*(t%32) + t/32
    of the last radix-8 pass and its mirror (128 for j = 0), bins j + 256 r,
    r = 0..3, as (class q = k mod 4, row i = k // 4, bin k)."""
    w, l = t >> 5, t & 31
    jb0 = 4 * l + w
    jb1 = 128 if jb0 == 0 else 256 - jb0
    bins = []
    for r in range(4):
        bins.append((w, l + 64 * r, jb0 + 256 * r))
        bins.append(((4 - w) & 3, (jb1 >> 2) + 64 * r, jb1 + 256 * r))
    return bins, jb0 == 0


def replay(C, S, o_rs, grid, box_at_channel_end=False):
    """box_at_channel_end: also use boxes at a channel's last tile (the
    layout the kernel avoids); such a box reaches past the row end."""
    tpc = ((S + 1) // 2 + Q - 1) // Q
    ntiles = C * tpc
    grid = max(1, min(grid, ntiles))
    orp = o_rs & 3
    nrows = [(C * F - m + 3) // 4 for m in range(4)]
    out = {}

    def wglob(c, k, s, val):
        assert 0 <= s < S and 0 <= k < F, (c, k, s)
        assert val == (c, k, s), (val, (c, k, s))
        assert (c, k, s) not in out, ("written twice", c, k, s)
        out[(c, k, s)] = val

    for cta in range(grid):
        fb, fe = cta * ntiles // grid, (cta + 1) * ntiles // grid
        carry = {}
        for f in range(fb, fe):
            c, tl = divmod(f, tpc)
            x0 = tl * W
            first = f == fb or tl == 0
            last = f + 1 == fe or tl + 1 == tpc
            nobox = tl + 1 == tpc and not box_at_channel_end
            stg = {}

            def wstg(key, val):
                q, i, sc = key
                assert 0 <= q < 4 and 0 <= i < ROWS and 0 <= sc < W, key
                assert key not in stg, ("staging written twice", key)
                stg[key] = val

            for g in range(Q):
                okA, okB = x0 + 2 * g < S, x0 + 2 * g + 1 < S
                for t in range(128):
                    bins, t0 = thread_bins(t)
                    for (q, i, k) in bins:
                        d = (((c * F + q) & 3) * orp) & 3
                        sA = 2 * g + d
                        A, B = (c, k, x0 + 2 * g), (c, k, x0 + 2 * g + 1)
                        slot = lambda s_: (g, t, q, i, s_)  # noqa: E731
                        direct = nobox or (first and d != 0)
                        if sA + 1 < W:
                            if direct:
                                if okA:
                                    wglob(*A, A)
                                if okB:
                                    wglob(*B, B)
                            else:
                                wstg((q, i, sA), A)
                                wstg((q, i, sA + 1), B)
                        elif sA < W:
                            if direct:
                                if okA:
                                    wglob(*A, A)
                            else:
                                wstg((q, i, sA), A)
                            if not first:
                                prev = carry[slot(0)]
                                if nobox:
                                    wglob(*prev, prev)
                                else:
                                    wstg((q, i, 0), prev)
                            if last:
                                if okB:
                                    wglob(*B, B)
                            else:
                                carry[slot(0)] = B
                        else:
                            s0 = sA - W
                            if not first:
                                pa, pb = carry[slot(s0)], carry[slot(s0 + 1)]
                                if nobox:
                                    wglob(*pa, pa)
                                    wglob(*pb, pb)
                                else:
                                    wstg((q, i, s0), pa)
                                    wstg((q, i, s0 + 1), pb)
                            if last:
                                if okA:
                                    wglob(*A, A)
                                if okB:
                                    wglob(*B, B)
                            else:
                                carry[slot(s0)] = A
                                carry[slot(s0 + 1)] = B
                    if t0:  # bin 1024
                        if okA:
                            wglob(c, 1024, x0 + 2 * g, (c, 1024, x0 + 2 * g))
                        if okB:
                            wglob(c, 1024, x0 + 2 * g + 1, (c, 1024, x0 + 2 * g + 1))
            # thread 0's boxes for this tile
            for q in range(4):
                R = c * F + q
                m = R & 3
                d = (m * orp) & 3
                if nobox or (first and d != 0):
                    continue
                y0, u0 = R >> 2, tl * W
                assert (2 * u0 * 4) % 16 == 0  # 16-byte aligned x
                for j in range(ROWS):
                    y = y0 + j
                    assert 0 <= y < nrows[m], "row outside the tensor map"
                    cc, k = divmod(4 * y + m, F)
                    assert cc == c and k == q + 4 * j
                    for sc in range(W):
                        u = u0 + sc
                        assert u < S + d, "box needs clipping"
                        s = u - d
                        assert s >= 0
                        assert (q, j, sc) in stg, ("stale staging", c, k, s)
                        val = stg[(q, j, sc)]
                        assert val == (c, k, s), (val, (c, k, s))
                        assert (c, k, s) not in out, ("written twice", c, k, s)
                        out[(c, k, s)] = val
    assert len(out) == C * F * S, "elements not written"


def test_every_bin_owned_once():
    ks = []
    for t in range(128):
        bins, t0 = thread_bins(t)
        for (q, i, k) in bins:
            assert k % 4 == q and k // 4 == i
            ks.append(k)
        if t0:
            ks.append(1024)
    assert sorted(ks) == list(range(F))


@pytest.mark.parametrize("C,S,o_rs,grid", [
    (1, 1, 1, 1), (1, 2, 2, 1), (1, 3, 3, 1), (1, 9, 9, 1), (2, 17, 17, 3),
    (5, 64, 64, 7), (3, 63, 64, 5), (3, 100, 101, 148), (2, 200, 203, 4),
    (4, 129, 131, 9), (1, 8189, 8189, 3), (2, 1000, 1002, 16),
    (6, 33, 35, 148), (2, 70, 72, 1), (1, 16, 16, 1), (2, 15, 18, 2)])
def test_tiling_writes_every_element_once(C, S, o_rs, grid):
    replay(C, S, o_rs, grid)


def test_boxes_at_a_channel_end_would_need_clipping():
    """Boxes at the last tile of a channel cover columns past the row end
    (TMA bounds stores in 16-byte chunks, so a row ending mid-chunk would lose
    its neighbour's first value): the replay rejects that layout."""
    with pytest.raises(AssertionError, match="clipping"):
        replay(1, 9, 9, 1, box_at_channel_end=True)
