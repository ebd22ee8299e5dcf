"""The weight items' symbol lookup (weight_stream in nr3_decode.cu, over the two-level rows that
build_image in nr3_host.cpp makes from a WNM2 model), emulated on the CPU with numpy's 32-bit wrap-around
arithmetic for every slot of every reachable context of a trained model: the quartile from the level-1
row, the rank from the level-2 row, and start and end taken by the byte permute and the funnel shift,
against a direct search of the context's CDF. Also the two-symbol payload window."""
import numpy as np

import synth

M32 = np.uint64(0xFFFFFFFF)


def u32(x):
    return (np.asarray(x, dtype=np.uint64) & M32)


def popc(x):
    x = u32(x)
    bits = np.unpackbits(np.atleast_1d(x).astype('>u4').view(np.uint8).reshape(-1, 4), axis=1)
    return bits.sum(axis=1).astype(np.uint64).reshape(x.shape)


def byte_perm(x, y, s):
    """__byte_perm with selector nibbles < 8 (no sign replication)."""
    b = np.stack([(u32(x) >> np.uint64(8 * i)) & np.uint64(255) for i in range(4)] +
                 [(u32(y) >> np.uint64(8 * i)) & np.uint64(255) for i in range(4)])
    s = u32(s)
    out = np.zeros_like(u32(x))
    for i in range(4):
        sel = ((s >> np.uint64(4 * i)) & np.uint64(7)).astype(np.int64)
        out |= np.take_along_axis(b, sel[None, ...], axis=0)[0] << np.uint64(8 * i)
    return out


def funnelshift_r(lo, hi, n):
    n = u32(n) & np.uint64(31)
    v = (u32(hi) << np.uint64(32)) | u32(lo)
    return (v >> n) & M32


def rows_of(cdf17):
    """The level-1 and level-2 rows of one context (as build_image lays them out)."""
    c = [int(v) for v in cdf17]
    l1 = (c[4] | c[8] << 16, c[12] | 16384 << 16)
    l2 = [(c[4 * q] | c[4 * q + 1] << 16, c[4 * q + 2] | c[4 * q + 3] << 16) for q in range(4)]
    return l1, l2


def lookup(l1, l2, slot):
    """The kernel's steps for a vector of slots: (symbol, start, freq)."""
    slot = u32(slot)
    gs = u32(slot * np.uint64(0x10001) + np.uint64(0x80008000))
    cx, cy = np.uint64(l1[0]), np.uint64(l1[1])
    d1 = u32(gs - cy)
    q = popc((u32(gs - cx) & np.uint64(0x80008000)) | ((d1 >> np.uint64(1)) & np.uint64(0x4000)))
    rx = np.array([l2[int(k)][0] for k in q], dtype=np.uint64)
    ry = np.array([l2[int(k)][1] for k in q], dtype=np.uint64)
    r = popc((u32(gs - ry) & np.uint64(0x80008000)) | (u32(gs - rx) >> np.uint64(31)))
    bound = byte_perm(np.full_like(q, cx), np.full_like(q, cy), np.uint64(0x10) + np.uint64(0x22) * q)
    two = (r & np.uint64(2)) != 0
    lo = np.where(two, ry, rx)
    hi = np.where(two, bound, ry)
    pair = funnelshift_r(lo, hi, r << np.uint64(4))
    start = pair & np.uint64(0xFFFF)
    freq = u32((pair >> np.uint64(16)) - start)
    return np.uint64(4) * q + r, start, freq


def test_lookup_matches_a_direct_search_on_every_slot():
    blob, ex = synth.make_experts(256, 128, [(0, i) for i in range(2)], seed=3, sigma=0.03, train_every=1)
    wc = np.frombuffer(blob[32:32 + 3 * 567 * 34], dtype='<u2').reshape(3, 567, 17)
    slots = np.arange(16384, dtype=np.uint64)
    checked = 0
    for m in range(3):
        for srel in range(7):
            for mx in range(9):
                for pm in range(mx + 1):
                    if mx == 8 and pm != 8:
                        continue   # reachable: pm <= mx < 8, or the block start pm = mx = 8
                    cdf = wc[m, (srel * 9 + pm) * 9 + mx].astype(np.int64)
                    l1, l2 = rows_of(cdf)
                    sym, start, freq = lookup(l1, l2, slots)
                    want = np.searchsorted(cdf, slots.astype(np.int64), side='right') - 1
                    assert np.array_equal(sym.astype(np.int64), want)
                    assert np.array_equal(start.astype(np.int64), cdf[want])
                    assert np.array_equal(freq.astype(np.int64), cdf[want + 1] - cdf[want])
                    checked += 1
    assert checked == 3 * 7 * 37


def test_two_symbol_window():
    """One big-endian 4-byte window serves a pair of symbols: whatever the first takes (0, 8 or 16 bits,
    from the top), the second's two bytes are the window shifted left by that."""
    rng = np.random.default_rng(1)
    for _ in range(2000):
        stream = bytes(rng.integers(0, 256, 8, dtype=np.uint8))
        win = int.from_bytes(stream[:4], 'big')
        for b1 in (0, 8, 16):
            second = ((win << b1) & 0xFFFFFFFF) >> 16
            assert second == int.from_bytes(stream[b1 // 8:b1 // 8 + 2], 'big')
