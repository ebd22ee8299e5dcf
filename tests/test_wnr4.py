"""WNR4 kind MX (draft codec 8): the oracle restatement pinned against the reference's own CPU tools
(oracle/_ref/wnr4_tools.so: its encoder makes the records, its decoder is the reference), then the CUDA
tile decoder through the ABI 5 (include/wnr4_cuda.h) against the oracle: bit-exact slabs, refusals of
damaged records, status rules and tickets."""
import ctypes
import random

import numpy as np
import pytest

import oracle
import synth
import wexcuda

P, U32, U64, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int
POISON = 0xA5


def ref():
    L = oracle.ref_lib('wnr4_tools')
    if L is None:
        pytest.skip('reference WNR4 tools not built (make -C oracle ref)')
    return L


def geo_of(entry):
    e = np.frombuffer(bytes(entry), np.uint8)
    u16 = lambda at: int.from_bytes(e[at:at + 2], 'little')
    u32 = lambda at: int.from_bytes(e[at:at + 4], 'little')
    scount = [u16(20 + 4 * m) * u16(22 + 4 * m) for m in range(3)]
    scols = [u16(22 + 4 * m) for m in range(3)]
    return [0] + scount + scols + [u32(44 + 4 * m) for m in range(3)] + [u32(56 + 4 * m) for m in range(3)]


def make_wnr4(hidden, ffn, owners, seed, pb=1, G=32, cz=False, neg_zero=0.0, mode=2, sigma=0.02):
    """(model blob, model id, experts with .wnr4 record) encoded by the reference WNR4 encoder."""
    L = ref()
    experts = [synth.Expert(hidden, ffn, l, i, seed * 7919 + l * 131 + i, sigma, cz, mode, neg_zero) for l, i in owners]
    geo = (U32 * 13)(*geo_of(experts[0].entry))
    counts = np.zeros(L.wnr4t_counts_words(0, pb), np.uint64)
    for e in experts:
        assert L.wnr4t_count(geo, e.coded, pb, counts.ctypes.data) == 0
    blob = ctypes.create_string_buffer(L.wnr4t_model_bytes(0, pb))
    mid = L.wnr4t_build(0, pb, counts.ctypes.data, blob)
    assert mid
    h = L.wnr4t_model_open(blob, len(blob.raw))
    assert h
    for e in experts:
        cap = 2 * len(e.coded) + (1 << 20)
        out = ctypes.create_string_buffer(cap)
        n = L.wnr4t_encode(h, geo, e.coded, e.flags, e.owner, G, out, cap)
        assert n > 0
        e.wnr4 = out.raw[:n]
        e.geo = list(geo)
    L.wnr4t_model_close(h)
    return blob.raw, mid, experts


@pytest.mark.parametrize('pb,cz', [(1, False), (5, True)])
def test_oracle_matches_reference_wnr4_decoder(pb, cz):
    L = ref()
    blob, mid, ex = make_wnr4(1024, 512, [(0, 0), (0, 1)], seed=5 + pb, pb=pb, cz=cz, neg_zero=0.03 if cz else 0)
    assert oracle.lib().oracle_wnm4_id(blob, len(blob)) == mid
    h = L.wnr4t_model_open(blob, len(blob))
    for e in ex:
        raw = len(e.source)
        out = ctypes.create_string_buffer(raw)
        err = L.wnr4t_decode(h, (U32 * 13)(*e.geo), e.wnr4, len(e.wnr4), e.owner, out, 1)
        assert err == 0 and out.raw == e.expected
        err2, slab = oracle.wnr4_decode(blob, e.geo, e.wnr4, e.owner, raw)
        assert err2 == 0 and slab == e.expected
        # a damaged record: both refuse, with the same error bits
        bad = bytearray(e.wnr4)
        bad[len(bad) // 3] ^= 0x10
        err = L.wnr4t_decode(h, (U32 * 13)(*e.geo), bytes(bad), len(bad), e.owner, out, 1)
        err2, _ = oracle.wnr4_decode(blob, e.geo, bytes(bad), e.owner, raw)
        assert err != 0 and err2 == err
    L.wnr4t_model_close(h)


def lib():
    W = wexcuda.lib()
    W.wnr4_cuda_abi.restype = U32
    W.wnr4_cuda_register_model.argtypes = [P, SZ, I]
    W.wnr4_cuda_batch_submit.argtypes = [I, P, P, P, P, U32, I, P, P, P]
    W.wnr4_cuda_batch_wait.argtypes = [I, P]
    W.wnr4_cuda_decode_batch.argtypes = [I, P, P, P, P, U32, I, P, P, P]
    return W


def _dst(torch, entry, n):
    e = np.frombuffer(bytes(entry), np.uint8)
    shapes = [(int.from_bytes(e[20 + 4 * m:22 + 4 * m], 'little'), int.from_bytes(e[22 + 4 * m:24 + 4 * m], 'little'))
              for m in range(3)]
    ts, sp, wp = [], [], []
    for _ in range(n):
        for r, c in shapes:
            s = torch.full((r * c,), POISON, dtype=torch.uint8, device='cuda')
            w = torch.full((r * c * 16,), POISON, dtype=torch.uint8, device='cuda')
            ts += [s, w]; sp.append(s.data_ptr()); wp.append(w.data_ptr())
    return ts, sp, wp


def _slab(ts, j):
    t = ts[6 * j:6 * j + 6]
    return b''.join(bytes(x.cpu().numpy()) for x in (t[0], t[2], t[4])) + \
        b''.join(bytes(x.cpu().numpy()) for x in (t[1], t[3], t[5]))


def _decode(W, torch, blob, mid, ex, records=None, owners=None):
    records = records or [e.wnr4 for e in ex]
    owners = owners or [e.owner for e in ex]
    n = len(records)
    ts, sp, wp = _dst(torch, ex[0].entry, n)
    recs = [np.frombuffer(r, np.uint8) for r in records]
    totals = (SZ * n)(*[len(r) for r in records])
    status = (ctypes.c_int * n)()
    bad = W.wnr4_cuda_decode_batch(n, (U32 * 13)(*ex[0].geo), wexcuda._ptrs([r.ctypes.data for r in recs]), totals,
                                   (U32 * n)(*owners), mid, 0, wexcuda._ptrs(sp), wexcuda._ptrs(wp), status)
    return bad, list(status), ts


@pytest.mark.gpu
@pytest.mark.parametrize('hidden,ffn,pb,G,cz', [(1024, 512, 1, 32, False), (1024, 512, 5, 32, True),
                                               (2048, 768, 1, 32, True), (256, 96, 1, 4, False), (1024, 512, 5, 1, False)])
def test_wnr4_kernel_bit_exact(hidden, ffn, pb, G, cz):
    import torch
    W = lib()
    assert W.wnr4_cuda_abi() == 5
    blob, mid, ex = make_wnr4(hidden, ffn, [(1, i) for i in range(3)], seed=hidden + pb + G, pb=pb, G=G, cz=cz,
                              neg_zero=0.03 if cz else 0)
    assert W.wnr4_cuda_register_model(blob, len(blob), 0) == 0
    bad, st, ts = _decode(W, torch, blob, mid, ex)
    assert bad == 0 and st == [0, 0, 0]
    for j, e in enumerate(ex):
        assert _slab(ts, j) == e.expected, j
        err, slab = oracle.wnr4_decode(blob, e.geo, e.wnr4, e.owner, len(e.source))
        assert err == 0 and slab == e.expected


@pytest.mark.gpu
def test_wnr4_corruption_refused_like_the_oracle():
    import torch
    W = lib()
    blob, mid, ex = make_wnr4(1024, 512, [(2, i) for i in range(2)], seed=99, cz=True, neg_zero=0.03)
    assert W.wnr4_cuda_register_model(blob, len(blob), 0) == 0
    rng = random.Random(7)
    records, owners, expect = [], [], []
    for trial in range(24):
        e = ex[trial % 2]
        rec = bytearray(e.wnr4)
        used = len(rec) - 1
        while rec[used] == 0:
            used -= 1
        rec[rng.randrange(64, used + 1)] ^= 1 << rng.randrange(8)
        err, _ = oracle.wnr4_decode(blob, e.geo, bytes(rec), e.owner, len(e.source))
        records.append(bytes(rec)); owners.append(e.owner); expect.append(err)
    bad, st, ts = _decode(W, torch, blob, mid, [ex[0]] * 24, records, owners)
    for j, err in enumerate(expect):
        assert (st[j] == 0) == (err == 0), (j, st[j], err)
    assert sum(1 for s in st if s) >= 20


@pytest.mark.gpu
def test_wnr4_status_rules_and_tickets():
    import torch
    W = lib()
    blob, mid, ex = make_wnr4(1024, 512, [(3, 0), (3, 1)], seed=3)
    assert W.wnr4_cuda_register_model(blob, len(blob), 0) == 0
    assert W.wnr4_cuda_register_model(blob, len(blob), 0) == 0       # again: no-op
    assert W.wnr4_cuda_register_model(blob[:64], 64, 0) == -1
    # wrong owner -> -1 (not queued); unregistered model -> every status 1
    bad, st, ts = _decode(W, torch, blob, mid, ex, owners=[ex[0].owner, ex[1].owner ^ 1])
    assert st == [0, -1] and _slab(ts, 0) == ex[0].expected
    bad, st, ts = _decode(W, torch, blob, mid ^ 0x55, ex)
    assert st == [1, 1] and bad == 2
    # four tickets in flight on this thread, then a fifth is refused until one is waited for
    n = 2
    keep, tickets = [], []
    geo = (U32 * 13)(*ex[0].geo)
    for k in range(5):
        t_s, sp, wp = _dst(torch, ex[0].entry, n)
        recs = [np.frombuffer(e.wnr4, np.uint8) for e in ex]
        keep.append((t_s, recs, wexcuda._ptrs(sp), wexcuda._ptrs(wp)))
        t = W.wnr4_cuda_batch_submit(n, geo, wexcuda._ptrs([r.ctypes.data for r in recs]),
                                     (SZ * n)(*[len(e.wnr4) for e in ex]), (U32 * n)(*[e.owner for e in ex]), mid, 0,
                                     keep[-1][2], keep[-1][3], None)
        tickets.append(t)
    assert all(t >= 0 for t in tickets[:4]) and tickets[4] == -4
    for k, t in enumerate(tickets[:4]):
        status = (ctypes.c_int * n)()
        assert W.wnr4_cuda_batch_wait(t, status) == 0 and list(status) == [0, 0]
        assert _slab(keep[k][0], 0) == ex[0].expected and _slab(keep[k][0], 1) == ex[1].expected
    assert W.wnr4_cuda_batch_wait(tickets[0], None) == -1   # already waited for
    W.wnr4_cuda_release_thread()
