"""Parity of the CUDA WNR2/WNR3 decoder (through the C-ABI of libwexb200.so) with the oracle: the
reference's conformance vectors, seeded synthetic experts at several shapes and chunk pairs, with
and without canonical zero and the ceil form, WNR2 records, host-injected corruption (the decoder
must refuse exactly what the oracle refuses, and leave the destination untouched), and the
argument rules of every entry point."""
import ctypes
import json
import os
import random

import numpy as np
import pytest

import oracle
import synth
import wexcuda

pytestmark = pytest.mark.gpu
POISON = 0xA5


@pytest.fixture(scope='module')
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    assert wexcuda.lib().wex_cuda_helper_abi() == 1
    return torch


def _dst(torch, entry, n=1):
    """Poisoned device buffers for n records of this entry shape: (tensors, scale ptrs, weight ptrs)."""
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
    """Canonical slab bytes of record j from its six destination tensors."""
    t = ts[6 * j:6 * j + 6]
    return b''.join(bytes(x.cpu().numpy()) for x in (t[0], t[2], t[4])) + \
        b''.join(bytes(x.cpu().numpy()) for x in (t[1], t[3], t[5]))


def _untouched(ts, j):
    return all(bool((x == POISON).all()) for x in ts[6 * j:6 * j + 6])


def _decode_device(torch, entries, records):
    ts, sp, wp = _dst(torch, entries[0], len(entries))
    bad, st = wexcuda.decode_batch_to_device(entries, records, 0, sp, wp)
    return bad, st, ts


# ---- the reference's conformance vectors --------------------------------------------------------
def test_conformance_vector_records(torch_cuda, golden_dir):
    items = json.load(open(os.path.join(golden_dir, 'vectors.json')))
    n = 0
    for name, item in sorted(items.items()):
        if not any(r['codec'] == 5 for r in item['records']):
            continue
        f = oracle.Wex4File(open(os.path.join(golden_dir, 'vectors', name), 'rb').read())
        for rr in item['records']:
            if rr['codec'] != 5:
                continue
            rec = f.records[rr['r']]
            blob = f.blob(rec['blob'] - 1)
            if wexcuda.register_model(blob) != 0:   # an invalid model blob is refused at registration
                assert oracle.wnm2_id(blob) is None
                continue
            entry, stored = bytes.fromhex(rr['entry']), f.stored(rr['r'])
            st_o, where, slab_o = oracle.nrx_decode(blob, entry, stored, rec['decoded'])
            bad, st, ts = _decode_device(torch_cuda, [entry], [stored])
            assert (st[0] == 0) == (st_o == 0), (name, rr['r'], where, st)
            if st[0] == 0:
                assert _slab(ts, 0) == slab_o, (name, rr['r'])
            else:   # a record naming a model that is not registered is "unavailable" (1), not invalid
                assert st[0] == (1 if where == 6 else -1) and _untouched(ts, 0), (name, rr['r'], where)
            n += 1
    assert n >= 20


# ---- synthetic experts ----------------------------------------------------------------------------
CASES = [
    # hidden, ffn, chunks, cz, neg_zero, nr3, mode
    (1024, 512, (2048, 512), False, 0.0, True, 2),
    (1024, 512, (2048, 512), True, 0.03, True, 2),
    (1024, 512, (2048, 512), True, 0.0, True, 3),
    (1024, 512, (2048, 512), False, 0.0, True),
    (1024, 512, (2048, 512), True, 0.03, True),
    (1024, 512, (512, 256), True, 0.03, True),
    (1024, 512, (4096, 1024), False, 0.0, True),
    (1024, 512, (16384, 16384), True, 0.0, True),
    (256, 96, (512, 256), False, 0.0, True),      # scale counts that are not multiples of 16
    (2048, 768, (2048, 512), False, 0.0, True),   # the mid expert shape
    (1024, 512, (2048, 512), False, 0.0, False),  # WNR2
]
CASES = [c if len(c) == 7 else c + (0,) for c in CASES]


@pytest.mark.parametrize('hidden,ffn,chunks,cz,neg_zero,nr3,mode', CASES)
def test_synthetic_experts_bit_exact(torch_cuda, hidden, ffn, chunks, cz, neg_zero, nr3, mode):
    sig = lambda layer: 0.01 + 0.01 * layer
    blob, ex = synth.make_experts(hidden, ffn, [(l, i) for l in range(3) for i in range(2)], seed=hidden + ffn,
                                  sigma=sig, cz=cz, neg_zero=neg_zero, train_every=2, wchunk=chunks[0],
                                  schunk=chunks[1], nr3=nr3, mode=mode)
    assert all(e.codec == (5 if nr3 else 4) for e in ex)
    assert wexcuda.register_model(blob) == 0
    bad, st, ts = _decode_device(torch_cuda, [e.entry for e in ex], [e.record for e in ex])
    assert bad == 0 and st == [0] * len(ex)
    for j, e in enumerate(ex):
        got = _slab(ts, j)
        assert got == e.expected, j
        st_o, _, slab_o = oracle.nrx_decode(blob, e.entry, e.record, len(e.source))
        assert st_o == 0 and slab_o == got


def test_ceil_form_blocks_really_occur():
    """Mode 2 exercises the ceil inverse (blocks stored halved, scale + 1) in every matrix; mode 3
    keeps it off in w2, whose block of maximum 5 fails the gate."""
    blob, ex = synth.make_experts(1024, 512, [(0, 0), (0, 1)], seed=3, sigma=0.02, train_every=1, mode=lambda i: 2 + i)
    assert ex[0].flags & 7 == 7 and ex[1].flags & 7 == 5
    assert ex[0].coded != ex[0].source
    s = np.frombuffer(ex[0].coded[:49152], np.uint8).astype(int) - np.frombuffer(ex[0].source[:49152], np.uint8)
    assert (s == 1).sum() > 1000 and set(np.unique(s)) <= {0, 1}


# ---- corruption injected on the host ------------------------------------------------------------
def test_corrupted_records_refused_like_the_oracle(torch_cuda):
    blob, ex = synth.make_experts(1024, 512, [(0, i) for i in range(4)], seed=77, sigma=0.02, cz=True,
                                  neg_zero=0.03, train_every=1)
    assert wexcuda.register_model(blob) == 0
    rng = random.Random(1234)
    entries, records, expect = [], [], []
    for trial in range(48):
        e = ex[trial % 4]
        rec = bytearray(e.record)
        used = len(rec) - 1
        while used > 0 and rec[used] == 0:
            used -= 1
        kind = trial % 6
        if kind == 0:      # a bit flip anywhere in the payload
            at = rng.randrange(32 + 2 * 100, used + 1); rec[at] ^= 1 << rng.randrange(8)
        elif kind == 1:    # a byte of a stream length
            at = 32 + 2 * rng.randrange(50); rec[at] ^= 1 << rng.randrange(8)
        elif kind == 2:    # a non-zero padding byte
            rec[rng.randrange(used + 1, len(rec))] = 1
        elif kind == 3:    # another owner (the stream hashes cover it)
            rec[28] ^= 1
        elif kind == 4:    # an anchor byte
            rec[24 + rng.randrange(3)] ^= 1
        else:              # the canonical-zero flag cleared (data then hashes to other end states)
            rec[27] ^= 8
        rec = bytes(rec)
        st_o, _, slab_o = oracle.nrx_decode(blob, e.entry, rec, len(e.source))
        entries.append(e.entry); records.append(rec); expect.append((st_o, slab_o))
    bad, st, ts = _decode_device(torch_cuda, entries, records)
    refused = 0
    for j, (st_o, slab_o) in enumerate(expect):
        assert (st[j] == 0) == (st_o == 0), j
        if st[j]:
            assert st[j] == -1 and _untouched(ts, j), j
            refused += 1
        else:
            assert _slab(ts, j) == slab_o
    assert refused >= 40


def test_integrity_error_bits(torch_cuda):
    """A CZ record carrying a -0 nibble reports bit 8; a damaged stream bit 1 or 2."""
    blob, ex = synth.make_experts(1024, 512, [(0, 0)], seed=21, sigma=0.02, train_every=1)
    e = ex[0]
    assert wexcuda.register_model(blob) == 0
    rec = bytearray(e.record)
    rec[200 * 4] ^= 0x10
    bad, st, ts = _decode_device(torch_cuda, [e.entry], [bytes(rec)])
    assert st == [-1] and wexcuda.lib().wexb_last_error_bits() & 3


# ---- entry points and argument rules ----------------------------------------------------------
@pytest.fixture(scope='module')
def tiny(torch_cuda):
    blob, ex = synth.make_experts(1024, 512, [(5, i) for i in range(3)], seed=31, sigma=0.02, cz=True,
                                  neg_zero=0.03, train_every=1)
    assert wexcuda.register_model(blob) == 0
    return blob, ex


def test_decode_to_host_in_place(tiny):
    blob, ex = tiny
    for e in ex:
        raw = len(e.source)
        aligned = (raw + 4095) & ~4095
        slab = bytearray(aligned)
        slab[aligned - len(e.record):] = e.record
        assert wexcuda.decode_to_host(e.entry, slab) == 0
        assert bytes(slab[:raw]) == e.expected


def test_decode_to_host_failure_keeps_the_slab(tiny):
    blob, ex = tiny
    e = ex[0]
    aligned = (len(e.source) + 4095) & ~4095
    slab = bytearray(aligned)
    rec = bytearray(e.record); rec[5000] ^= 4
    slab[aligned - len(rec):] = rec
    before = bytes(slab)
    assert wexcuda.decode_to_host(e.entry, slab) == -1
    assert bytes(slab) == before


def test_decode_to_device_single(torch_cuda, tiny):
    blob, ex = tiny
    e = ex[1]
    ts, sp, wp = _dst(torch_cuda, e.entry)
    assert wexcuda.decode_to_device(e.entry, e.record, 0, sp, wp) == 0
    assert _slab(ts, 0) == e.expected


def test_batch_to_host(tiny):
    blob, ex = tiny
    dsts = [np.full(len(e.source), POISON, np.uint8) for e in ex]
    bad, st = wexcuda.decode_batch_to_host([e.entry for e in ex], [e.record for e in ex], 0, dsts)
    assert bad == 0 and st == [0, 0, 0]
    assert all(d.tobytes() == e.expected for d, e in zip(dsts, ex))


def test_batch_to_host_pinned_in_place(tiny):
    """dst[i] overlapping record i itself (the in-place decode of a slab holding its record)."""
    blob, ex = tiny
    bufs, dsts, recs = [], [], []
    for e in ex:
        aligned = (len(e.source) + 4095) & ~4095
        b = np.zeros(aligned, np.uint8)
        b[aligned - len(e.record):] = np.frombuffer(e.record, np.uint8)
        assert wexcuda.host_register(b) == 0
        bufs.append(b); dsts.append(b); recs.append(b[aligned - len(e.record):])
    bad, st = wexcuda.decode_batch_to_host([e.entry for e in ex], recs, 0, dsts)
    assert bad == 0
    for b, e in zip(bufs, ex):
        assert b[:len(e.source)].tobytes() == e.expected
        assert wexcuda.host_unregister(b) == 0


def test_status_rules(torch_cuda, tiny):
    blob, ex = tiny
    e = ex[0]
    ts, sp, wp = _dst(torch_cuda, e.entry, 4)
    other = synth.make_experts(1024, 512, [(0, 0)], seed=99, sigma=0.03, train_every=1)[1][0]  # unregistered model
    wnr1 = synth.entry_with(e.entry, codec=3)
    bad_entry = bytearray(e.entry); bad_entry[20] ^= 1   # scale rows differ from weight rows
    entries = [e.entry, other.entry, bytes(bad_entry), wnr1]
    records = [e.record, other.record, e.record, e.record]
    bad, st = wexcuda.decode_batch_to_device(entries, records, 0, sp, wp)
    assert st == [0, 1, -1, -1] and bad == 3
    assert _slab(ts, 0) == e.expected and _untouched(ts, 1) and _untouched(ts, 2)
    L = wexcuda.lib()
    assert L.wex_cuda_decode_batch_to_device(0, None, None, 0, None, None, None) == 0
    assert L.wex_cuda_decode_batch_to_device(2, None, None, 0, None, None, None) == 2
    st1 = (ctypes.c_int * 1)()
    ptrs = (ctypes.c_void_p * 3)(*sp[:3])
    assert L.wex_cuda_decode_batch_to_device(1, None, None, 0, ptrs, ptrs, st1) == 1   # entries NULL
    assert wexcuda.decode_to_device(wnr1, e.record, 0, sp[:3], wp[:3]) == 1           # WNR1: unavailable
    assert L.wex_cuda_register_model(b'\0' * 59408, 59408) == -1
    assert wexcuda.register_model(blob) == 0                                           # again: no-op
    assert L.wex_cuda_helper_features() == 63


def test_resident_decode(torch_cuda, tiny):
    blob, ex = tiny
    res = wexcuda.Resident([e.entry for e in ex], [e.record for e in ex], 0)
    assert res.failures == 0 and res.bytes > sum(len(e.record) for e in ex)
    order = [2, 0, 1, 2]
    ts, sp, wp = _dst(torch_cuda, ex[0].entry, len(order))
    assert res.decode(order, sp, wp) == 0
    bad, st = res.wait()
    assert bad == 0 and st == [0] * 4 and res.launches() == 1   # one persistent launch (one model)
    for j, x in enumerate(order):
        assert _slab(ts, j) == ex[x].expected
    res.close()


def test_resident_two_decodes_queued(torch_cuda, tiny):
    """Two decodes of one resident set queued at once (different subsets and destinations): each wait
    returns the oldest decode's statuses; a third decode with two queued drops the oldest's statuses;
    a wait with nothing queued returns -1."""
    blob, ex = tiny
    res = wexcuda.Resident([e.entry for e in ex], [e.record for e in ex], 0)
    res.profile(True)
    a, b, c = [1, 2], [0, 1, 2], [2]
    ta, sa, wa = _dst(torch_cuda, ex[0].entry, len(a))
    tb, sb, wb = _dst(torch_cuda, ex[0].entry, len(b))
    tc, sc, wc = _dst(torch_cuda, ex[0].entry, len(c))
    L = wexcuda.lib()
    status = (ctypes.c_int * 3)()

    def queue(index, sp, wp):
        idx = (ctypes.c_int * len(index))(*index)
        return L.wexb_resident_decode(res.handle, len(index), idx, wexcuda._ptrs(sp), wexcuda._ptrs(wp), None)
    assert queue(a, sa, wa) == 0 and queue(b, sb, wb) == 0
    assert L.wexb_resident_wait(res.handle, status) == 0 and list(status)[:2] == [0, 0]   # a
    ms = (ctypes.c_float * 3)()
    assert L.wexb_resident_kernel_ms(res.handle, ms) == 0 and ms[1] > 0 and all(v >= 0 for v in ms)
    assert queue(c, sc, wc) == 0                       # b and c queued
    assert queue(a, sa, wa) == 0                       # b waited for and dropped; c and a queued
    assert L.wexb_resident_wait(res.handle, status) == 0 and list(status)[:1] == [0]        # c
    assert L.wexb_resident_wait(res.handle, status) == 0 and list(status)[:2] == [0, 0]     # a
    assert L.wexb_resident_wait(res.handle, status) == -1
    for ts, index in ((ta, a), (tb, b), (tc, c)):
        for j, x in enumerate(index):
            assert _slab(ts, j) == ex[x].expected
    res.close()


def test_bounded_wait_gives_up_and_the_context_stays_usable(torch_cuda, tiny):
    """The mbarrier wait every kernel uses, on a barrier nothing arrives on, gives up after its polls
    with error bit 16 (no spin without end, no fault); a decode right after it is bit-exact."""
    st, bits = wexcuda.selftest_bounded_wait(0, 2000)
    assert st == 0 and bits == 16
    blob, ex = tiny
    bad, st2, ts = _decode_device(torch_cuda, [e.entry for e in ex], [e.record for e in ex])
    assert bad == 0 and all(_slab(ts, j) == e.expected for j, e in enumerate(ex))


def test_host_wait_gives_up_before_a_long_device_wait(torch_cuda, tiny):
    """Every host wait of the library is bounded (wexb_set_wait_limit). With a host limit shorter than a
    device-side bounded wait, the self-test call returns 1 (host gave up) while its probe still polls; the
    probe then gives up on its own, the device stays usable, and a decode afterwards is bit-exact."""
    import time
    default = wexcuda.wait_limit()
    assert wexcuda.set_wait_limit(0) == -1 and wexcuda.set_wait_limit(-1) == -1
    assert wexcuda.selftest_bounded_wait(0, (1 << 24) + 1)[0] == -1   # above the kernels' own limit
    t = time.perf_counter()
    assert wexcuda.selftest_bounded_wait(0, 1 << 16) == (0, 16)
    per_poll = (time.perf_counter() - t) / (1 << 16)
    polls = min(1 << 24, max(1 << 16, int(0.5 / max(per_poll, 1e-9))))   # about half a second of polling
    if polls * per_poll < 0.1:
        pytest.skip(f'2^24 polls take only {polls * per_poll:.3f} s here')
    try:
        assert wexcuda.set_wait_limit(0.02) == 0
        t = time.perf_counter()
        st, _ = wexcuda.selftest_bounded_wait(0, polls)
        gave_up = time.perf_counter() - t
        assert st == 1 and gave_up < 0.5 * polls * per_poll, (st, gave_up)
    finally:
        assert wexcuda.set_wait_limit(default) == 0
    deadline = time.perf_counter() + 60
    while True:   # 1 while the previous probe still runs, then a clean self-test
        st, bits = wexcuda.selftest_bounded_wait(0, 2000)
        if st != 1 or time.perf_counter() > deadline:
            break
        time.sleep(0.01)
    assert (st, bits) == (0, 16)
    blob, ex = tiny
    bad, st2, ts = _decode_device(torch_cuda, [e.entry for e in ex], [e.record for e in ex])
    assert bad == 0 and all(_slab(ts, j) == e.expected for j, e in enumerate(ex))


def test_verified_batches(torch_cuda, tiny):
    """wexb_batch_submit_verified: each record's stored bytes hashed (SHA-256) on the GPU against the digest
    given for it before its decode may write the destination. Right digests: bit-exact, as the plain
    batch; a wrong digest: that record alone refused with bit 32, its destination untouched; a damaged
    record whose digest matches its damaged bytes: refused by the stream hashes instead."""
    import hashlib
    blob, ex = tiny
    digests = [hashlib.sha256(e.record).digest() for e in ex]
    for _ in range(2):   # two calls in flight
        pending = []
        for d in (digests, [digests[0], bytes(32), digests[2]]):
            ts, sp, wp = _dst(torch_cuda, ex[0].entry, len(ex))
            pending.append((wexcuda.submit_batch_to_device([e.entry for e in ex], [e.record for e in ex], 0, sp, wp,
                                                           sha256=d), ts))
        (t0, ts0), (t1, ts1) = pending
        assert t1.wait()[1] == [0, -1, 0] and wexcuda.lib().wexb_last_error_bits() & 32
        assert t0.wait() == (0, [0, 0, 0])
        for j, e in enumerate(ex):
            assert _slab(ts0, j) == e.expected
        assert _slab(ts1, 0) == ex[0].expected and _slab(ts1, 2) == ex[2].expected
        assert _untouched(ts1, 1)
    damaged = bytearray(ex[2].record)
    damaged[7000] ^= 8
    ts, sp, wp = _dst(torch_cuda, ex[0].entry, 1)
    t = wexcuda.submit_batch_to_device([ex[2].entry], [bytes(damaged)], 0, sp, wp,
                                       sha256=[hashlib.sha256(bytes(damaged)).digest()])
    assert t.wait() == (1, [-1]) and _untouched(ts, 0)


def test_verified_windows(torch_cuda, tiny):
    """Verified calls gather in hash windows (at most 16 calls or 64 records a window): 20 calls in flight
    fill one window by their count and leave a partial one that the first wait queues; a wrong digest in
    a call of either window refuses only that record; waited in reverse order, every slab is bit-exact."""
    import hashlib
    blob, ex = tiny
    digests = [hashlib.sha256(e.record).digest() for e in ex]
    pending = []
    for c in range(20):
        d = list(digests)
        if c in (3, 18):
            d[1] = bytes(32)
        ts, sp, wp = _dst(torch_cuda, ex[0].entry, len(ex))
        pending.append((c, wexcuda.submit_batch_to_device([e.entry for e in ex], [e.record for e in ex], 0, sp, wp,
                                                          sha256=d), ts))
    for c, t, ts in reversed(pending):
        want = [0, -1, 0] if c in (3, 18) else [0, 0, 0]
        assert t.wait()[1] == want, c
        for j, e in enumerate(ex):
            if want[j] == 0:
                assert _slab(ts, j) == e.expected, (c, j)
            else:
                assert _untouched(ts, j), (c, j)


def test_upload_flags_shared_by_small_records(torch_cuda):
    """A call's records share an upload flag per 8 MiB: a call of 7 mid-shape records (2.3 MB each), one
    damaged and one refused on the host in the middle, has two flags each covering several records.
    Queued and synchronous, in turn and twice over (the flags' tokens advance per call of a workspace):
    every clean record bit-exact, the damaged and the refused ones -1 with their destinations
    untouched."""
    blob, mids = synth.make_experts(2048, 768, [(0, i) for i in range(6)], seed=77, sigma=0.02, train_every=1)
    assert wexcuda.register_model(blob) == 0
    damaged = bytearray(mids[3].record)
    damaged[9000] ^= 16
    bad_entry = bytearray(mids[4].entry)
    bad_entry[24] ^= 1   # a scale shape that does not match its record
    entries = [e.entry for e in mids] + [mids[0].entry]
    records = [e.record for e in mids] + [mids[5].record]
    records[3] = bytes(damaged)
    entries[4] = bytes(bad_entry)
    want = [0, 0, 0, -1, -1, 0, 0]   # the last: record 5 again, under record 0's entry (the same shape)
    for rep in range(2):
        for queued in (True, False):
            ts, sp, wp = _dst(torch_cuda, mids[0].entry, len(entries))
            if queued:
                bad, st = wexcuda.submit_batch_to_device(entries, records, 0, sp, wp).wait()
            else:
                bad, st = wexcuda.decode_batch_to_device(entries, records, 0, sp, wp)
            assert st == want and bad == 2, (rep, queued, st)
            for j, src in ((0, 0), (1, 1), (2, 2), (5, 5), (6, 5)):
                assert _slab(ts, j) == mids[src].expected, (rep, queued, j)
            for j in (3, 4):
                assert _untouched(ts, j), (rep, queued, j)


def test_queued_batches(torch_cuda, tiny):
    """wexb_batch_submit / wexb_batch_wait: several batches in flight, one with a damaged and an
    unavailable record; each wait gives the statuses of the synchronous call; tickets are single-use."""
    blob, ex = tiny
    other = synth.make_experts(1024, 512, [(0, 0)], seed=98, sigma=0.03, train_every=1)[1][0]   # unregistered model
    damaged = bytearray(ex[2].record); damaged[7000] ^= 8
    calls = [([e.entry for e in ex], [e.record for e in ex], [0, 0, 0]),
             ([ex[1].entry, other.entry, ex[2].entry], [ex[1].record, other.record, bytes(damaged)], [0, 1, -1]),
             ([ex[2].entry] * 2, [ex[2].record] * 2, [0, 0])]
    pending = []
    for _ in range(3):
        for entries, records, want in calls:
            ts, sp, wp = _dst(torch_cuda, entries[0], len(entries))
            pending.append((wexcuda.submit_batch_to_device(entries, records, 0, sp, wp), ts, records, want))
    for t, ts, records, want in reversed(pending):
        bad, st = t.wait()
        assert st == want and bad == sum(1 for s in want if s)
        for j, s in enumerate(st):
            if s == 0:
                x = next(e for e in ex if e.record == records[j])
                assert _slab(ts, j) == x.expected
            else:
                assert _untouched(ts, j)
    L = wexcuda.lib()
    assert L.wexb_batch_wait(pending[0][0].ticket, None) == -1
    assert L.wexb_batch_submit(0, None, None, 0, None, None) == -1
