"""Seeded mutants of written containers, in the three modes of the reference's in-process fuzzer
(wex4/wex4_tools.c:250-312): 0, one bit of any byte of the file; 1, one bit of a compressed record
with its index hash and the header resealed, so that only the decode can refuse it; 2, one bit of the
header page or of the index, resealed. Every mutant gets the reference tool's verdict from the GPU
check, and when both accept, the same content digest. Then the helper under thread churn: decode
calls from 8 host threads at once keep the device memory bounded (the reference's GPU test allows
64 MiB of growth, c/tests/test_wex_nr3_gpu.cu:318)."""
import ctypes
import hashlib
import random
import struct
import threading

import pytest

import oracle
import synth
import wexcuda
from test_wex4_written import lib, ref, tiny_file


def _reseal(b, f):
    index_bytes = struct.unpack_from('<Q', b, 40)[0]
    b[96:128] = hashlib.sha256(bytes(b[f.index_offset:f.index_offset + index_bytes])).digest()
    b[4064:4096] = hashlib.sha256(bytes(b[:4064])).digest()


def mutants(data, n, seed):
    f = oracle.Wex4File(data)
    rng = random.Random(seed)
    coded = [r for r, rec in enumerate(f.records) if rec['codec'] != 0]
    index_bytes = struct.unpack_from('<Q', data, 40)[0]
    for i in range(n):
        mode = i % 3
        b = bytearray(data)
        bit = 1 << rng.randrange(8)
        if mode == 0:
            b[rng.randrange(len(b))] ^= bit
        elif mode == 1:
            r = rng.choice(coded)
            rec = f.records[r]
            b[rec['offset'] + rng.randrange(rec['stored'])] ^= bit
            at = f.index_offset + 64 * f.nblobs + 72 * r + 36
            b[at:at + 32] = hashlib.sha256(bytes(b[rec['offset']:rec['offset'] + rec['stored']])).digest()
            _reseal(b, f)
        else:
            at = rng.randrange(4064) if rng.random() < 0.3 else f.index_offset + rng.randrange(index_bytes)
            b[at] ^= bit
            _reseal(b, f)
        yield mode, bytes(b)


def test_mutants_are_mutants():
    data, ex, recs = tiny_file(False)
    seen = [m for _, m in mutants(data, 12, 5)]
    assert all(m != data and len(m) == len(data) for m in seen) and len(set(seen)) == 12


@pytest.mark.gpu
@pytest.mark.parametrize('cz', [False, True])
def test_gpu_mutants_get_the_reference_verdict(cz):
    R, L = ref(), lib()
    data, ex, recs = tiny_file(cz)
    verdicts = {}
    for mode, m in mutants(data, 60, 1000 + cz):
        d1, d2 = ctypes.create_string_buffer(32), ctypes.create_string_buffer(32)
        a = L.wex4_check(m, len(m), 3, d1)
        b = R.wex4_check(m, len(m), 3, d2)
        assert a == b, (mode, a, b)
        if a == 0:
            assert d1.raw == d2.raw, mode
        verdicts.setdefault(mode, set()).add(a)
    # the modes reach different checks: the record hash (mode 0), the decode (mode 1), the index (mode 2)
    assert -3 in verdicts[0] and -14 in verdicts[1] and verdicts[2] - {0}


@pytest.mark.gpu
def test_gpu_thread_churn_keeps_memory_bounded():
    import torch
    blob, ex = synth.make_experts(1024, 512, [(0, i) for i in range(4)], seed=31, sigma=0.02, train_every=1)
    assert wexcuda.register_model(blob) == 0
    raw = len(ex[0].expected)
    so = [int.from_bytes(ex[0].entry[44 + 4 * m:48 + 4 * m], 'little') for m in range(3)]
    wo = [int.from_bytes(ex[0].entry[56 + 4 * m:60 + 4 * m], 'little') for m in range(3)]
    dst = torch.empty((8, 4, raw), dtype=torch.uint8, device='cuda')
    errors = []

    def worker(t, calls):
        try:
            for _ in range(calls):
                ds = [dst[t, j].data_ptr() + o for j in range(4) for o in so]
                dw = [dst[t, j].data_ptr() + o for j in range(4) for o in wo]
                bad, st = wexcuda.decode_batch_to_device([e.entry for e in ex], [e.record for e in ex], 0, ds, dw)
                if bad:
                    errors.append(st)
        except Exception as exc:   # reported below
            errors.append(repr(exc))

    def churn(calls):
        ts = [threading.Thread(target=worker, args=(t, calls)) for t in range(8)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    churn(2)   # the workspaces of 8 concurrent callers
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    churn(25)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert not errors, errors[:3]
    assert free0 - free1 <= 64 << 20, (free0 - free1) >> 20
    for t in range(8):
        assert all(bytes(dst[t, j].cpu().numpy()) == ex[j].expected for j in range(4))
