"""The largest expert shape of the workloads (hidden 7168, FFN 2048: 23,396,352 decoded bytes, 24,192
streams, a 48,384-byte length table), canonical zero with injected -0 nibbles. CPU: the oracle decodes
the record to the expected slab. GPU: the record decodes bit-exactly through the batch entry point, the
resident set and the no-allocation entry point; the GPU writer gives the same record bytes; a flipped
payload byte is refused with the destination untouched."""
import hashlib

import numpy as np
import pytest

import oracle
import synth
import wexcuda

POISON = 0x5A


@pytest.fixture(scope='module')
def large():
    blob, ex = synth.make_experts(7168, 2048, [(3, 17)], seed=77, sigma=0.02, cz=True, neg_zero=0.03, train_every=1)
    e = ex[0]
    assert e.codec == synth.CODEC_WNR3 and len(e.expected) == 23396352
    return blob, e


def test_oracle_decodes_the_largest_record(large):
    blob, e = large
    st, where, slab = oracle.nrx_decode(blob, e.entry, e.record, len(e.expected))
    assert st == 0, where
    assert hashlib.sha256(slab).digest() == hashlib.sha256(e.expected).digest()


def _regions(entry):
    b = bytes(entry)
    soff = [int.from_bytes(b[44 + 4 * m:48 + 4 * m], 'little') for m in range(3)]
    woff = [int.from_bytes(b[56 + 4 * m:60 + 4 * m], 'little') for m in range(3)]
    return soff, woff


@pytest.mark.gpu
def test_gpu_largest_record_every_entry_point(large):
    import ctypes
    import torch
    blob, e = large
    assert wexcuda.register_model(blob) == 0
    raw = len(e.expected)
    want = hashlib.sha256(e.expected).digest()
    soff, woff = _regions(e.entry)

    def fresh():
        slab = torch.full((raw,), POISON, dtype=torch.uint8, device='cuda')
        return slab, [slab.data_ptr() + o for o in soff], [slab.data_ptr() + o for o in woff]

    def digest(slab):
        torch.cuda.synchronize()
        return hashlib.sha256(bytes(slab.cpu().numpy())).digest()
    # the drop-in batch call
    slab, ds, dw = fresh()
    bad, st = wexcuda.decode_batch_to_device([e.entry], [e.record], 0, ds, dw)
    assert bad == 0 and digest(slab) == want
    # the resident set
    r = wexcuda.Resident([e.entry], [e.record], 0)
    assert r.failures == 0
    slab, ds, dw = fresh()
    assert r.decode([0], ds, dw) == 0
    assert r.wait() == (0, [0])
    assert digest(slab) == want
    r.close()
    # the no-allocation entry point (records up to 24 MiB)
    L = wexcuda.lib()
    L.wexb_decode_to_device_noalloc.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] + [ctypes.c_void_p] * 2
    slab, ds, dw = fresh()
    ent = np.frombuffer(bytes(e.entry), np.uint8).copy()
    rec = np.frombuffer(e.record, np.uint8)
    assert L.wexb_decode_to_device_noalloc(ent.ctypes.data, rec.ctypes.data, 0, wexcuda._ptrs(ds), wexcuda._ptrs(dw)) == 0
    assert digest(slab) == want
    # a flipped payload byte: refused, destination untouched
    bad_rec = bytearray(e.record)
    bad_rec[len(bad_rec) // 2] ^= 0x10
    slab, ds, dw = fresh()
    bad, st = wexcuda.decode_batch_to_device([e.entry], [bytes(bad_rec)], 0, ds, dw)
    torch.cuda.synchronize()
    assert st == [-1] and bool((slab == POISON).all())


@pytest.mark.gpu
def test_gpu_writer_on_the_largest_record(large):
    blob, e = large
    res = wexcuda.encode_batch(blob, [e.entry], [e.coded], [e.flags], [e.owner])
    assert res[0][0] == 0 and res[0][1] == e.record
    st, wc, sc = wexcuda.count_batch([e.entry], [e.coded])
    ref_wc = np.zeros(3 * 567 * 16, np.uint64)
    ref_sc = np.zeros(3 * 256, np.uint64)
    assert synth.tools().wexb_count_expert(e.entry, e.coded, 1, ref_wc.ctypes.data, ref_sc.ctypes.data) == 0
    assert st == [0] and np.array_equal(wc, ref_wc) and np.array_equal(sc, ref_sc)
