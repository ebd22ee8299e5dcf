"""The GPU record writer (wexb_encode_batch, wexb_count_batch) against the writer tools' CPU encoder and
counter (byte-identical to the reference's wex_nr3_encode_record and counts: tests/test_synth_encoder.py)
and, where it is built, against the reference encoder itself. Covers WNR3 in both canonical-zero modes,
WNR2, every chunk pair the format allows at its ends, the RAW verdict, the refusals, and a round trip
through the GPU decoder."""
import ctypes

import numpy as np
import pytest

import oracle
import synth
import wexcuda


def _experts(hidden, ffn, n, cz, chunks=(2048, 512), nr3=True, seed=21):
    blob, ex = synth.make_experts(hidden, ffn, [(0, i) for i in range(n)], seed=seed, sigma=0.02, cz=cz,
                                  neg_zero=0.03 if cz else 0.0, train_every=1, wchunk=chunks[0], schunk=chunks[1],
                                  nr3=nr3)
    return blob, ex


def _encode(blob, ex, chunks=(2048, 512), nr3=True, **kw):
    return wexcuda.encode_batch(blob, [e.entry for e in ex], [e.coded for e in ex], [e.flags for e in ex],
                                [e.owner if nr3 else 0 for e in ex], nr3, chunks[0], chunks[1], **kw)


def test_refusals_before_the_device():
    blob, ex = _experts(256, 128, 1, False)
    bad = bytearray(blob)
    bad[32] ^= 1   # the first CDF entry of context 0 is no longer 0: the model does not validate
    assert [r[0] for r in _encode(bytes(bad), ex)] == [-1]
    assert [r[0] for r in _encode(blob, ex, chunks=(2048, 100))] == [-1]   # schunk not a power of two >= 256
    assert wexcuda.encode_batch(blob, [], [], [], []) == []


@pytest.mark.gpu
@pytest.mark.parametrize('cz', [False, True])
@pytest.mark.parametrize('chunks', [(2048, 512), (512, 256), (4096, 1024), (16384, 16384)])
def test_gpu_records_equal_the_cpu_encoder(cz, chunks):
    blob, ex = _experts(1024, 512, 3, cz, chunks)
    ex += synth.make_experts(1024, 512, [(0, 3)], seed=21, sigma=0.02, cz=cz, mode=1, blob=blob,
                             wchunk=chunks[0], schunk=chunks[1])[1]   # uniform nibbles: stored RAW
    res = _encode(blob, ex, chunks)
    for e, (st, rec, used, total) in zip(ex, res):
        if e.codec == synth.CODEC_RAW:
            assert st == 1 and rec is None and total >= len(e.record)
        else:
            assert st == 0 and rec == e.record and total == len(rec) and used <= total
    L = oracle.ref_lib('wex_nr3_tools')
    if L is not None:   # and the reference's own encoder
        e = ex[0]
        cap = 4 * len(e.coded) + 65536
        out = ctypes.create_string_buffer(cap)
        used, total = ctypes.c_size_t(), ctypes.c_size_t()
        assert L.wex_nr3_encode_record(blob, e.entry, e.coded, e.flags, e.owner, chunks[0], chunks[1], out, cap,
                                       ctypes.byref(used), ctypes.byref(total)) == 0
        assert out.raw[:total.value] == res[0][1]


@pytest.mark.gpu
def test_gpu_wnr2_and_mid_shape_records():
    blob, ex = _experts(1024, 512, 2, False, nr3=False)
    assert [r[1] for r in _encode(blob, ex, nr3=False)] == [e.record for e in ex]
    blob, ex = _experts(2048, 768, 2, True, seed=5)
    res = _encode(blob, ex)
    assert [r[1] for r in res] == [e.record for e in ex]
    # round trip through the GPU decoder
    import torch
    raw = len(ex[0].expected)
    dst = torch.empty((2, raw), dtype=torch.uint8, device='cuda')
    soff = [int.from_bytes(ex[0].entry[44 + 4 * m:48 + 4 * m], 'little') for m in range(3)]
    woff = [int.from_bytes(ex[0].entry[56 + 4 * m:60 + 4 * m], 'little') for m in range(3)]
    ds = [dst.data_ptr() + j * raw + o for j in range(2) for o in soff]
    dw = [dst.data_ptr() + j * raw + o for j in range(2) for o in woff]
    assert wexcuda.register_model(blob) == 0
    bad, st = wexcuda.decode_batch_to_device([e.entry for e in ex], [r[1] for r in res], 0, ds, dw)
    assert bad == 0, st
    assert [bytes(dst[j].cpu().numpy()) for j in range(2)] == [e.expected for e in ex]


@pytest.mark.gpu
def test_gpu_refusals_per_record():
    blob, ex = _experts(1024, 512, 3, False)
    # record 0: a -0 nibble in a record flagged canonical zero; record 1: cap below its size
    w = bytearray(ex[0].coded)
    w[len(w) - 1] = (w[-1] & 0x0f) | 0x80
    coded = [bytes(w), ex[1].coded, ex[2].coded]
    flags = [ex[0].flags | 8, ex[1].flags, ex[2].flags]
    res = wexcuda.encode_batch(blob, [e.entry for e in ex], coded, flags, [e.owner for e in ex], True,
                               caps=[4 * len(w), 4096, 4 * len(w)])
    assert [r[0] for r in res] == [-1, -1, 0]
    assert res[2][1] == ex[2].record


@pytest.mark.gpu
@pytest.mark.parametrize('nr3', [True, False])
def test_gpu_counts_equal_the_cpu_counts(nr3):
    blob, ex = _experts(1024, 512, 3, nr3, nr3=nr3, seed=8)
    wc = np.zeros(3 * 567 * 16, np.uint64)
    sc = np.zeros(3 * 256, np.uint64)
    for e in ex:
        assert synth.tools().wexb_count_expert(e.entry, e.coded, 1 if nr3 else 0, wc.ctypes.data, sc.ctypes.data) == 0
    st, gwc, gsc = wexcuda.count_batch([e.entry for e in ex], [e.coded for e in ex], nr3)
    assert st == [0, 0, 0]
    assert np.array_equal(gwc, wc) and np.array_equal(gsc, sc)
    built = ctypes.create_string_buffer(synth.MODEL_BYTES)
    assert synth.tools().wexb_build_model(gwc.ctypes.data, gsc.ctypes.data, built) != 0
    assert built.raw == blob
