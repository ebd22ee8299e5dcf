"""The writer-side tools (synthetic experts, WNR3 encoder) against the reference's own encoder and
decoder (oracle/_ref, compiled from the reference sources) and the oracle restatement."""
import ctypes

import numpy as np
import pytest

import oracle
import synth

SHAPES = [(256, 128), (1024, 512)]


def _ref_tools():
    L = oracle.ref_lib('wex_nr3_tools')
    if L is None:
        pytest.skip('reference tools not built (make -C oracle ref)')
    return L


def test_mxfp4_generator_is_seeded_and_sane():
    a = synth.synth_expert(1024, 512, seed=7, sigma=0.02)
    b = synth.synth_expert(1024, 512, seed=7, sigma=0.02)
    c = synth.synth_expert(1024, 512, seed=8, sigma=0.02)
    assert a == b and a != c and len(a) == 835584
    e = synth.expert_entry(1024, 512)
    s = np.frombuffer(a[:49152 // 3 * 3], np.uint8)
    # sigma 0.02: amax of 32 normals ~ 2.1 sigma -> exponent floor(log2 0.042) - 2 = -7 -> byte 120
    assert 115 <= np.median(s) <= 124
    w = np.frombuffer(a[49152:], np.uint8)
    nib = np.concatenate([w & 15, w >> 4])
    assert (nib == 8).sum() == 0          # no -0 from the quantizer
    assert 0 < (nib & 7).max() <= 7 and (nib & 7).mean() > 1


def test_neg_zero_injection():
    a = synth.synth_expert(1024, 512, seed=3, sigma=0.02, neg_zero=0.03)
    w = np.frombuffer(a[49152:], np.uint8)
    nib = np.concatenate([w & 15, w >> 4])
    frac = (nib == 8).sum() / ((nib == 8).sum() + (nib == 0).sum())
    assert 0.02 < frac < 0.04


@pytest.mark.parametrize('hidden,ffn', SHAPES)
@pytest.mark.parametrize('cz', [False, True])
@pytest.mark.parametrize('chunks', [(2048, 512), (512, 256), (4096, 1024)])
def test_encoder_bytes_equal_reference_encoder(hidden, ffn, cz, chunks):
    """Same coded slab, same model, same chunks: the record bytes equal wex_nr3_encode_record's."""
    L = _ref_tools()
    owners = [(0, i) for i in range(3)]
    blob, experts = synth.make_experts(hidden, ffn, owners, seed=11, sigma=0.02, cz=cz, neg_zero=0.03 if cz else 0,
                                       train_every=1, wchunk=chunks[0], schunk=chunks[1])
    # the reference's prepare, counts and model build give the same coded bytes and model
    wc = np.zeros(3 * 567 * 16, np.uint64); sc = np.zeros(3 * 256, np.uint64)
    for e in experts:
        coded = ctypes.create_string_buffer(len(e.source))
        flags = L.wex_nr3_prepare(e.entry, e.source, 1 if cz else 0, coded, None)
        assert flags == e.flags and coded.raw == e.coded
        assert L.wex_nr3_count_expert(e.entry, coded, wc.ctypes.data, sc.ctypes.data) == 0
    ref_blob = ctypes.create_string_buffer(synth.MODEL_BYTES)
    assert L.wex_nr3_build_model(wc.ctypes.data, sc.ctypes.data, ref_blob, None) == 0
    assert ref_blob.raw == blob
    for e in experts:
        cap = 4 * len(e.coded) + 65536
        out = ctypes.create_string_buffer(cap)
        used, total = ctypes.c_size_t(), ctypes.c_size_t()
        st = L.wex_nr3_encode_record(blob, e.entry, e.coded, e.flags, e.owner, chunks[0], chunks[1], out, cap,
                                     ctypes.byref(used), ctypes.byref(total))
        assert st == (0 if e.codec == 5 else 1)
        if st == 0:
            assert out.raw[:total.value] == e.record


@pytest.mark.parametrize('cz', [False, True])
def test_records_decode_with_reference_and_oracle(cz):
    L = _ref_tools()
    blob, experts = synth.make_experts(1024, 512, [(2, i) for i in range(4)], seed=5, sigma=0.03, cz=cz,
                                       neg_zero=0.03 if cz else 0, train_every=2)
    for e in experts:
        assert e.codec == 5
        out = ctypes.create_string_buffer(len(e.source))
        assert L.wex_nr3_decode(blob, e.entry, e.record, e.layer, e.index, out) == 0
        assert out.raw == e.expected
        st, where, slab = oracle.nrx_decode(blob, e.entry, e.record, len(e.source))
        assert st == 0 and slab == e.expected, where


def test_wnr2_records_decode_with_oracle():
    blob, experts = synth.make_experts(1024, 512, [(0, i) for i in range(2)], seed=9, nr3=False, train_every=1)
    for e in experts:
        assert e.codec == 4
        st, where, slab = oracle.nrx_decode(blob, e.entry, e.record, len(e.source))
        assert st == 0 and slab == e.source, where


def test_incompressible_expert_falls_back_to_raw():
    blob, experts = synth.make_experts(1024, 512, [(0, 0), (0, 1)], seed=2, mode=lambda i: i, train_every=2)
    assert experts[0].codec == 5 and experts[1].codec == 0
    assert experts[1].record[:len(experts[1].source)] == experts[1].source
