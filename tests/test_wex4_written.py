"""WEX4 containers written by wex-wrn2_b200/wex4file.py for the tiny workload (8 WNR3 experts of hidden
1024 / FFN 512, sigma 0.02, plus one expert of uniform-random nibbles that the encoder stores RAW) and a
canonical-zero variant. CPU: the reference's own tool (oracle/_ref/wex4_tools_ref.so) accepts the file,
decodes it on the host, and its content digest equals the one computed from the source slabs. GPU: the
CUDA path (wex4_check, wex4_decode_record_buf) gives the same verdicts and digests, also for damaged
records (a flipped payload byte, with and without its record hash fixed)."""
import ctypes
import hashlib
import struct

import pytest

import oracle
import synth
import wex4file
import wexcuda

P, U32, U64, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int


def ref():
    L = oracle.ref_lib('wex4_tools_ref')
    if L is None:
        pytest.skip('reference tools not built (make -C oracle ref)')
    L.wex4_check.argtypes = [P, U64, I, P]
    L.wex4_validate.argtypes = [P, U64, P, SZ]
    return L


def lib():
    L = wexcuda.lib()
    L.wex4_check.argtypes = [P, U64, I, P]
    L.wex4_validate.argtypes = [P, U64, P, SZ]
    L.wex4_decode_record_buf.argtypes = [P, U64, P, SZ, U32, P, P, I, P]
    return L


def tiny_file(cz=False):
    """(file bytes, experts, records): 8 WNR3 experts and one RAW expert, canonical layout."""
    kw = dict(seed=4242 + cz, sigma=0.02, cz=cz, neg_zero=0.03 if cz else 0.0)
    blob, ex = synth.make_experts(1024, 512, [(0, i) for i in range(8)], train_every=1, **kw)
    ex += synth.make_experts(1024, 512, [(0, 8)], mode=1, blob=blob, **kw)[1]   # the model never saw it
    assert [e.codec for e in ex] == [5] * 8 + [0]
    recs = [wex4file.expert_record(e, 0, value_exact=cz) for e in ex]
    data = wex4file.write(recs, [(wex4file.BLOB_WNM2, oracle.lib().oracle_fnv1a(blob, len(blob)), blob)], grid=(1, 9),
                          value_exact=cz)
    return data, ex, recs


def test_written_file_is_accepted_and_decoded_by_the_reference():
    R = ref()
    for cz in (False, True):
        data, ex, recs = tiny_file(cz)
        f = oracle.Wex4File(data)
        assert R.wex4_validate(f.page, f.file_bytes, f.index, len(f.index)) == 0
        assert lib().wex4_validate(f.page, f.file_bytes, f.index, len(f.index)) == 0
        digest = ctypes.create_string_buffer(32)
        assert R.wex4_check(data, len(data), 3, digest) == 0
        assert digest.raw == wex4file.content_digest(recs, [e.expected for e in ex])


def _damaged(data, r, fix_hash):
    """The file with one payload byte of record r flipped (its index hash fixed on request, then the
    index and header hashes fixed so that only the record is at fault)."""
    f = oracle.Wex4File(data)
    rec = f.records[r]
    b = bytearray(data)
    b[rec['offset'] + 1000] ^= 0x20
    if fix_hash:
        new = hashlib.sha256(bytes(b[rec['offset']:rec['offset'] + rec['stored']])).digest()
        at = f.index_offset + 64 * f.nblobs + 72 * r + 36
        b[at:at + 32] = new
        index_bytes = struct.unpack_from('<Q', b, 40)[0]
        b[96:128] = hashlib.sha256(bytes(b[f.index_offset:f.index_offset + index_bytes])).digest()
        b[4064:4096] = hashlib.sha256(bytes(b[:4064])).digest()
    return bytes(b)


@pytest.mark.gpu
@pytest.mark.parametrize('cz', [False, True])
def test_gpu_check_matches_reference_on_written_files(cz):
    R, L = ref(), lib()
    data, ex, recs = tiny_file(cz)
    want = wex4file.content_digest(recs, [e.expected for e in ex])
    for flags in (1, 2, 3):
        d = ctypes.create_string_buffer(32)
        assert L.wex4_check(data, len(data), flags, d) == R.wex4_check(data, len(data), flags, None) == 0
        if flags & 2:
            assert d.raw == want
    for r, fix in [(0, False), (3, True), (8, False), (8, True)]:
        bad = _damaged(data, r, fix)
        for flags in (1, 2, 3):
            assert L.wex4_check(bad, len(bad), flags, None) == R.wex4_check(bad, len(bad), flags, None), (r, fix, flags)


@pytest.mark.gpu
def test_gpu_decode_record_buf_on_written_file():
    L = lib()
    data, ex, recs = tiny_file(True)
    f = oracle.Wex4File(data)
    for r, e in enumerate(ex):
        rec = f.records[r]
        out = ctypes.create_string_buffer(rec['decoded'])
        blob = f.blob(rec['blob'] - 1) if rec['blob'] else None
        assert L.wex4_decode_record_buf(f.page, f.file_bytes, f.index, len(f.index), r, f.stored(r), blob, 1, out) == 0
        assert out.raw == e.expected


def mixed_file():
    """(file, experts, records, blob4): records 0-5 WNR3 canonical-zero experts, 6-7 WNR4 kind-MX expert slabs
    (draft codec 8: non-EXPERT records owning themselves, encoded by the reference's WNR4 encoder, with a
    kind-3 WNM4 blob), 8 a RAW expert."""
    import numpy as np
    W = oracle.ref_lib('wnr4_tools')
    if W is None:
        pytest.skip('reference WNR4 tools not built (make -C oracle ref)')
    kw = dict(seed=777, sigma=0.02, cz=True, neg_zero=0.03)
    blob, ex = synth.make_experts(1024, 512, [(0, i) for i in range(8)], train_every=1, **kw)
    ex += synth.make_experts(1024, 512, [(0, 8)], mode=1, blob=blob, **kw)[1]
    import test_wnr4
    geo = (U32 * 13)(*test_wnr4.geo_of(ex[6].entry))
    counts = np.zeros(W.wnr4t_counts_words(0, 1), np.uint64)
    for e in ex[6:8]:
        assert W.wnr4t_count(geo, e.coded, 1, counts.ctypes.data) == 0
    blob4 = ctypes.create_string_buffer(W.wnr4t_model_bytes(0, 1))
    assert W.wnr4t_build(0, 1, counts.ctypes.data, blob4)
    h = W.wnr4t_model_open(blob4, len(blob4.raw))
    recs = [wex4file.expert_record(e, 0, value_exact=True) for e in ex[:6]]
    for r in (6, 7):
        e = ex[r]
        cap = 2 * len(e.coded) + (1 << 20)
        out = ctypes.create_string_buffer(cap)
        n = W.wnr4t_encode(h, geo, e.coded, e.flags, r, 32, out, cap)   # owner = the record's index
        assert n > 0
        recs.append(wex4file.expert_record(e, 1, codec=wex4file.CODEC_WNR4, stored=out.raw[:n]))
    W.wnr4t_model_close(h)
    recs.append(wex4file.expert_record(ex[8]))
    blob4 = blob4.raw
    blobs = [(wex4file.BLOB_WNM2, oracle.lib().oracle_fnv1a(blob, len(blob)), blob),
             (wex4file.BLOB_WNM4, oracle.lib().oracle_wnm4_id(blob4, len(blob4)), blob4)]
    data = wex4file.write(recs, blobs, grid=(1, 9), value_exact=True)
    return data, ex, recs


def test_mixed_file_is_accepted_by_the_reference():
    """The reference validates the mixed container and, not decoding codec 8, refuses its check with
    WEX4_E_UNSUPPORTED (-15) once it reaches record 6; the hashes alone pass."""
    R = ref()
    data, ex, recs = mixed_file()
    f = oracle.Wex4File(data)
    assert R.wex4_validate(f.page, f.file_bytes, f.index, len(f.index)) == 0
    assert R.wex4_check(data, len(data), 1, None) == 0
    assert R.wex4_check(data, len(data), 3, None) == -15


@pytest.mark.gpu
def test_gpu_check_decodes_codec8_on_request():
    R, L = ref(), lib()
    data, ex, recs = mixed_file()
    for flags in (1, 2, 3):
        assert L.wex4_check(data, len(data), flags, None) == R.wex4_check(data, len(data), flags, None)
    d = ctypes.create_string_buffer(32)
    assert L.wex4_check(data, len(data), 7, d) == 0
    assert d.raw == wex4file.content_digest(recs, [e.expected for e in ex])
    # a damaged WNR4 tile with its record hash fixed: refused by the decode (-14), hash-only passes
    bad = _damaged(data, 6, True)
    assert L.wex4_check(bad, len(bad), 5, None) == 0
    assert L.wex4_check(bad, len(bad), 7, None) == -14
    bad = _damaged(data, 7, False)
    assert L.wex4_check(bad, len(bad), 7, None) == -3


def test_bench_containers_are_valid_for_the_reference():
    """The containers bench.py times (tiny-file, and a 12-record prefix of a mixed step) pass the
    reference's validation; the tiny one decodes to the digest the bench verifies against."""
    import os
    import sys
    R = ref()
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    cfg = bench.CONFIGS['tiny-file']
    data, decoded, counts, vdata, vdigest = bench.build_container(cfg, bench.container_owners(cfg, 0, 1, 1), 4)
    assert counts == {0: 1, 5: 8, 8: 0}
    f = oracle.Wex4File(data)
    assert R.wex4_validate(f.page, f.file_bytes, f.index, len(f.index)) == 0
    d = ctypes.create_string_buffer(32)
    assert R.wex4_check(vdata, len(vdata), 3, d) == 0 and d.raw == vdigest
    cfg = dict(bench.CONFIGS['mixed'], hidden=1024, ffn=512)   # the mixed recipe at a small shape
    owners = bench.container_owners(cfg, 0, 1, 2)[:12]
    data, decoded, counts, vdata, vdigest = bench.build_container(cfg, owners, 4)
    f = oracle.Wex4File(data)
    assert R.wex4_validate(f.page, f.file_bytes, f.index, len(f.index)) == 0
    assert R.wex4_check(data, len(data), 1, None) == 0
    assert sum(counts.values()) == 12


@pytest.mark.gpu
def test_gpu_check_of_a_bench_mixed_container():
    """A small-shape mixed step (RAW, WNR4 kind MX and WNR3 canonical-zero records) checked and decoded on
    the GPU with codec 8 on: the content digest of its source slabs, and a throughput-pass check (no
    digest) that passes too."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    L = lib()
    cfg = dict(bench.CONFIGS['mixed'], hidden=1024, ffn=512)
    owners = bench.container_owners(cfg, 0, 1, 3)[:12]
    data, decoded, counts, vdata, vdigest = bench.build_container(cfg, owners, 4)
    assert counts[0] + counts[5] + counts[8] == 12 and counts[8] > 0
    d = ctypes.create_string_buffer(32)
    assert L.wex4_check(vdata, len(vdata), 7, d) == 0 and d.raw == vdigest
    assert L.wex4_check(data, len(data), 15, None) == 0
