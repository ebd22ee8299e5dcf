"""The WEX4 container ABI (include/wex4_tools.h) against the reference's own compiled tool
(oracle/_ref/wex4_tools_ref.so) and the reference's conformance manifest.

CPU tests (no decode): header and index validation of every vector the reference ships (read from
the reference tree when it is present, else the copies under tests/golden/vectors), the legacy expert
table, and wex4_check without hashes or decode. GPU tests: wex4_check with record hashes and decodes
(content digests), and wex4_decode_record_buf record by record."""
import ctypes
import json
import os

import pytest

import oracle
import wexcuda

REF_VECTORS = os.path.join(oracle.REFERENCE, 'wex4', 'vectors')
P, U32, U64, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int
def lib():
    L = wexcuda.lib()
    L.wex4_tools_abi.restype = U32
    L.wex4_check.argtypes = [P, U64, I, P]
    L.wex4_fuzz_check.argtypes = [P, U64, I, P]
    L.wex4_validate.argtypes = [P, U64, P, SZ]
    L.wex4_decode_record_buf.argtypes = [P, U64, P, SZ, U32, P, P, I, P]
    L.wex4_expert_table.argtypes = [P, U64, P, SZ, P]
    L.wex4_sha256_bytes.argtypes = [P, SZ, P]
    return L


def all_vectors(golden_dir):
    """(relative path, bytes, manifest row) of every vector available here."""
    if os.path.isdir(REF_VECTORS):
        rows = [l.rstrip('\n').split('\t') for l in open(os.path.join(REF_VECTORS, 'MANIFEST.tsv'), encoding='utf-8')
                if l.strip() and not l.startswith('#')]
        for row in rows:
            p = os.path.join(REF_VECTORS, row[0])
            if os.path.exists(p):
                yield row[0], open(p, 'rb').read(), row
    else:
        for name, item in sorted(json.load(open(os.path.join(golden_dir, 'vectors.json'))).items()):
            yield item['path'], open(os.path.join(golden_dir, 'vectors', name), 'rb').read(), \
                [item['path'], item['verdict'], item['cls'], item['root'], item['sha256'], '-', item['content']]


def index_of(data):
    """(page, file_bytes, index as read from disk) of a file, or None when the header is unusable."""
    if len(data) < 4096:
        return None
    f = oracle.Wex4File.__new__(oracle.Wex4File)
    import struct
    file_bytes, index_offset, index_bytes = struct.unpack_from('<QQQ', data, 24)
    n = (index_bytes + 4095) & ~4095
    if index_offset > len(data) or n > 1 << 30:
        return data[:4096], len(data), b''
    return data[:4096], len(data), data[index_offset:index_offset + n].ljust(n, b'\0')


def test_sha256_bytes():
    import hashlib
    out = ctypes.create_string_buffer(32)
    for n in (0, 1, 55, 56, 64, 4064, 100001):
        data = bytes((i * 7 + 3) & 255 for i in range(n))
        lib().wex4_sha256_bytes(data, n, out)
        assert out.raw == hashlib.sha256(data).digest()


def test_validate_matches_reference_on_every_vector(golden_dir):
    ref = oracle.ref_lib('wex4_tools_ref')
    if ref is None:
        pytest.skip('reference tools not built')
    L = lib()
    n = 0
    for path, data, row in all_vectors(golden_dir):
        ix = index_of(data)
        if ix is None:
            continue
        page, fb, index = ix
        assert L.wex4_validate(page, fb, index, len(index)) == ref.wex4_validate(page, fb, index, len(index)), path
        n += 1
    assert n >= 25


def test_check_without_hashes_matches_reference(golden_dir):
    """wex4_check with flags 0 (header, index, blobs and models; no GPU work) on every vector."""
    ref = oracle.ref_lib('wex4_tools_ref')
    if ref is None:
        pytest.skip('reference tools not built')
    L = lib()
    for path, data, row in all_vectors(golden_dir):
        assert L.wex4_check(data, len(data), 0, None) == ref.wex4_check(data, len(data), 0, None), path


def test_guarded_check_without_hashes_matches_reference(golden_dir):
    """wex4_fuzz_check (the same check on a copy that ends at an inaccessible page) with flags 0, on every
    vector: the reference's guard-paged verdict, and never a fault from a read past the file's end."""
    ref = oracle.ref_lib('wex4_tools_ref')
    L = lib()
    n = 0
    for path, data, row in all_vectors(golden_dir):
        got = L.wex4_fuzz_check(data, len(data), 0, None)
        assert got == L.wex4_check(data, len(data), 0, None), path
        if ref is not None:
            assert got == ref.wex4_fuzz_check(data, len(data), 0, None), path
        n += 1
        for cut in (1, 4096):   # truncated copies end at the guard page too
            if len(data) > cut:
                assert L.wex4_fuzz_check(data[:-cut], len(data) - cut, 0, None) == \
                    L.wex4_check(data[:-cut], len(data) - cut, 0, None), (path, cut)
    assert n >= 25


def test_expert_table_matches_reference(golden_dir):
    ref = oracle.ref_lib('wex4_tools_ref')
    if ref is None:
        pytest.skip('reference tools not built')
    L = lib()
    for path, data, row in all_vectors(golden_dir):
        if row[1] != 'accept':
            continue
        page, fb, index = index_of(data)
        f = oracle.Wex4File(data)
        cap = max(1, f.layers * f.experts * 72)
        a, b = ctypes.create_string_buffer(cap), ctypes.create_string_buffer(cap)
        sa = L.wex4_expert_table(page, fb, index, len(index), a)
        sb = ref.wex4_expert_table(page, fb, index, len(index), b)
        assert sa == sb and a.raw == b.raw, path


@pytest.mark.gpu
@pytest.mark.parametrize('flags', [1, 2, 3])
def test_check_with_hashes_and_decode(golden_dir, flags):
    """Verdict, class and content digest of wex4_check equal the reference's on every vector, the WBP1
    (codec 6) ones included."""
    import torch
    assert torch.cuda.is_available()
    L = lib()
    items = json.load(open(os.path.join(golden_dir, 'vectors.json')))
    checked = 0
    for name, item in sorted(items.items()):
        data = open(os.path.join(golden_dir, 'vectors', name), 'rb').read()
        digest = ctypes.create_string_buffer(32)
        st = L.wex4_check(data, len(data), flags, digest)
        guarded = ctypes.create_string_buffer(32)
        assert L.wex4_fuzz_check(data, len(data), flags, guarded) == st, (name, flags)
        assert guarded.raw == digest.raw, name
        ref = oracle.ref_lib('wex4_tools_ref')
        want = ref.wex4_check(data, len(data), flags, None) if ref is not None else (item['ref_check'] if flags == 3 else None)
        if want is not None:
            assert st == want, (name, flags, st, want)
        if flags & 2 and item['verdict'] == 'accept':
            assert st == 0 and digest.raw.hex() == item['content'], name
        checked += 1
    assert checked >= 20


@pytest.mark.gpu
def test_decode_record_buf_matches_reference(golden_dir):
    import hashlib
    L = lib()
    items = json.load(open(os.path.join(golden_dir, 'vectors.json')))
    n = 0
    for name, item in sorted(items.items()):
        if not item['records']:
            continue
        data = open(os.path.join(golden_dir, 'vectors', name), 'rb').read()
        f = oracle.Wex4File(data)
        for rr in item['records']:
            rec = f.records[rr['r']]
            out = ctypes.create_string_buffer(rec['decoded'])
            blob = f.blob(rec['blob'] - 1) if rec['blob'] else None
            st = L.wex4_decode_record_buf(f.page, f.file_bytes, f.index, len(f.index), rr['r'], f.stored(rr['r']), blob, 1,
                                          out)
            assert st == rr['ref_status'], (name, rr['r'], st)
            if st == 0:
                assert hashlib.sha256(out.raw).hexdigest() == rr['ref_sha'], (name, rr['r'])
            n += 1
    assert n >= 60
