"""Pins the oracle (the C restatement under oracle/) before anything is checked against it:
the reference's hash known answers, SHA-256 test vectors, and the reference decoder's own results
on its WNR3 conformance vectors (committed under tests/golden/)."""
import hashlib
import json
import os
import struct

import pytest

import oracle


def test_murmur3_smhasher_verification_value():
    # c/tests/test_wex_format.c:668-676: SMHasher's Murmur3A verification value
    key = bytes(range(256))
    hashes = b''.join(struct.pack('<I', oracle.murmur3(key[:i], 256 - i)) for i in range(256))
    assert oracle.murmur3(hashes, 0) == 0xB0F57EE3


def test_murmur3_known_answers():
    # c/tests/test_wex_format.c:677-679
    key = bytes(range(16))
    assert oracle.murmur3(b'', 0) == 0
    assert oracle.murmur3(b'', 0x33524E57) == 0xE7F741F1
    assert oracle.murmur3(key, 0x33524E57) == 0x31CE0919


def test_stream_x0_known_answers():
    # c/tests/test_wex_format.c:680-684: stream end states (ident = model, owner, g, word24)
    ident = [0x299DC586, 0x00270078, 2165, 0x0F787978]
    data = bytes(((37 * i + 11) & 0x77) for i in range(1024))
    assert oracle.nr3_x0(ident, data) == 0x00E485B2
    ident[2] = 719
    assert oracle.nr3_x0(ident, bytes([0x7F, 0x7E, 0x80, 0x7F, 0x7D])) == 0x00C976D8


def test_rule_g_anchor():
    # c/tests/test_wex_format.c:685-688
    assert oracle.anchor(bytes([10, 11, 20, 21])) == 10
    assert oracle.anchor(bytes([5, 5, 6, 7, 7])) == 5
    assert oracle.anchor(bytes([254, 255, 255])) == 254


@pytest.mark.parametrize('n', [0, 1, 3, 55, 56, 63, 64, 65, 119, 120, 128, 1000, 4096, 100003])
def test_sha256_matches_fips(n):
    data = bytes((i * 131 + 7) & 0xFF for i in range(n))
    assert oracle.sha256(data) == hashlib.sha256(data).digest()


def _vectors(golden_dir):
    return json.load(open(os.path.join(golden_dir, 'vectors.json')))


def _container_ok(f, r, rec, stored, blob_id):
    """The cross-checks wex4_decode_record makes before the codec (c/wex4.h:693-695)."""
    if rec['codec'] != 5:
        return True
    return (struct.unpack_from('<I', stored, 28)[0] == rec['owner'] and
            bool(stored[27] & 8) == bool(rec['flags'] & 1) and
            struct.unpack_from('<I', stored, 4)[0] == blob_id)


def test_oracle_matches_reference_decoder_on_vectors(golden_dir):
    """Every expert record of the conformance vectors: the oracle's verdict and bytes equal the
    reference decoder's (wex4_decode_record_buf, whose results make_golden.py recorded)."""
    checked = 0
    for name, item in sorted(_vectors(golden_dir).items()):
        data = open(os.path.join(golden_dir, 'vectors', name), 'rb').read()
        assert hashlib.sha256(data).hexdigest() == item['sha256']
        if not item['records']:
            continue
        f = oracle.Wex4File(data)
        for rr in item['records']:
            rec = f.records[rr['r']]
            stored = f.stored(rr['r'])
            if rec['codec'] == 0:
                ok = not any(stored[rec['decoded']:])
                assert (0 if ok else -14) == rr['ref_status']
                if ok:
                    assert hashlib.sha256(stored[:rec['decoded']]).hexdigest() == rr['ref_sha']
                continue
            blob = f.blob(rec['blob'] - 1)
            st, where, slab = oracle.nrx_decode(blob, bytes.fromhex(rr['entry']), stored, rec['decoded'])
            verdict = 0 if (st == 0 and _container_ok(f, rr['r'], rec, stored, f.blobs[rec['blob'] - 1]['id'])) else -14
            assert verdict == rr['ref_status'], (name, rr['r'], where)
            if verdict == 0:
                assert hashlib.sha256(slab).hexdigest() == rr['ref_sha'], (name, rr['r'])
            checked += 1
    assert checked >= 20


def test_oracle_content_digest_of_valid_vectors(golden_dir):
    """Content digests of the accepted expert vectors, rebuilt from oracle decodes, equal the
    reference manifest's column 7."""
    for name, item in sorted(_vectors(golden_dir).items()):
        if item['verdict'] != 'accept':
            continue
        data = open(os.path.join(golden_dir, 'vectors', name), 'rb').read()
        f = oracle.Wex4File(data)
        decoded = []
        for r, rec in enumerate(f.records):
            stored = f.stored(r)
            assert oracle.sha256(stored) == rec['sha']
            if rec['codec'] == 0:
                decoded.append(stored[:rec['decoded']])
            elif rec['codec'] == 5:
                st, _, slab = oracle.nrx_decode(f.blob(rec['blob'] - 1), f.expert_entry(r), stored, rec['decoded'])
                assert st == 0
                decoded.append(slab)
            else:
                pytest.fail(f'codec {rec["codec"]} in {name}')
        assert oracle.content_digest(f, decoded).hex() == item['content'], name
