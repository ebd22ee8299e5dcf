"""Builds tests/golden/ from the reference project (run in a container that has it; the GPU host
never runs this). Writes:

  vectors/<name>.wex4   the reference's WEX4 conformance vectors that hold expert records (its
                        wex4/vectors/, Apache-2.0, copied byte for byte with their manifest rows)
  vectors.json          per file: the manifest verdict, class, root and content digest; per expert
                        record: codec, owner, the 72-byte legacy entry, and the reference decoder's
                        status and SHA-256 of its decoded bytes (oracle/_ref/wex4_tools_ref.so, the
                        reference's wex4_decode_record_buf, record hash checked)
  synth.json            seeded synthetic MXFP4 experts encoded by the reference WNR3 encoder
                        (oracle/_ref/wex_nr3_tools.so) at several chunk pairs, with and without
                        canonical zero: the SHA-256 of every encoded record and of its decode

Usage:  python tests/golden/make_golden.py [--reference /root/reference]
"""
import argparse
import ctypes
import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, 'oracle'))
import oracle  # noqa: E402

# the vectors of the reference's manifest that hold expert records, valid and refused
PICK_VALID = ['valid/wnr3-one-expert.wex4', 'valid/wnr3-ceil-form-chunk-pairs-and-anchors.wex4',
              'valid/tiny2-cz-upgraded.wex4', 'valid/tiny-raw-upgraded.wex4']


def pick(row):
    path, verdict, cls = row[0], row[1], row[2]
    if path in PICK_VALID:
        return True
    if not path.startswith('invalid/'):
        return False
    return any(k in path for k in ('wnr3', 'wnm2', 'canonical-zero', 'value-exact', 'raw-expert')) or cls == 'WEX4_E_DATA'


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', default='/root/reference')
    a = ap.parse_args()
    vec = os.path.join(a.reference, 'wex4', 'vectors')
    oracle.build()
    ref = oracle.ref_lib('wex4_tools_ref')
    assert ref is not None and ref.wex4_tools_abi() == 1
    out_dir = os.path.join(HERE, 'vectors')
    os.makedirs(out_dir, exist_ok=True)
    rows = [l.rstrip('\n').split('\t') for l in open(os.path.join(vec, 'MANIFEST.tsv'), encoding='utf-8')
            if l.strip() and not l.startswith('#')]
    files = {}
    for row in rows:
        if not pick(row):
            continue
        path, verdict, cls, root, sha, _, content = row
        data = open(os.path.join(vec, path), 'rb').read()
        assert hashlib.sha256(data).hexdigest() == sha, path
        name = os.path.basename(path)
        shutil.copyfile(os.path.join(vec, path), os.path.join(out_dir, name))
        item = dict(path=path, verdict=verdict, cls=cls, root=root, sha256=sha, content=content, records=[])
        digest = ctypes.create_string_buffer(32)
        item['ref_check'] = ref.wex4_check(data, len(data), 3, digest)
        item['ref_content'] = digest.raw.hex() if item['ref_check'] == 0 else None
        try:
            f = oracle.Wex4File(data)
        except Exception:   # a refused file whose index cannot even be sliced
            f = None
        if f is not None and item['ref_check'] in (0, -14):
            for r, rec in enumerate(f.records):
                if not rec['flags'] & 2 or rec['count'] != 6:
                    continue
                out = ctypes.create_string_buffer(rec['decoded'])
                blob = f.blob(rec['blob'] - 1) if rec['blob'] else None
                st = ref.wex4_decode_record_buf(f.page, f.file_bytes, f.index, len(f.index), r, f.stored(r), blob, 1, out)
                item['records'].append(dict(r=r, codec=rec['codec'], owner=rec['owner'], flags=rec['flags'],
                                            blob=rec['blob'], entry=f.expert_entry(r).hex(), ref_status=st,
                                            ref_sha=hashlib.sha256(out.raw).hexdigest() if st == 0 else None))
        files[name] = item
    json.dump(files, open(os.path.join(HERE, 'vectors.json'), 'w'), indent=1, sort_keys=True)
    print(f'{len(files)} vectors, {sum(len(v["records"]) for v in files.values())} expert records')


if __name__ == '__main__':
    main()
