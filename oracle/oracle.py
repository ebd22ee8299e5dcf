"""ORACLE — test infrastructure only. ctypes access to the C restatement (liboracle.so) and, when
built, to the reference's own CPU tools compiled from its sources (oracle/_ref/*.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module; the
product never does.
"""
import ctypes
import os
import struct
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, '_ref')
# Where the reference tree is read from when it is present (this recipe's build of oracle/_ref and the
# tests that read its vectors); WEXB_REFERENCE overrides it. Absent on hosts that only run the prebuilt
# checkers.
REFERENCE = os.environ.get('WEXB_REFERENCE', '/root/reference')
P, U32, U64, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int

_lib = None


def build():
    """Compile liboracle.so (and the reference tools when the reference sources are present)."""
    subprocess.run(['make', '-s', '-C', HERE], check=True)
    if os.path.isdir(REFERENCE):
        subprocess.run(['make', '-s', '-C', HERE, 'ref', f'REF={REFERENCE}'], check=True)
        if os.path.exists(os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')):
            subprocess.run(['make', '-s', '-C', HERE, 'gpuref', f'REF={REFERENCE}'], check=True)


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, 'liboracle.so')
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.oracle_murmur3.argtypes = [P, SZ, U32]; L.oracle_murmur3.restype = U32
        L.oracle_nr3_x0.argtypes = [P, P, U32]; L.oracle_nr3_x0.restype = U32
        L.oracle_fnv1a.argtypes = [P, SZ]; L.oracle_fnv1a.restype = U32
        L.oracle_anchor.argtypes = [P, U32]; L.oracle_anchor.restype = ctypes.c_uint8
        L.oracle_wnm2_open.argtypes = [P, SZ, P]; L.oracle_wnm2_open.restype = I
        L.oracle_nrx_decode.argtypes = [P, P, P, P, P]; L.oracle_nrx_decode.restype = I
        L.oracle_sha256.argtypes = [P, SZ, P]; L.oracle_sha256.restype = None
        L.oracle_wnr4_decode.argtypes = [P, SZ, P, P, SZ, U32, P]; L.oracle_wnr4_decode.restype = U32
        L.oracle_wnm4_id.argtypes = [P, SZ]; L.oracle_wnm4_id.restype = U32
        _lib = L
    return _lib


def murmur3(data, seed):
    return lib().oracle_murmur3(bytes(data), len(data), seed)


def nr3_x0(ident, data):
    arr = (U32 * 4)(*ident)
    return lib().oracle_nr3_x0(arr, bytes(data), len(data))


def sha256(data):
    out = ctypes.create_string_buffer(32)
    lib().oracle_sha256(bytes(data), len(data), out)
    return out.raw


def anchor(scales):
    return lib().oracle_anchor(bytes(scales), len(scales))


def wnm2_id(blob):
    out = U32()
    return out.value if lib().oracle_wnm2_open(bytes(blob), len(blob), ctypes.byref(out)) == 0 else None


def nrx_decode(blob, entry, record, raw_bytes):
    """(status, where, slab) of a codec-4/5 record; slab is None unless status == 0."""
    out = ctypes.create_string_buffer(max(raw_bytes, 1))
    where = I()
    st = lib().oracle_nrx_decode(bytes(blob), bytes(entry), bytes(record), out, ctypes.byref(where))
    return st, where.value, (out.raw[:raw_bytes] if st == 0 else None)


def wnr4_decode(model, geo, record, owner, raw_bytes):
    out = ctypes.create_string_buffer(max(raw_bytes, 1))
    g = (U32 * 13)(*geo)
    err = lib().oracle_wnr4_decode(bytes(model), len(model), g, bytes(record), len(record), owner, out)
    return err, (out.raw[:raw_bytes] if err == 0 else None)


# ---- the reference's own compiled CPU tools (present when `make -C oracle ref` ran) ----------
def ref_path(name):
    p = os.path.join(REF_DIR, name)
    return p if os.path.exists(p) else None


_ref = {}


def ref_lib(name):
    """ctypes handle of oracle/_ref/<name>.so with its argtypes, or None if it was not built."""
    if name in _ref:
        return _ref[name]
    p = ref_path(name + '.so')
    L = ctypes.CDLL(p) if p else None
    if L is not None and name.startswith('wex4_tools'):
        L.wex4_tools_abi.restype = U32
        L.wex4_check.argtypes = [P, U64, I, P]
        L.wex4_fuzz_check.argtypes = [P, U64, I, P]
        L.wex4_validate.argtypes = [P, U64, P, SZ]
        L.wex4_decode_record_buf.argtypes = [P, U64, P, SZ, U32, P, P, I, P]
        L.wex4_expert_table.argtypes = [P, U64, P, SZ, P]
        L.wex4_sha256_bytes.argtypes = [P, SZ, P]
    if L is not None and name == 'wex_nr3_tools':
        L.wex_nr3_prepare.argtypes = [P, P, I, P, P]
        L.wex_nr3_count_expert.argtypes = [P, P, P, P]
        L.wex_nr3_build_model.argtypes = [P, P, P, P]
        L.wex_nr3_encode_record.argtypes = [P, P, P, U32, U32, U32, U32, P, SZ, P, P]
        L.wex_nr3_decode.argtypes = [P, P, P, U32, U32, P]
        L.wex_nr3_decode.restype = I
    if L is not None and name == 'wnr4_tools':
        L.wnr4t_counts_words.argtypes = [U32, U32]; L.wnr4t_counts_words.restype = SZ
        L.wnr4t_model_bytes.argtypes = [U32, U32]; L.wnr4t_model_bytes.restype = SZ
        L.wnr4t_count.argtypes = [P, P, U32, P]
        L.wnr4t_build.argtypes = [U32, U32, P, P]; L.wnr4t_build.restype = U32
        L.wnr4t_model_open.argtypes = [P, SZ]; L.wnr4t_model_open.restype = P
        L.wnr4t_model_close.argtypes = [P]
        L.wnr4t_encode.argtypes = [P, P, P, U32, U32, U32, P, SZ]; L.wnr4t_encode.restype = SZ
        L.wnr4t_decode.argtypes = [P, P, P, SZ, U32, P, I]; L.wnr4t_decode.restype = U32
    _ref[name] = L
    return L


# ---- a minimal WEX4 index reader (c/wex4.h:185-236), enough to pull records out of a file ------
class Wex4File:
    """Header fields, blob / record / tensor rows of a WEX4 file held in memory (no validation
    beyond what slicing needs: the reference tools decide validity in the tests)."""

    def __init__(self, data):
        self.data = data = bytes(data)
        u = lambda fmt, at: struct.unpack_from(fmt, data, at)
        (self.file_bytes, self.index_offset, self.index_bytes) = u('<QQQ', 24)
        (self.nblobs, self.nrecords, self.ntensors, self.layers, self.experts, self.max_decoded) = u('<6I', 48)
        (self.names_bytes, self.meta_bytes, self.total_decoded) = u('<QQQ', 72)
        ix = self.index_offset
        self.index = data[ix:ix + ((self.index_bytes + 4095) & ~4095)]
        self.page = data[:4096]
        self.blobs, self.records, self.tensors = [], [], []
        at = ix
        for _ in range(self.nblobs):
            kind, bid, off, n = u('<IIQQ', at)
            self.blobs.append(dict(kind=kind, id=bid, offset=off, bytes=n, sha=data[at + 24:at + 56]))
            at += 64
        for _ in range(self.nrecords):
            off, stored, decoded, codec, flags, blob, owner, first, count = u('<QIIHHIIII', at)
            self.records.append(dict(offset=off, stored=stored, decoded=decoded, codec=codec, flags=flags,
                                     blob=blob, owner=owner, first=first, count=count, sha=data[at + 36:at + 68]))
            at += 72
        names_at = at + self.ntensors * 96 + self.ntensors * 4
        for _ in range(self.ntensors):
            name_at, name_len, dtype, rank = u('<IHBB', at)
            shape = u('<8Q', at + 8)
            rec, rcount, off, nbytes = u('<IIQQ', at + 72)
            name = data[names_at + name_at:names_at + name_at + name_len]
            self.tensors.append(dict(name=name, dtype=dtype, rank=rank, shape=shape, record=rec, record_count=rcount,
                                     offset=off, nbytes=nbytes))
            at += 96

    def stored(self, r):
        rec = self.records[r]
        return self.data[rec['offset']:rec['offset'] + rec['stored']]

    def blob(self, i):
        b = self.blobs[i]
        return self.data[b['offset']:b['offset'] + b['bytes']]

    def expert_entry(self, r):
        """The 72-byte legacy entry of EXPERT record r (c/wex4.h:264-290, layout c/wex_format.h:57-67)."""
        rec = self.records[r]
        ts = self.tensors[rec['first']:rec['first'] + 6]
        e = bytearray(72)
        struct.pack_into('<QI', e, 0, rec['offset'], rec['stored'])
        struct.pack_into('<I', e, 12, sum(t['nbytes'] for t in ts[:3]))
        struct.pack_into('<I', e, 16, sum(t['nbytes'] for t in ts[3:]))
        for m in range(3):
            struct.pack_into('<HH', e, 20 + 4 * m, ts[m]['shape'][0], ts[m]['shape'][1])
            struct.pack_into('<HH', e, 32 + 4 * m, ts[3 + m]['shape'][0], ts[3 + m]['shape'][1])
            struct.pack_into('<I', e, 44 + 4 * m, ts[m]['offset'])
            struct.pack_into('<I', e, 56 + 4 * m, ts[3 + m]['offset'])
        struct.pack_into('<I', e, 68, rec['codec'])
        return bytes(e)


def content_digest(f, decoded_records):
    """WEX4 content digest (wex4/wex4_tools.c:125-158) from a list of decoded record bytes."""
    import hashlib
    h = hashlib.sha256()

    def meta(t, nbytes):
        h.update(struct.pack('<H', len(t['name'])) + t['name'] +
                 struct.pack('<BB8QQ', t['dtype'], t['rank'], *t['shape'], nbytes))
    used = 0
    for r, rec in enumerate(f.records):
        data = decoded_records[r]
        if not rec['count']:
            h.update(data)
        for t in f.tensors[rec['first']:rec['first'] + rec['count']]:
            meta(t, t['nbytes'])
            h.update(data[t['offset']:t['offset'] + t['nbytes']] if t['record_count'] == 1 else data)
        used = max(used, rec['first'] + rec['count'])
    first_empty = len(f.tensors)
    while first_empty and not f.tensors[first_empty - 1]['nbytes']:
        first_empty -= 1
    for t in f.tensors[first_empty:]:
        meta(t, 0)
    return h.digest()
