"""Seeded synthetic MXFP4 experts and their WNR3 records (the inputs of tests and of bench.py).

An expert of hidden size H and expert FFN size F has three MXFP4 matrices in FP4 elements:
w1 gate [F x H], w2 down [H x F], w3 up [F x H]; each stores E2M1 nibbles packed two per byte
[rows, cols / 2] and one E8M0 scale per 32 elements [rows, cols / 32]. The decoded slab is the
scales of w1, w2, w3 then the packed weights of w1, w2, w3 (the legacy 72-byte entry layout).
"""
import ctypes
import os
import struct
from concurrent.futures import ThreadPoolExecutor

import numpy as np

import build as _build

P, U32, U64, SZ, I, D = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int, ctypes.c_double
MODEL_BYTES = 59408
CODEC_RAW, CODEC_WNR2, CODEC_WNR3 = 0, 4, 5
_tools = None


def tools():
    global _tools
    if _tools is None:
        L = ctypes.CDLL(_build.build_tools())
        L.wexb_tools_abi.restype = U32
        L.wexb_synth_matrix.argtypes = [U64, U32, U32, D, I, D, P, P]
        L.wexb_nr3_prepare.argtypes = [P, P, I, P]
        L.wexb_count_expert.argtypes = [P, P, I, P, P]
        L.wexb_build_model.argtypes = [P, P, P]; L.wexb_build_model.restype = U32
        L.wexb_encode_record.argtypes = [P, P, P, I, U32, U32, U32, U32, P, SZ, P, P]
        L.wexb_w4_model_bytes.argtypes = [U32]; L.wexb_w4_model_bytes.restype = SZ
        L.wexb_w4_counts_words.argtypes = [U32]; L.wexb_w4_counts_words.restype = SZ
        L.wexb_w4_count.argtypes = [P, P, U32, P]
        L.wexb_w4_build.argtypes = [U32, P, P]; L.wexb_w4_build.restype = U32
        L.wexb_w4_encode.argtypes = [P, SZ, P, P, U32, U32, U32, P, SZ]; L.wexb_w4_encode.restype = ctypes.c_longlong
        assert L.wexb_tools_abi() == 1
        _tools = L
    return _tools


def matrices(hidden, ffn):
    """(rows, cols) in FP4 elements of w1 gate, w2 down, w3 up."""
    return [(ffn, hidden), (hidden, ffn), (ffn, hidden)]


def expert_entry(hidden, ffn, codec=CODEC_WNR3, total=0, offset=0):
    """The 72-byte legacy entry (c/wex_format.h:57-67) of an expert of this shape."""
    mats = matrices(hidden, ffn)
    e = bytearray(72)
    soff, s = [], 0
    for r, c in mats:
        soff.append(s); s += r * c // 32
    woff, w = [], s
    for r, c in mats:
        woff.append(w); w += r * c // 2
    struct.pack_into('<QIII', e, 0, offset, total, s, w - s)
    for m, (r, c) in enumerate(mats):
        struct.pack_into('<HH', e, 20 + 4 * m, r, c // 32)
        struct.pack_into('<HH', e, 32 + 4 * m, r, c // 2)
        struct.pack_into('<I', e, 44 + 4 * m, soff[m])
        struct.pack_into('<I', e, 56 + 4 * m, woff[m])
    struct.pack_into('<I', e, 68, codec)
    return bytes(e)


def entry_with(entry, total=None, codec=None, offset=None):
    e = bytearray(entry)
    if offset is not None:
        struct.pack_into('<Q', e, 0, offset)
    if total is not None:
        struct.pack_into('<I', e, 8, total)
    if codec is not None:
        struct.pack_into('<I', e, 68, codec)
    return bytes(e)


def raw_bytes(hidden, ffn):
    return sum(r * c // 32 + r * c // 2 for r, c in matrices(hidden, ffn))


def synth_expert(hidden, ffn, seed, sigma=0.02, mode=0, neg_zero=0.0):
    """Decoded slab of one expert: seeded N(0, sigma) quantized to MXFP4 (mode 0), uniform random
    nibbles (mode 1, incompressible), Gaussian with every WNR3 block case mixed in (mode 2), or mode 2
    with a block of maximum 5 in w2 that keeps the ceil form off there (mode 3); neg_zero = fraction
    of zero nibbles written as -0."""
    mats = matrices(hidden, ffn)
    out = np.zeros(raw_bytes(hidden, ffn), np.uint8)
    scale_at = 0
    weight_at = sum(r * c // 32 for r, c in mats)
    for m, (r, c) in enumerate(mats):
        ns, nw = r * c // 32, r * c // 2
        sc = out[scale_at:scale_at + ns]
        wt = out[weight_at:weight_at + nw]
        md = 2 if (mode == 3 and m != 1) else mode   # mode 3: the maximum-5 block in w2 only
        assert tools().wexb_synth_matrix(seed * 3 + m, r, c, sigma, md, neg_zero,
                                         wt.ctypes.data, sc.ctypes.data) == 0
        scale_at += ns
        weight_at += nw
    return out.tobytes()


def canonical_zero(entry, slab):
    """Z(slab): every -0 nibble (8) of the weights becomes +0."""
    s = struct.unpack_from('<I', entry, 12)[0]
    a = np.frombuffer(slab, np.uint8).copy()
    w = a[s:]
    lo, hi = w & 15, w >> 4
    w[:] = np.where(lo == 8, 0, lo) | (np.where(hi == 8, 0, hi) << 4)
    return a.tobytes()


def prepare(entry, source, cz):
    """(flags, coded slab): canonical zero (cz) then the ceil form."""
    coded = ctypes.create_string_buffer(len(source))
    flags = tools().wexb_nr3_prepare(entry, source, 1 if cz else 0, coded)
    assert flags >= 0
    return flags, coded.raw


def train_model(pairs, nr3=True):
    """WNM2 blob trained on (entry, coded slab) pairs."""
    wc = np.zeros(3 * 567 * 16, np.uint64)
    sc = np.zeros(3 * 256, np.uint64)
    for entry, coded in pairs:
        assert tools().wexb_count_expert(entry, coded, 1 if nr3 else 0, wc.ctypes.data, sc.ctypes.data) == 0
    blob = ctypes.create_string_buffer(MODEL_BYTES)
    assert tools().wexb_build_model(wc.ctypes.data, sc.ctypes.data, blob) != 0
    return blob.raw


def encode(blob, entry, coded, flags=0, owner=0, wchunk=2048, schunk=512, nr3=True):
    """(status, record): status 0 encoded (record zero-padded to 4096), 1 not smaller than raw."""
    cap = 4 * len(coded) + 65536
    out = ctypes.create_string_buffer(cap)
    used, total = SZ(), SZ()
    st = tools().wexb_encode_record(blob, entry, coded, 1 if nr3 else 0, flags, owner, wchunk, schunk, out, cap,
                                    ctypes.byref(used), ctypes.byref(total))
    if st < 0:
        raise ValueError('encode failed')
    return st, out.raw[:total.value]


class Expert:
    """One synthetic expert: its source slab, coded slab, record and entry."""

    def __init__(self, hidden, ffn, layer, index, seed, sigma, cz=False, mode=0, neg_zero=0.0, nr3=True):
        self.hidden, self.ffn, self.layer, self.index = hidden, ffn, layer, index
        self.owner = layer << 16 | index
        self.source = synth_expert(hidden, ffn, seed, sigma, mode, neg_zero)
        self.cz = cz and nr3
        self.entry = expert_entry(hidden, ffn)
        if nr3:   # WNR3 codes the canonical-zero and ceil-form domain; WNR2 the source itself
            self.flags, self.coded = prepare(self.entry, self.source, self.cz)
        else:
            self.flags, self.coded = 0, self.source
        self.expected = canonical_zero(self.entry, self.source) if self.cz else self.source
        self.record = None
        self.codec = None

    def encode(self, blob, wchunk=2048, schunk=512, nr3=True):
        st, rec = encode(blob, self.entry, self.coded, self.flags if nr3 else 0, self.owner if nr3 else 0,
                         wchunk, schunk, nr3)
        if st == 0:
            self.record, self.codec = rec, (CODEC_WNR3 if nr3 else CODEC_WNR2)
        else:   # not smaller than raw: stored RAW with the source bytes (c/tools/wex_nr3_tools.c:85-103)
            raw = len(self.source)
            self.record = self.source + bytes(((raw + 4095) & ~4095) - raw)
            self.codec = CODEC_RAW
            self.expected = self.source
        self.entry = entry_with(self.entry, total=len(self.record), codec=self.codec)
        return self


def make_experts(hidden, ffn, owners, seed=1, sigma=0.02, cz=False, mode=0, neg_zero=0.0, train_every=8,
                 wchunk=2048, schunk=512, nr3=True, threads=None, blob=None, lean=False):
    """Experts for (layer, index) owners, a WNM2 model trained on every train_every-th of them (or the
    given blob), and their records. Generation and encoding run on host threads. lean (with a given
    blob): each expert keeps only its entry, record, decoded size (.raw) and the SHA-256 of its
    expected slab (.expected_sha), so that large pools fit in host memory."""
    import hashlib
    sig = sigma if callable(sigma) else (lambda layer: sigma)
    threads = threads or min(32, os.cpu_count() or 4)

    def make(i_owner):
        i, (layer, idx) = i_owner
        md = mode(i) if callable(mode) else mode
        return Expert(hidden, ffn, layer, idx, seed * 1000003 + layer * 4099 + idx, sig(layer), cz, md, neg_zero, nr3)

    def make_encoded(i_owner):
        e = make(i_owner).encode(blob, wchunk, schunk, nr3)
        e.raw = len(e.source)
        e.expected_sha = hashlib.sha256(e.expected).digest()
        if lean:
            e.source = e.coded = e.expected = None
        return e
    with ThreadPoolExecutor(threads) as pool:
        if blob is not None:
            return blob, list(pool.map(make_encoded, enumerate(owners)))
        experts = list(pool.map(make, enumerate(owners)))
        blob = train_model([(e.entry, e.coded) for e in experts[::train_every]], nr3)
        list(pool.map(lambda e: e.encode(blob, wchunk, schunk, nr3), experts))
    for e in experts:
        e.raw = len(e.source)
        e.expected_sha = hashlib.sha256(e.expected).digest()
    return blob, experts


# ---- WNR4 kind MX (draft codec 8) ------------------------------------------------------------------
def train_model4(pairs, pb=1):
    """WNM4 kind-MX blob trained on (entry, coded slab) pairs."""
    L = tools()
    counts = np.zeros(L.wexb_w4_counts_words(pb), np.uint64)
    for entry, coded in pairs:
        assert L.wexb_w4_count(entry, coded, pb, counts.ctypes.data) == 0
    blob = ctypes.create_string_buffer(L.wexb_w4_model_bytes(pb))
    assert L.wexb_w4_build(pb, counts.ctypes.data, blob) != 0
    return blob.raw


def encode4(blob4, entry, coded, flags, owner, G=32):
    """WNR4 record of a coded expert (zero-padded to 4096), or None when not smaller than raw."""
    cap = 2 * len(coded) + (1 << 20)
    out = ctypes.create_string_buffer(cap)
    n = tools().wexb_w4_encode(blob4, len(blob4), entry, coded, flags, owner, G, out, cap)
    if n < 0:
        raise ValueError('WNR4 encode failed')
    return out.raw[:n] if n else None


def geo4(entry):
    """The 13 geometry words of an expert slab for the WNR4 ABI: kind 0, cells, cols, offsets."""
    g = [0] * 13
    for m in range(3):
        r, c = struct.unpack_from('<HH', entry, 20 + 4 * m)
        g[1 + m], g[4 + m] = r * c, c
        g[7 + m] = struct.unpack_from('<I', entry, 44 + 4 * m)[0]
        g[10 + m] = struct.unpack_from('<I', entry, 56 + 4 * m)[0]
    return g

