"""A WEX4 container writer (canonical layout: header page, index, blobs, records) for the synthetic
workloads, following the container format of the reference (docs/WEX4-SPEC.md sections 3-5: header
page, blob / record / tensor tables, name order, name pool, metadata; the index and header SHA-256).

Expert records hold the six MXFP4 tensors of a routed expert (scales of w1, w2, w3 as F8_E8M0
[rows, cols], then packed weights as I8 [rows, 16 * cols]) and carry the EXPERT flag and owner
layer << 16 | expert (c/wex4.h:264-290 rebuilds the 72-byte WexEntry from them). A WNR4 (codec 8)
expert slab is written as a non-EXPERT record owning itself, with the same six tensors, since the
container's 4.0 rules allow EXPERT only with codecs 0 and 5."""
import hashlib
import struct

PAGE = 4096
MAGIC = 0x57455834
DT_I8, DT_F8_E8M0 = 3, 6
CODEC_RAW, CODEC_WNR3, CODEC_WNR4 = 0, 5, 8
FLAG_VALUE_EXACT, FLAG_EXPERT = 1, 2
BLOB_WNM2, BLOB_WNM4 = 1, 3


def align(n):
    return (n + PAGE - 1) & ~(PAGE - 1)


def expert_tensors(prefix, hidden, ffn):
    """The six tensors of an expert slab: (name, dtype, shape, nbytes) in slab order."""
    shapes = [(ffn, hidden // 32), (hidden, ffn // 32), (ffn, hidden // 32)]
    out = [(f'{prefix}.w{m + 1}.scales', DT_F8_E8M0, (r, c), r * c) for m, (r, c) in enumerate(shapes)]
    out += [(f'{prefix}.w{m + 1}.weight', DT_I8, (r, 16 * c), r * 16 * c) for m, (r, c) in enumerate(shapes)]
    return out


class Record:
    """One record: stored bytes (padded to the page here), decoded size, codec, flags, blob (0 or 1 +
    blob index), owner (layer << 16 | expert for EXPERT records; the writer sets it to the record index
    otherwise) and its tensors."""

    def __init__(self, stored, decoded_bytes, codec, tensors, flags=0, blob=0, owner=None):
        self.stored = bytes(stored) + bytes(align(len(stored)) - len(stored))
        self.decoded_bytes, self.codec, self.tensors = decoded_bytes, codec, tensors
        self.flags, self.blob, self.owner = flags, blob, owner


def expert_record(expert, blob_index=0, value_exact=False, codec=None, stored=None):
    """Record of a synth.Expert (its WNR3 or RAW record, or a WNR4 record given as `stored`)."""
    codec = expert.codec if codec is None else codec
    stored = expert.record if stored is None else stored
    tensors = expert_tensors(f'layers.{expert.layer}.experts.{expert.index}', expert.hidden, expert.ffn)
    decoded = sum(t[3] for t in tensors)
    if codec == CODEC_WNR4:
        return Record(stored, decoded, codec, tensors, 0, 1 + blob_index)
    flags = FLAG_EXPERT | (FLAG_VALUE_EXACT if value_exact and codec == CODEC_WNR3 else 0)
    return Record(stored, decoded, codec, tensors, flags, 1 + blob_index if codec == CODEC_WNR3 else 0,
                  expert.layer << 16 | expert.index)


def write(records, blobs=(), grid=(0, 0), value_exact=False, meta=b''):
    """The container bytes. blobs: (kind, id, bytes). grid: (num_layers, num_experts)."""
    records = list(records)
    tensors, names = [], []
    for r, rec in enumerate(records):
        rec.first = len(tensors)
        at = 0
        for name, dtype, shape, nbytes in rec.tensors:
            tensors.append((name.encode(), dtype, shape, r, at, nbytes))
            at += nbytes
        assert at == rec.decoded_bytes, 'tensors must tile the record'
    names = b''.join(t[0] for t in tensors)
    index_bytes = 64 * len(blobs) + 72 * len(records) + 100 * len(tensors) + len(names) + len(meta)
    at = PAGE + align(index_bytes)
    blob_rows = []
    for kind, bid, data in blobs:
        blob_rows.append(struct.pack('<IIQQ32sQ', kind, bid, at, len(data), hashlib.sha256(data).digest(), 0))
        at += align(len(data))
    rec_rows = []
    for r, rec in enumerate(records):
        owner = rec.owner if rec.flags & FLAG_EXPERT else r
        rec_rows.append(struct.pack('<QIIHHIIII32sI', at, len(rec.stored), rec.decoded_bytes, rec.codec, rec.flags,
                                    rec.blob, owner, rec.first, len(rec.tensors), hashlib.sha256(rec.stored).digest(), 0))
        at += len(rec.stored)
    file_bytes = at
    ten_rows, off = [], 0
    for name, dtype, shape, r, offset, nbytes in tensors:
        dims = list(shape) + [0] * (8 - len(shape))
        ten_rows.append(struct.pack('<IHBB8QIIQQ', off, len(name), dtype, len(shape), *dims, r, 1, offset, nbytes))
        off += len(name)
    order = sorted(range(len(tensors)), key=lambda i: tensors[i][0])
    index = b''.join(blob_rows) + b''.join(rec_rows) + b''.join(ten_rows) + struct.pack(f'<{len(order)}I', *order) + \
        names + meta
    assert len(index) == index_bytes
    max_dec = max((rec.decoded_bytes for rec in records), default=0)
    total_dec = sum(rec.decoded_bytes for rec in records)
    head = struct.pack('<IHHQQQQQIIIIIIQQQ32s', MAGIC, 4, 0, 1 if value_exact else 0, 0, file_bytes, PAGE, index_bytes,
                       len(blobs), len(records), len(tensors), grid[0], grid[1], max_dec, len(names), len(meta),
                       total_dec, hashlib.sha256(index).digest())
    head += bytes(4064 - len(head))
    head += hashlib.sha256(head).digest()
    parts = [head, index + bytes(align(index_bytes) - index_bytes)]
    for kind, bid, data in blobs:
        parts.append(data + bytes(align(len(data)) - len(data)))
    parts += [rec.stored for rec in records]
    out = b''.join(parts)
    assert len(out) == file_bytes
    return out


def content_digest(records, decoded):
    """The content digest (SHA-256 over name length, name, dtype, rank, shape, size and bytes of every
    tensor in table order) from each record's decoded bytes."""
    h = hashlib.sha256()
    for rec, data in zip(records, decoded):
        at = 0
        for name, dtype, shape, nbytes in rec.tensors:
            dims = list(shape) + [0] * (8 - len(shape))
            h.update(struct.pack('<H', len(name)) + name.encode() + struct.pack('<BB8QQ', dtype, len(shape), *dims, nbytes))
            h.update(data[at:at + nbytes])
            at += nbytes
    return h.digest()
