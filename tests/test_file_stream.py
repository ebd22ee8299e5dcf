"""Expert records read from a WEX4 container file (wexb_file_*: reader threads, a ring of page-locked
buffers, uploads and decodes batch by batch), on the tiny written container (8 WNR3 experts and one RAW
expert, hidden 1024 / FFN 512). CPU: open-time validation (header, index, model blobs), the read stage
with SHA-256 checks against the index, ring reuse over more records than the ring holds. GPU: every
decoded slab equals the oracle's expected bytes, in both canonical-zero modes, for repeated and missing
keys, through O_DIRECT where the filesystem allows it; a damaged record fails alone and its
destination stays untouched."""
import hashlib
import os
import random
import struct

import pytest

import wex4file
import wexcuda
from test_wex4_written import _damaged, tiny_file


def _write(tmp_path, data, name='experts.wex4'):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def test_open_reports_the_grid_and_reads_every_record(tmp_path):
    data, ex, recs = tiny_file(False)
    f = wexcuda.ExpertFile(_write(tmp_path, data))
    layers, experts, records, largest = f.info()
    assert (layers, experts, records) == (1, 9, 9)
    assert largest == max(len(r.stored) for r in recs)
    keys = [(0, i) for i in range(9)]
    bad, status, got = f.read(keys, check=True)
    assert bad == 0 and status == [0] * 9 and got == sum(len(r.stored) for r in recs)
    # missing experts: -1, the others still read
    bad, status, got = f.read([(0, 9), (1, 0), (0, 4), (70000, 1)], check=True)
    assert status == [-1, -1, 0, -1] and bad == 3 and got == len(recs[4].stored)
    assert f.read([], check=True) == (0, [], 0)
    f.close()


def test_ring_is_reused_over_many_records(tmp_path):
    """60 keys (with repeats) are 8 ring batches, more than the ring's 3 slots hold at once."""
    data, ex, recs = tiny_file(True)
    f = wexcuda.ExpertFile(_write(tmp_path, data), readers=3)
    rng = random.Random(5)
    keys = [(0, rng.randrange(9)) for _ in range(60)]
    bad, status, got = f.read(keys, check=True)
    assert bad == 0 and got == sum(len(recs[e].stored) for _, e in keys)
    assert f.evict() in (0, 1)
    assert f.read(keys, check=True)[0] == 0
    f.close()


def test_read_check_names_the_damaged_record(tmp_path):
    """A flipped payload byte (the index still holds the old hash): only that record fails its check."""
    data, ex, recs = tiny_file(False)
    f = wexcuda.ExpertFile(_write(tmp_path, _damaged(data, 3, False)))
    bad, status, got = f.read([(0, i) for i in range(9)], check=True)
    assert bad == 1 and status == [0, 0, 0, -1, 0, 0, 0, 0, 0]
    assert f.read([(0, 3)], check=False)[1] == [0]   # without the check the bytes are only read
    f.close()


def test_open_refuses_bad_files(tmp_path):
    data, ex, recs = tiny_file(False)
    with pytest.raises(OSError) as e:
        wexcuda.ExpertFile(str(tmp_path / 'missing.wex4'))
    assert e.value.errno == 1
    for at in (8, 4096 + 10):   # header field (header hash), index byte (index hash)
        b = bytearray(data)
        b[at] ^= 1
        with pytest.raises(OSError) as e:
            wexcuda.ExpertFile(_write(tmp_path, bytes(b), f'bad{at}.wex4'))
        assert e.value.errno == -1
    # a model blob byte: its SHA-256 no longer matches the index
    blob_at = struct.unpack_from('<Q', data, 32)[0] + ((struct.unpack_from('<Q', data, 40)[0] + 4095) & ~4095)
    b = bytearray(data)
    b[blob_at + 100] ^= 1
    with pytest.raises(OSError) as e:
        wexcuda.ExpertFile(_write(tmp_path, bytes(b), 'badblob.wex4'))
    assert e.value.errno == -1
    with pytest.raises(OSError):
        wexcuda.ExpertFile(_write(tmp_path, data[:8192], 'short.wex4'))


def test_direct_reads_where_the_filesystem_allows_them(tmp_path):
    data, ex, recs = tiny_file(False)
    path = _write(tmp_path, data)
    try:
        f = wexcuda.ExpertFile(path, direct=True)
    except OSError as e:   # 1: this filesystem refuses O_DIRECT
        assert e.errno == 1
        return
    bad, status, got = f.read([(0, i) for i in range(9)], check=True)
    assert bad == 0 and got == sum(len(r.stored) for r in recs)
    f.close()


# ---- GPU ----------------------------------------------------------------------------------------

def _offsets(entry):
    v = struct.unpack('<QIII6H6H3I3II', bytes(entry))
    return v[16:19], v[19:22]   # scale offsets, weight offsets


def _decode(f, keys, ex, fill=0xAB):
    """Decode keys into one device slab each (at the entry's offsets); (statuses, host slabs)."""
    import torch
    slabs, ds, dw = [], [], []
    for layer, e in keys:
        x = ex[e] if layer == 0 and e < len(ex) else ex[0]
        slab = torch.full((len(x.expected),), fill, dtype=torch.uint8, device='cuda')
        so, wo = _offsets(x.entry)
        ds += [slab.data_ptr() + o for o in so]
        dw += [slab.data_ptr() + o for o in wo]
        slabs.append(slab)
    bad, status = f.decode(keys, 0, ds, dw)
    torch.cuda.synchronize()
    return bad, status, [s.cpu().numpy().tobytes() for s in slabs]


@pytest.mark.gpu
@pytest.mark.parametrize('cz', [False, True])
def test_gpu_file_decode_matches_the_expected_slabs(tmp_path, cz):
    data, ex, recs = tiny_file(cz)
    path = _write(tmp_path, data)
    rng = random.Random(11 + cz)
    keys = [(0, i) for i in range(9)] + [(0, rng.randrange(9)) for _ in range(40)] + [(0, 9), (2, 1)]
    for direct in (False, True):
        try:
            f = wexcuda.ExpertFile(path, direct=direct, readers=4)
        except OSError as e:
            assert direct and e.errno == 1   # the filesystem refuses O_DIRECT
            continue
        f.evict()
        bad, status, out = _decode(f, keys, ex)
        assert bad == 2 and status == [0] * 49 + [-1, -1]
        for (layer, e), got in zip(keys[:49], out):
            assert hashlib.sha256(got).digest() == hashlib.sha256(ex[e].expected).digest(), (direct, e)
        assert out[49] == bytes([0xAB]) * len(ex[0].expected)   # untouched
        f.close()


@pytest.mark.gpu
def test_gpu_file_decode_refuses_a_damaged_record_alone(tmp_path):
    """A flipped payload byte with the index hash fixed: the decode's own checks refuse record 2 (-1),
    its destination is untouched, and the other records decode."""
    data, ex, recs = tiny_file(True)
    f = wexcuda.ExpertFile(_write(tmp_path, _damaged(data, 2, True)))
    keys = [(0, i) for i in range(9)]
    bad, status, out = _decode(f, keys, ex)
    assert bad == 1 and status == [0, 0, -1, 0, 0, 0, 0, 0, 0]
    assert out[2] == bytes([0xAB]) * len(ex[2].expected)
    for i in (0, 1, 3, 4, 5, 6, 7, 8):
        assert out[i] == ex[i].expected
    f.close()
