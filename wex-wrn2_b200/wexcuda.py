"""ctypes binding of libwexb200.so: the CUDA helper ABI (include/wex_cuda_helper.h), the engine API
(include/wex_decode.h), the WEX4 tools ABI (include/wex4_tools.h), the WNR4 ABI (include/wnr4_cuda.h)
and the B200 additions (include/wexb200.h: queued batches, resident records, file reads).

Device buffers are plain integers (device pointers: torch tensors' data_ptr() work, any runtime of
the process shares the device's primary context). Host buffers are numpy uint8 arrays or bytes.
The library must be present: this module never falls back to anything else.
"""
import ctypes
import os

import numpy as np

import build as _build

P, U32, U64, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int
_lib = None


def lib_path():
    return _build.CUDA_LIB


def lib():
    """The loaded library (built in-tree first if it is missing and nvcc is available)."""
    global _lib
    if _lib is None:
        path = lib_path()
        if not os.path.exists(path):
            _build.build_cuda()
        if not os.path.exists(path):
            raise RuntimeError(f'{path} is missing: run `python wex-wrn2_b200/build.py`')
        L = ctypes.CDLL(path)
        L.wex_cuda_helper_abi.restype = U32
        L.wex_cuda_helper_features.restype = U32
        L.wex_cuda_register_model.argtypes = [P, SZ]
        L.wex_cuda_decode_to_host.argtypes = [P, P, SZ]
        L.wex_cuda_decode_to_device.argtypes = [P, P, I, P, P]
        L.wex_cuda_decode_batch_to_device.argtypes = [I, P, P, I, P, P, P]
        L.wex_cuda_decode_batch_to_host.argtypes = [I, P, P, I, P, P]
        L.wex_cuda_host_register.argtypes = [P, SZ]
        L.wex_cuda_host_unregister.argtypes = [P]
        L.wexb_abi.restype = U32
        L.wexb_last_error_bits.restype = U32
        L.wexb_batch_submit.argtypes = [I, P, P, I, P, P]
        L.wexb_batch_wait.argtypes = [I, P]
        L.wexb_batch_submit_verified.argtypes = [I, P, P, P, I, P, P]
        L.wexb_resident_create.argtypes = [I, P, P, I, P, P]
        L.wexb_resident_bytes.argtypes = [P]; L.wexb_resident_bytes.restype = SZ
        L.wexb_resident_decode.argtypes = [P, I, P, P, P, P]
        L.wexb_resident_wait.argtypes = [P, P]
        L.wexb_resident_launches.argtypes = [P]
        L.wexb_resident_profile.argtypes = [P, I]
        L.wexb_resident_kernel_ms.argtypes = [P, P]
        L.wexb_resident_destroy.argtypes = [P]; L.wexb_resident_destroy.restype = None
        L.wexb_file_open.argtypes = [ctypes.c_char_p, ctypes.c_uint, I, P]
        L.wexb_file_info.argtypes = [P, P, P, P, P]
        L.wexb_file_evict.argtypes = [P]
        L.wexb_file_read.argtypes = [P, I, P, P, I, P, P]
        L.wexb_file_decode.argtypes = [P, I, I, P, P, P, P, P]
        L.wexb_file_close.argtypes = [P]; L.wexb_file_close.restype = None
        L.wexb_encode_batch.argtypes = [I, P, P, P, P, I, ctypes.c_uint, ctypes.c_uint, P, SZ, I, P, P, P, P, P]
        L.wexb_count_batch.argtypes = [I, P, P, I, I, P, P, P]
        L.wexb_selftest_bounded_wait.argtypes = [I, ctypes.c_uint, P]
        L.wexb_set_wait_limit.argtypes = [ctypes.c_double]
        L.wexb_wait_limit.restype = ctypes.c_double
        _lib = L
    return _lib


def _buf(x):
    """(address, keep-alive) of a host buffer: numpy array, bytearray or bytes."""
    if isinstance(x, np.ndarray):
        assert x.flags['C_CONTIGUOUS']
        return x.ctypes.data, x
    if isinstance(x, bytearray):
        a = (ctypes.c_char * len(x)).from_buffer(x)
        return ctypes.addressof(a), a
    if isinstance(x, (bytes, memoryview)):
        a = np.frombuffer(bytes(x), np.uint8)
        return a.ctypes.data, a
    raise TypeError(type(x))


def _ptrs(values):
    return (ctypes.c_void_p * len(values))(*[v or None for v in values])


def _entries(entries):
    """Array of WexEntry pointers from 72-byte entries (keeps the storage alive in the result)."""
    store = [np.frombuffer(bytes(e), np.uint8).copy() for e in entries]
    return _ptrs([a.ctypes.data for a in store]), store


def register_model(blob):
    return lib().wex_cuda_register_model(bytes(blob), len(blob))


def decode_to_host(entry, slab):
    """slab: bytearray / numpy array holding the record at its read offset; returns the status."""
    a, keep = _buf(slab)
    e = np.frombuffer(bytes(entry), np.uint8).copy()
    return lib().wex_cuda_decode_to_host(e.ctypes.data, a, len(slab))


def decode_to_device(entry, record, device, dst_scale, dst_weight):
    a, keep = _buf(record)
    e = np.frombuffer(bytes(entry), np.uint8).copy()
    return lib().wex_cuda_decode_to_device(e.ctypes.data, a, device, _ptrs(dst_scale), _ptrs(dst_weight))


def decode_batch_to_device(entries, records, device, dst_scale, dst_weight):
    """(failures, statuses). dst_scale / dst_weight: 3 * n device pointers."""
    n = len(entries)
    ep, keep_e = _entries(entries)
    bufs = [_buf(r) for r in records]
    status = (ctypes.c_int * max(n, 1))()
    bad = lib().wex_cuda_decode_batch_to_device(n, ep, _ptrs([b[0] for b in bufs]), device, _ptrs(dst_scale),
                                                _ptrs(dst_weight), status)
    return bad, list(status)[:n]


def decode_batch_to_host(entries, records, device, dsts):
    n = len(entries)
    ep, keep_e = _entries(entries)
    bufs = [_buf(r) for r in records]
    outs = [_buf(d) for d in dsts]
    status = (ctypes.c_int * max(n, 1))()
    bad = lib().wex_cuda_decode_batch_to_host(n, ep, _ptrs([b[0] for b in bufs]), device, _ptrs([o[0] for o in outs]),
                                              status)
    return bad, list(status)[:n]


class Ticket:
    """A queued device batch (wexb_batch_submit); keeps its arguments alive until wait()."""

    def __init__(self, entries, records, device, dst_scale, dst_weight, sha256=None):
        """sha256: the records' expected SHA-256 digests (32 bytes each) for a verified batch
        (wexb_batch_submit_verified), or None."""
        self.n = len(entries)
        ep, keep_e = _entries(entries)
        bufs = [_buf(r) for r in records]
        sp, wp = _ptrs(dst_scale), _ptrs(dst_weight)
        digests = None if sha256 is None else np.frombuffer(b''.join(bytes(d) for d in sha256), np.uint8).copy()
        self._keep = (ep, keep_e, bufs, sp, wp, digests)
        rp = _ptrs([b[0] for b in bufs])
        if digests is None:
            self.ticket = lib().wexb_batch_submit(self.n, ep, rp, device, sp, wp)
        else:
            assert len(digests) == 32 * self.n
            self.ticket = lib().wexb_batch_submit_verified(self.n, ep, rp, digests.ctypes.data, device, sp, wp)
        if self.ticket < 0:
            raise RuntimeError(f'wexb_batch_submit: {self.ticket}')

    def wait(self):
        """(failures, statuses)."""
        status = (ctypes.c_int * max(self.n, 1))()
        bad = lib().wexb_batch_wait(self.ticket, status)
        self._keep = None
        return bad, list(status)[:self.n]


def submit_batch_to_device(entries, records, device, dst_scale, dst_weight, sha256=None):
    return Ticket(entries, records, device, dst_scale, dst_weight, sha256)


def host_register(array):
    return lib().wex_cuda_host_register(array.ctypes.data, array.nbytes)


def host_unregister(array):
    return lib().wex_cuda_host_unregister(array.ctypes.data)


class Resident:
    """Records kept in device memory (wexb_resident_*): decode any subset into device buffers."""

    def __init__(self, entries, records, device=0):
        n = len(entries)
        ep, keep_e = _entries(entries)
        bufs = [_buf(r) for r in records]
        self.status = (ctypes.c_int * n)()
        h = ctypes.c_void_p()
        self.failures = lib().wexb_resident_create(n, ep, _ptrs([b[0] for b in bufs]), device, ctypes.byref(h),
                                                   self.status)
        self.handle = h.value
        self._k = 0

    @property
    def bytes(self):
        return lib().wexb_resident_bytes(self.handle)

    def decode(self, index, dst_scale, dst_weight, stream=None):
        """Queue the decode of resident records `index` (0 queued)."""
        self._k = len(index)
        idx = (ctypes.c_int * len(index))(*index)
        self._keep = (idx, _ptrs(dst_scale), _ptrs(dst_weight))
        return lib().wexb_resident_decode(self.handle, len(index), idx, self._keep[1], self._keep[2], stream)

    def wait(self):
        status = (ctypes.c_int * max(self._k, 1))()
        bad = lib().wexb_resident_wait(self.handle, status)
        return bad, list(status)[:self._k]

    def launches(self):
        return lib().wexb_resident_launches(self.handle)

    def profile(self, on=True):
        return lib().wexb_resident_profile(self.handle, 1 if on else 0)

    def kernel_ms(self):
        """(metadata upload, decode launch, status read-back) milliseconds of the last waited decode, or None."""
        ms = (ctypes.c_float * 3)()
        return tuple(ms) if lib().wexb_resident_kernel_ms(self.handle, ms) == 0 else None

    def close(self):
        if self.handle:
            lib().wexb_resident_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


FILE_DIRECT = 1


class ExpertFile:
    """A WEX4 container file opened for expert reads (wexb_file_*): records read by a pool of reader
    threads into page-locked buffers, then uploaded and decoded batch by batch."""

    def __init__(self, path, direct=False, readers=0):
        h = ctypes.c_void_p()
        rc = lib().wexb_file_open(os.fsencode(path), FILE_DIRECT if direct else 0, readers, ctypes.byref(h))
        if rc:
            raise OSError(rc, f'wexb_file_open: {rc}')
        self._h = h

    def info(self):
        """(layers, experts, expert records, largest stored record)."""
        v = [ctypes.c_uint(), ctypes.c_uint(), ctypes.c_uint(), ctypes.c_ulonglong()]
        lib().wexb_file_info(self._h, *[ctypes.byref(x) for x in v])
        return tuple(x.value for x in v)

    def evict(self):
        return lib().wexb_file_evict(self._h)

    @staticmethod
    def _keys(keys):
        n = len(keys)
        lay = (ctypes.c_uint * max(n, 1))(*[k[0] for k in keys])
        exp = (ctypes.c_uint * max(n, 1))(*[k[1] for k in keys])
        return n, lay, exp

    def read(self, keys, check=False):
        """Read stage only. keys: (layer, expert) pairs. (failures, statuses, stored bytes)."""
        n, lay, exp = self._keys(keys)
        status = (ctypes.c_int * max(n, 1))()
        got = ctypes.c_ulonglong()
        bad = lib().wexb_file_read(self._h, n, lay, exp, 1 if check else 0, status, ctypes.byref(got))
        return bad, list(status)[:n], got.value

    def decode(self, keys, device, dst_scale, dst_weight):
        """keys: (layer, expert) pairs; dst_scale / dst_weight: 3 * n device pointers. (failures, statuses)."""
        n, lay, exp = self._keys(keys)
        status = (ctypes.c_int * max(n, 1))()
        bad = lib().wexb_file_decode(self._h, device, n, lay, exp, _ptrs(dst_scale), _ptrs(dst_weight), status)
        return bad, list(status)[:n]

    def close(self):
        if self._h:
            lib().wexb_file_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def encode_batch(blob, entries, coded, flags, owners, nr3=True, wchunk=2048, schunk=512, device=0, caps=None,
                 outs=None):
    """Records encoded on the GPU (wexb_encode_batch): a list of (status, record, used, total); status 0
    encoded, 1 store RAW, -1 invalid, -2 CUDA unavailable. outs: writable host buffers (numpy uint8) to
    encode into, whose sizes are the caps; then record is None and the caller reads outs[i][:total]."""
    n = len(entries)
    ep, keep_e = _entries(entries)
    srcs = [_buf(c) for c in coded]
    given = outs is not None
    if not given:
        outs = [np.empty(c, np.uint8) for c in (caps or [4 * len(c) + 65536 for c in coded])]
    dsts = [_buf(o) for o in outs]
    U = ctypes.c_uint * max(n, 1)
    used, total = (SZ * max(n, 1))(), (SZ * max(n, 1))()
    status = (ctypes.c_int * max(n, 1))()
    b = bytes(blob)
    lib().wexb_encode_batch(n, ep, _ptrs([x[0] for x in srcs]), U(*flags), U(*owners), 1 if nr3 else 0, wchunk, schunk,
                            b, len(b), device, _ptrs([d[0] for d in dsts]), (SZ * max(n, 1))(*[len(o) for o in outs]),
                            used, total, status)
    return [(status[i], None if given or status[i] else outs[i][:total[i]].tobytes(), used[i], total[i])
            for i in range(n)]


def count_batch(entries, coded, nr3=True, device=0):
    """(statuses, wc, sc): training counts on the GPU (wexb_count_batch), numpy uint64 [3*567*16], [3*256]."""
    n = len(entries)
    ep, keep_e = _entries(entries)
    srcs = [_buf(c) for c in coded]
    wc, sc = np.zeros(3 * 567 * 16, np.uint64), np.zeros(3 * 256, np.uint64)
    status = (ctypes.c_int * max(n, 1))()
    lib().wexb_count_batch(n, ep, _ptrs([x[0] for x in srcs]), 1 if nr3 else 0, device, wc.ctypes.data, sc.ctypes.data,
                           status)
    return list(status)[:n], wc, sc


def set_wait_limit(seconds):
    """Host wait limit of every entry point (wexb_set_wait_limit): 0, or -1 for a value out of range."""
    return lib().wexb_set_wait_limit(float(seconds))


def wait_limit():
    return lib().wexb_wait_limit()


def selftest_bounded_wait(device=0, polls=1000):
    """(status, error bits of the wait that nothing completes): wexb_selftest_bounded_wait."""
    bits = ctypes.c_uint()
    st = lib().wexb_selftest_bounded_wait(device, polls, ctypes.byref(bits))
    return st, bits.value
