"""WBP1 (codec 6, byte-plane rANS for non-expert tensors): the canonical encoder of libwexb200.so is byte
for byte the reference's (oracle/_ref/wex4_tools_ref.so, wex4_bp_encode_record) over element sizes 1, 2,
4, 8, chunk sizes 2^10 .. 2^15, both transforms and data from incompressible to constant; the GPU decoder
(wex4_bp_decode_record) returns what the reference decoder returns, refuses what it refuses, and
recovers the input bytes."""
import ctypes

import numpy as np
import pytest

import oracle
import wexcuda

P, U32, SZ = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t


def ref():
    L = oracle.ref_lib('wex4_tools_ref')
    if L is None:
        pytest.skip('reference tools not built (make -C oracle ref)')
    for lib in (L, ours()):
        lib.wex4_bp_encode_record.argtypes = [P, U32, U32, U32, U32, U32, P, SZ, ctypes.POINTER(SZ)]
        lib.wex4_bp_decode_record.argtypes = [P, SZ, U32, U32, P]
    return L


def ours():
    return wexcuda.lib()


def sample(kind, n, seed):
    rng = np.random.default_rng(seed)
    if kind == 'random':
        return rng.integers(0, 256, n, dtype=np.uint8).tobytes()
    if kind == 'zeros':
        return bytes(n)
    if kind == 'bf16':   # N(0, 0.02) in bfloat16: a compressible exponent byte, noisy mantissa
        f = (rng.standard_normal((n + 1) // 2) * 0.02).astype(np.float32)
        return (f.view(np.uint32) >> 16).astype(np.uint16).tobytes()[:n]
    if kind == 'f32':
        return (rng.standard_normal((n + 3) // 4) * 3).astype(np.float32).tobytes()[:n]
    return bytes((i * 7 // 3) & 255 for i in range(n))   # a ramp


CASES = [(kind, n, planes, clog, tr) for kind, n, planes, clog, tr in [
    ('random', 1, 1, 10, 0), ('random', 5000, 1, 10, 0), ('zeros', 70000, 2, 12, 0), ('bf16', 200000, 2, 12, 1),
    ('bf16', 200001, 2, 12, 0), ('f32', 400000, 4, 15, 1), ('f32', 400000, 4, 13, 0), ('ramp', 123457, 8, 11, 0),
    ('f32', 262144, 8, 10, 1), ('bf16', 1 << 20, 2, 12, 1), ('random', 65536, 4, 14, 0), ('ramp', 3, 8, 10, 0)]]


def encode(L, data, planes, clog, tr, owner):
    cap = 2 * len(data) + (1 << 16)
    out = ctypes.create_string_buffer(cap)
    written = SZ()
    st = L.wex4_bp_encode_record(data, len(data), planes, clog, tr, owner, out, cap, ctypes.byref(written))
    return st, out.raw[:written.value]


@pytest.mark.parametrize('kind,n,planes,clog,tr', CASES)
def test_encoder_matches_reference(kind, n, planes, clog, tr):
    R = ref()
    data = sample(kind, n, n + planes)
    st1, a = encode(R, data, planes, clog, tr, 17)
    st2, b = encode(ours(), data, planes, clog, tr, 17)
    assert st1 == st2 == 0 and a == b


def test_encoder_refuses_like_reference():
    R = ref()
    data = sample('bf16', 1001, 3)
    for planes, clog, tr in [(3, 12, 0), (2, 9, 0), (2, 16, 0), (1, 12, 1), (2, 12, 1), (4, 12, 2)]:
        assert encode(R, data, planes, clog, tr, 0)[0] == encode(ours(), data, planes, clog, tr, 0)[0] == -1


@pytest.mark.gpu
@pytest.mark.parametrize('kind,n,planes,clog,tr', CASES)
def test_gpu_decode_matches_reference(kind, n, planes, clog, tr):
    R = ref()
    L = ours()
    data = sample(kind, n, 7 * n + planes)
    st, rec = encode(R, data, planes, clog, tr, 5)
    assert st == 0
    out = ctypes.create_string_buffer(n)
    assert L.wex4_bp_decode_record(rec, len(rec), n, 5, out) == 0 and out.raw == data
    assert L.wex4_bp_decode_record(rec, len(rec), n, 6, out) == R.wex4_bp_decode_record(rec, len(rec), n, 6, out) == -1
    rng = np.random.default_rng(n)
    for trial in range(6):   # damaged bytes: the GPU refuses exactly what the reference refuses
        bad = bytearray(rec)
        used = len(bad) - 1
        while used > 16 and bad[used] == 0:
            used -= 1
        bad[int(rng.integers(0, used + 1))] ^= 1 << int(rng.integers(0, 8))
        want = R.wex4_bp_decode_record(bytes(bad), len(bad), n, 5, out)
        assert L.wex4_bp_decode_record(bytes(bad), len(bad), n, 5, out) == want, (trial, want)
