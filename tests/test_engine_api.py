"""The engine-facing API (include/wex_decode.h, the reference's c/wex_decode.h) over the GPU helper."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import synth
import wexcuda

P, U32, U64, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def lib():
    L = wexcuda.lib()
    L.coli_wex_register_model.argtypes = [P, SZ, P]
    L.coli_wex_decode_record.argtypes = [P, P, SZ]
    L.coli_wex_container_refused.argtypes = [U32, ctypes.c_char_p]
    L.coli_wex_cuda_decode_count.restype = U64
    L.coli_wex_cuda_device_decode_count.restype = U64
    L.coli_wex_cuda_decode_batch_to_device.argtypes = [I, P, P, I, P, P, P]
    return L


def test_register_model_returns_its_id():
    blob, ex = synth.make_experts(256, 96, [(0, 0)], seed=3, train_every=1)
    mid = U32()
    assert lib().coli_wex_register_model(blob, len(blob), ctypes.byref(mid)) == 0
    assert mid.value == int.from_bytes(ex[0].record[4:8], 'little')
    assert lib().coli_wex_register_model(blob[:100], 100, ctypes.byref(mid)) == -1


def test_container_refusal_policy():
    """Canonical-zero containers are refused only when DSV4_CUDA_MOE_MASKED != 0 (c/wex_decode.c:309-321);
    run in child processes so the environment is read fresh."""
    code = ('import sys; sys.path.insert(0, %r); import wexcuda, ctypes; L = wexcuda.lib(); '
            'L.coli_wex_container_refused.argtypes = [ctypes.c_uint32, ctypes.c_char_p]; '
            'print(L.coli_wex_container_refused(64, b"t"), L.coli_wex_container_refused(0, b"t"))') % os.path.join(ROOT, 'wex-wrn2_b200')
    for env, want in (({'DSV4_CUDA_MOE_MASKED': '1'}, '1 0'), ({'DSV4_CUDA_MOE_MASKED': '0'}, '0 0'), ({}, '0 0')):
        e = {k: v for k, v in os.environ.items() if k != 'DSV4_CUDA_MOE_MASKED'}
        e.update(env)
        out = subprocess.run([sys.executable, '-c', code], env=e, capture_output=True, text=True, check=True)
        assert out.stdout.strip() == want, (env, out.stdout, out.stderr)


def test_raw_entry_is_already_a_slab():
    e = synth.entry_with(synth.expert_entry(256, 96), total=0, codec=0)
    raw = synth.raw_bytes(256, 96)
    aligned = (raw + 4095) & ~4095
    slab = bytearray(aligned)
    assert lib().coli_wex_decode_record(synth.entry_with(e, total=aligned), (ctypes.c_char * aligned).from_buffer(slab), aligned) == 0
    assert lib().coli_wex_decode_record(synth.entry_with(e, total=aligned - 4096), (ctypes.c_char * aligned).from_buffer(slab), aligned) == -1


@pytest.mark.gpu
def test_decode_record_and_batch_count():
    import torch
    L = lib()
    blob, ex = synth.make_experts(1024, 512, [(1, 0), (1, 1)], seed=88, sigma=0.02, cz=True, neg_zero=0.03, mode=2,
                                  train_every=1)
    mid = U32()
    assert L.coli_wex_register_model(blob, len(blob), ctypes.byref(mid)) == 0
    assert L.coli_wex_cuda_nr3_available() == 1 and L.coli_wex_cuda_batch_available() == 1
    before = L.coli_wex_cuda_decode_count()
    for e in ex:
        raw = len(e.source)
        aligned = (raw + 4095) & ~4095
        slab = bytearray(aligned)
        slab[aligned - len(e.record):] = e.record
        assert L.coli_wex_decode_record(np.frombuffer(e.entry, np.uint8).ctypes.data,
                                        (ctypes.c_char * aligned).from_buffer(slab), aligned) == 0
        assert bytes(slab[:raw]) == e.expected
    assert L.coli_wex_cuda_decode_count() == before + 2
    dst = torch.full((2, len(ex[0].source)), 0xA5, dtype=torch.uint8, device='cuda')
    s = ex[0].entry
    soff = [int.from_bytes(s[44 + 4 * m:48 + 4 * m], 'little') for m in range(3)]
    woff = [int.from_bytes(s[56 + 4 * m:60 + 4 * m], 'little') for m in range(3)]
    raw = len(ex[0].source)
    sp = [dst.data_ptr() + j * raw + soff[m] for j in range(2) for m in range(3)]
    wp = [dst.data_ptr() + j * raw + woff[m] for j in range(2) for m in range(3)]
    ep, keep = wexcuda._entries([e.entry for e in ex])
    recs = [np.frombuffer(e.record, np.uint8) for e in ex]
    status = (ctypes.c_int * 2)()
    d0 = L.coli_wex_cuda_device_decode_count()
    assert L.coli_wex_cuda_decode_batch_to_device(2, ep, wexcuda._ptrs([r.ctypes.data for r in recs]), 0,
                                                  wexcuda._ptrs(sp), wexcuda._ptrs(wp), status) == 0
    assert L.coli_wex_cuda_device_decode_count() == d0 + 2
    out = dst.cpu().numpy()
    assert all(out[j].tobytes() == ex[j].expected for j in range(2))
