"""The decode entry point that allocates nothing (wexb_decode_to_device_noalloc), for callers that may
not allocate device memory at run time: an engine that reserves all of HBM in its own pool at start-up,
or whose serving streams must not stall on the device synchronisation that cudaMalloc / cudaFree can
cause. It works in a fixed device array inside the library, so this test checks that its output is
the allocating entry point's (wex_cuda_decode_to_device), bit for bit, on two calls in a row (the
second call must not see the first call's leftovers), that a damaged record is still refused with the
destination untouched, and that a record larger than the fixed array is rejected with -2.

This file is collected last on purpose; it registers its own model, so it passes alone in a fresh
process as well as after the other tests."""
import ctypes

import numpy as np
import pytest

import synth
import wexcuda

pytestmark = pytest.mark.gpu
POISON = 0xA5


def _noalloc():
    L = wexcuda.lib()
    f = L.wexb_decode_to_device_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int

    def call(entry, record, device, dst_scale, dst_weight):
        e = np.frombuffer(bytes(entry), np.uint8).copy()
        r = np.frombuffer(bytes(record), np.uint8)
        return f(e.ctypes.data, r.ctypes.data, device, wexcuda._ptrs(dst_scale), wexcuda._ptrs(dst_weight))
    return call


def _buffers(torch, entry):
    e = np.frombuffer(bytes(entry), np.uint8)
    shapes = [(int.from_bytes(e[20 + 4 * m:22 + 4 * m], 'little'), int.from_bytes(e[22 + 4 * m:24 + 4 * m], 'little'))
              for m in range(3)]
    s = [torch.full((r * c,), POISON, dtype=torch.uint8, device='cuda') for r, c in shapes]
    w = [torch.full((r * c * 16,), POISON, dtype=torch.uint8, device='cuda') for r, c in shapes]
    return s, w


def _bytes(ts):
    return b''.join(bytes(t.cpu().numpy()) for t in ts)


def test_noalloc_matches_the_allocating_entry_point():
    import torch
    assert torch.cuda.is_available()
    noalloc = _noalloc()
    # two experts of the mid shape, canonical zero and ceil-form blocks, then a damaged copy
    blob, ex = synth.make_experts(2048, 768, [(7, 3), (7, 9)], seed=606, sigma=0.025, cz=True, neg_zero=0.03,
                                  mode=2, train_every=1)
    assert wexcuda.register_model(blob) == 0
    for e in ex:   # two calls in a row through the fixed array
        ref_s, ref_w = _buffers(torch, e.entry)
        assert wexcuda.decode_to_device(e.entry, e.record, 0, [t.data_ptr() for t in ref_s],
                                        [t.data_ptr() for t in ref_w]) == 0
        got_s, got_w = _buffers(torch, e.entry)
        assert noalloc(e.entry, e.record, 0, [t.data_ptr() for t in got_s], [t.data_ptr() for t in got_w]) == 0
        torch.cuda.synchronize()
        assert _bytes(got_s) == _bytes(ref_s) and _bytes(got_w) == _bytes(ref_w)
        assert _bytes(got_s) + _bytes(got_w) == e.expected
    bad = bytearray(ex[1].record)
    bad[9000] ^= 0x21
    got_s, got_w = _buffers(torch, ex[1].entry)
    assert noalloc(ex[1].entry, bytes(bad), 0, [t.data_ptr() for t in got_s], [t.data_ptr() for t in got_w]) == -1
    assert all(bool((t == POISON).all()) for t in got_s + got_w)
    # and a clean call right after the refused one
    assert noalloc(ex[0].entry, ex[0].record, 0, [t.data_ptr() for t in got_s], [t.data_ptr() for t in got_w]) == 0
    assert _bytes(got_s) + _bytes(got_w) == ex[0].expected
    # what the entry point exists for: after the set-up call above, further calls leave the device's
    # free memory exactly as it was (no allocation of any size, by the library or the runtime)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(0)[0]
    for e in ex * 2:
        assert noalloc(e.entry, e.record, 0, [t.data_ptr() for t in got_s], [t.data_ptr() for t in got_w]) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free_before
    # and the caller's current device is the one it had before the call
    assert torch.cuda.current_device() == 0


def test_noalloc_rejects_records_beyond_its_fixed_size():
    import torch
    noalloc = _noalloc()
    # an expert of hidden 8192 and FFN 2048 decodes to 26.7 MB, above the 24 MiB maximum
    blob, ex = synth.make_experts(8192, 2048, [(0, 0)], seed=17, sigma=0.02, train_every=1)
    e = ex[0]
    assert e.codec == 5 and len(e.source) > 24 << 20
    assert wexcuda.register_model(blob) == 0
    s, w = _buffers(torch, e.entry)
    assert noalloc(e.entry, e.record, 0, [t.data_ptr() for t in s], [t.data_ptr() for t in w]) == -2
    assert all(bool((t == POISON).all()) for t in s + w)


def test_noalloc_holds_at_most_four_models_per_device():
    """The array has table room for 4 models per device: a model that finds every slot taken is
    refused with 1 (unavailable) and its destination is left untouched; models already held still decode.
    Runs last in this file, since it fills the slots; earlier tests (here or in other files) may have
    taken some, so at most 4 of 5 new models fit and the fifth is refused."""
    import torch
    noalloc = _noalloc()
    got = []
    experts = []
    for k in range(5):   # five different models, one small expert each
        blob, ex = synth.make_experts(1024, 512, [(k, 1)], seed=700 + k, sigma=0.02 + 0.002 * k, train_every=1)
        assert wexcuda.register_model(blob) == 0
        e = ex[0]
        s, w = _buffers(torch, e.entry)
        st = noalloc(e.entry, e.record, 0, [t.data_ptr() for t in s], [t.data_ptr() for t in w])
        torch.cuda.synchronize()
        got.append(st)
        experts.append((e, st))
        if st == 0:
            assert _bytes(s) + _bytes(w) == e.expected
        else:
            assert all(bool((t == POISON).all()) for t in s + w)
    fit = got.count(0)
    assert got == [0] * fit + [1] * (5 - fit) and 1 <= fit <= 4, got
    e, _ = experts[0]   # a model that got a slot keeps decoding
    s, w = _buffers(torch, e.entry)
    assert noalloc(e.entry, e.record, 0, [t.data_ptr() for t in s], [t.data_ptr() for t in w]) == 0
    torch.cuda.synchronize()
    assert _bytes(s) + _bytes(w) == e.expected
