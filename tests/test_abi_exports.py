"""CPU checks of the C-ABI library: it loads without a GPU and exports every function the headers
under include/ declare (no compute call is made here)."""
import ctypes
import os
import re

import wexcuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, 'include'))):
        if not h.endswith('.h'):
            continue
        text = open(os.path.join(ROOT, 'include', h)).read()
        text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
        for m in re.finditer(r'^\s*(?:const\s+)?(?:unsigned\s+int|int|void|size_t|uint32_t|uint64_t|unsigned)\s*\**\s*'
                             r'(\w+)\s*\(', text, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_function():
    L = wexcuda.lib()
    names = declared_functions()
    assert len(names) >= 17
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing


def test_abi_versions_without_gpu():
    L = wexcuda.lib()
    assert L.wex_cuda_helper_abi() == 1
    assert L.wex_cuda_helper_features() == 63
    assert L.wexb_abi() == 1


def test_argument_errors_need_no_gpu():
    L = wexcuda.lib()
    assert L.wex_cuda_decode_to_host(None, None, 0) == -1
    assert L.wex_cuda_decode_to_device(None, None, 0, None, None) == -1
    assert L.wex_cuda_decode_batch_to_device(0, None, None, 0, None, None, None) == 0
    assert L.wex_cuda_decode_batch_to_host(3, None, None, 0, None, None) == 3
    assert L.wex_cuda_host_register(None, 0) == -1
    assert L.wex_cuda_register_model(b'\0' * 16, 16) == -1
    assert wexcuda.selftest_bounded_wait(0, 0)[0] == -1 and wexcuda.selftest_bounded_wait(-1, 10)[0] == -1
