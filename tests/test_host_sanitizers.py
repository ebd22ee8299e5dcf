"""The library's host sources built with AddressSanitizer and UndefinedBehaviorSanitizer (g++, every
sanitizer error fatal; the kernel launchers stubbed out, no GPU) and driven by tests/sanitize/fuzz_host.cpp:
the WEX4 header and index checks and the record parsers (WNR2/WNR3, WBP1, WNR4 kind MX) over the golden
vectors, the written containers (RAW, WNR3 in both canonical-zero modes, WBP1, WNR4) and seeded mutants
of all of them. Skipped when g++ or the CUDA runtime headers and library are missing."""
import ctypes
import glob
import os
import shutil
import subprocess

import numpy as np
import pytest

import wex4file
import wexcuda
from test_wex4_written import tiny_file

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get('CUDA_HOME', '/usr/local/cuda')


def wbp1_file():
    """A container of three WBP1 (codec 6) records written by this library's encoder."""
    L = wexcuda.lib()
    L.wex4_bp_encode_record.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_void_p]
    rng = np.random.default_rng(3)
    recs = []
    for r, (n, planes, clog, tr) in enumerate([(70000, 2, 12, 1), (40000, 4, 10, 0), (5000, 1, 11, 0)]):
        f = (rng.standard_normal((n + 3) // 4) * 0.05).astype(np.float32).tobytes()[:n]
        cap = 2 * n + (1 << 16)
        out = ctypes.create_string_buffer(cap)
        written = ctypes.c_size_t()
        assert L.wex4_bp_encode_record(f, n, planes, clog, tr, r, out, cap, ctypes.byref(written)) == 0
        recs.append(wex4file.Record(out.raw[:written.value], n, 6, [(f'tensors.{r}', 2, (n,), n)]))
    return wex4file.write(recs)


def test_host_parsers_under_sanitizers(tmp_path):
    gxx = shutil.which('g++')
    lib = os.path.join(CUDA, 'lib64')
    if not gxx or not os.path.exists(os.path.join(CUDA, 'include', 'cuda_runtime.h')) or \
            not glob.glob(os.path.join(lib, 'libcudart.so*')):
        pytest.skip('g++ or the CUDA runtime is not installed')
    csrc = os.path.join(ROOT, 'wex-wrn2_b200', 'csrc')
    exe = str(tmp_path / 'fuzz_host')
    cmd = [gxx, '-std=c++17', '-O1', '-g', '-fsanitize=address,undefined', '-fno-sanitize-recover=all',
           '-fno-omit-frame-pointer', '-x', 'c++', '-I', os.path.join(CUDA, 'include'), '-I', os.path.join(ROOT, 'include'),
           '-I', csrc, os.path.join(ROOT, 'tests', 'sanitize', 'fuzz_host.cpp'),
           os.path.join(ROOT, 'tests', 'sanitize', 'stubs.cpp'), *sorted(glob.glob(os.path.join(csrc, '*.cpp'))),
           '-o', exe, '-L', lib, '-lcudart', '-lpthread']
    subprocess.run(cmd, check=True, timeout=900)
    files = sorted(glob.glob(os.path.join(ROOT, 'tests', 'golden', 'vectors', '*.wex4')))
    written = {'tiny.wex4': tiny_file(False)[0], 'tiny-cz.wex4': tiny_file(True)[0], 'wbp1.wex4': wbp1_file()}
    try:
        from test_wex4_written import mixed_file
        written['mixed.wex4'] = mixed_file()[0]
    except pytest.skip.Exception:   # the reference's WNR4 tool is not built here
        pass
    for name, data in written.items():
        (tmp_path / name).write_bytes(data)
        files.append(str(tmp_path / name))
    env = dict(os.environ, ASAN_OPTIONS='detect_leaks=0:abort_on_error=0',
               LD_LIBRARY_PATH=lib + ':' + os.environ.get('LD_LIBRARY_PATH', ''))
    r = subprocess.run([exe, '11', '30', *files], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-4000:])
    import re
    runs = int(r.stdout.split()[0])
    by_codec = dict(re.findall(r'(\d+) (\d+)[,\n]', r.stdout.split(':', 1)[1] + '\n'))
    by_codec = {k: int(v) for k, v in by_codec.items()}
    assert runs > 30 * len(files)
    assert by_codec['5'] > 0 and by_codec['6'] > 0 and ('mixed.wex4' not in written or by_codec['8'] > 0), r.stdout


def test_decode_queue_waits_only_for_earlier_items(tmp_path):
    """The decode launch's work queue (queue_fill) on 400 seeded random launches: every weight item after
    all scale items of its matrix, every commit item after all weight items of its record, every stream
    and commit chunk exactly once, and the descriptors' item counts equal to the queue's (the kernel's
    items wait only for earlier items, so the queue always drains). Built with the sanitizers as above."""
    gxx = shutil.which('g++')
    lib = os.path.join(CUDA, 'lib64')
    if not gxx or not os.path.exists(os.path.join(CUDA, 'include', 'cuda_runtime.h')) or \
            not glob.glob(os.path.join(lib, 'libcudart.so*')):
        pytest.skip('g++ or the CUDA runtime is not installed')
    csrc = os.path.join(ROOT, 'wex-wrn2_b200', 'csrc')
    exe = str(tmp_path / 'queue_order')
    cmd = [gxx, '-std=c++17', '-O1', '-g', '-fsanitize=address,undefined', '-fno-sanitize-recover=all',
           '-x', 'c++', '-I', os.path.join(CUDA, 'include'), '-I', os.path.join(ROOT, 'include'), '-I', csrc,
           os.path.join(ROOT, 'tests', 'sanitize', 'queue_order.cpp'), os.path.join(ROOT, 'tests', 'sanitize', 'stubs.cpp'),
           os.path.join(csrc, 'nr3_host.cpp'), os.path.join(csrc, 'host_wait.cpp'),
           '-o', exe, '-L', lib, '-lcudart', '-lpthread']
    subprocess.run(cmd, check=True, timeout=600)
    env = dict(os.environ, ASAN_OPTIONS='detect_leaks=0', LD_LIBRARY_PATH=lib + ':' + os.environ.get('LD_LIBRARY_PATH', ''))
    r = subprocess.run([exe, '5', '400'], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-4000:])
    assert int(r.stdout.split()[0]) > 10000
