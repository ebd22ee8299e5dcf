"""The reference's own Python entry point, wex4/wex4.py, unmodified, over this library.

`python -I wex4/wex4.py {info,verify} FILE --dll LIB` binds LIB through its CLib class
(wex4/wex4.py:292-310): it loads the library, checks wex4_tools_abi() == 1 and sets the argument types
of every entry point it uses, then reads the container with its own Python reader and hands WNR3 / WBP1
records to the library (wex4/wex4.py:528-545, :687-710). These tests run the reference script itself
from the reference tree, so they run only where that tree is present (this host, not the GPU host):
  - `info` on every valid vector prints the same report through this library as through the
    reference's own compiled tool, which shows that every binding of CLib resolves here;
  - `verify` needs the GPU decode: without a GPU it is refused cleanly (status 1, "REFUSED"), never a
    crash. With a GPU, the same calls are covered by tests/test_wex4_container.py (wex4_check and
    wex4_decode_record_buf against the reference tool and the manifest digests)."""
import os
import subprocess
import sys

import pytest

import oracle
import wexcuda

WEX4_PY = os.path.join(oracle.REFERENCE, 'wex4', 'wex4.py')
VECTORS = os.path.join(oracle.REFERENCE, 'wex4', 'vectors')
pytestmark = pytest.mark.skipif(not os.path.exists(WEX4_PY), reason='the reference tree is not on this host')


def _run(*args):
    return subprocess.run([sys.executable, '-I', WEX4_PY, *args], capture_output=True, text=True, timeout=300)


def _valid_vectors():
    rows = [l.rstrip('\n').split('\t') for l in open(os.path.join(VECTORS, 'MANIFEST.tsv'), encoding='utf-8')
            if l.strip() and not l.startswith('#')]
    return [(os.path.join(VECTORS, r[0]), r) for r in rows if r[1] == 'accept' and os.path.exists(os.path.join(VECTORS, r[0]))]


def test_info_through_the_unmodified_reference_script():
    ref = oracle.ref_path('wex4_tools_ref.so')
    if ref is None:
        pytest.skip('reference tools not built')
    vectors = _valid_vectors()
    assert len(vectors) >= 10
    for path, _ in vectors:
        mine, theirs = _run('info', path, '--dll', wexcuda.lib_path()), _run('info', path, '--dll', ref)
        assert mine.returncode == 0 and theirs.returncode == 0, (path, mine.stderr, theirs.stderr)
        assert mine.stdout == theirs.stdout, path


def test_verify_without_a_gpu_is_refused_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip('a GPU is present: the decode path is covered by test_wex4_container.py')
    path, _ = next(p for p in _valid_vectors() if 'wnr3' in p[0])
    got = _run('verify', path, '--dll', wexcuda.lib_path())
    assert got.returncode == 1 and 'REFUSED' in got.stdout, (got.stdout, got.stderr)
