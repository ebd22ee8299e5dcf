"""Builds the native libraries of the package in-tree (wex-wrn2_b200/lib/):

  libwexb200.so      the CUDA decoder and every C-ABI entry point declared in include/*.h
                     (nvcc, sm_100a only)
  libwexb_tools.so   the writer-side tools (synthetic MXFP4 experts, WNR3 and WNR4 encoders), host C

Run `python wex-wrn2_b200/build.py` or call build(). Rebuilds only what is older than its sources.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, 'lib')
CSRC = os.path.join(HERE, 'csrc')
CUDA_LIB = os.path.join(LIB, 'libwexb200.so')
TOOLS_LIB = os.path.join(LIB, 'libwexb_tools.so')
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def cuda_sources():
    return sorted(glob.glob(os.path.join(CSRC, '*.cu')) + glob.glob(os.path.join(CSRC, '*.cpp')))


def cuda_deps():
    return cuda_sources() + sorted(glob.glob(os.path.join(CSRC, '*.cuh')) + glob.glob(os.path.join(CSRC, '*.h')) +
                                   glob.glob(os.path.join(ROOT, 'include', '*.h')))


def build_tools(verbose=False):
    src = [os.path.join(CSRC, 'tools', 'wexb_tools.c'), os.path.join(CSRC, 'tools', 'wexb_wnr4.c')]
    if _stale(TOOLS_LIB, src):
        os.makedirs(LIB, exist_ok=True)
        cmd = ['gcc', '-O2', '-Wall', '-Wextra', '-shared', '-fPIC', '-o', TOOLS_LIB] + src + ['-lm', '-lpthread']
        if verbose:
            print(' '.join(cmd))
        subprocess.run(cmd, check=True)
    return TOOLS_LIB


def build_cuda(verbose=False, extra=()):
    deps = cuda_deps()
    if not deps:
        return None
    if _stale(CUDA_LIB, deps) or extra:
        os.makedirs(LIB, exist_ok=True)
        objs, cmds = [], []
        for src in cuda_sources():
            obj = os.path.join(LIB, os.path.basename(src) + '.o')
            cmd = [NVCC, '-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC,-fvisibility=hidden', '-I',
                   os.path.join(ROOT, 'include'), '-I', CSRC, *ARCH, *extra, '-c', src, '-o', obj]
            if src.endswith('.cpp'):
                cmd.insert(1, '-x'); cmd.insert(2, 'cu')
            if verbose:
                print(' '.join(cmd))
            cmds.append(cmd)
            objs.append(obj)
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(max(1, min(len(cmds), os.cpu_count() or 4))) as pool:
            for r in list(pool.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds)):
                if r.returncode:
                    sys.stderr.write(r.stdout + r.stderr)
                    raise subprocess.CalledProcessError(r.returncode, r.args)
                if verbose and (r.stdout or r.stderr):
                    sys.stderr.write(r.stdout + r.stderr)
        cmd = [NVCC, '-shared', *ARCH, '-o', CUDA_LIB, *objs, '-lcudart_static', '-lpthread', '-ldl', '-lrt']
        if verbose:
            print(' '.join(cmd))
        subprocess.run(cmd, check=True)
        for o in objs:
            os.remove(o)
    return CUDA_LIB


def build(verbose=False):
    build_tools(verbose)
    build_cuda(verbose)


if __name__ == '__main__':
    build(verbose='-v' in sys.argv)
