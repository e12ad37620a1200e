"""Builds libflashwhisper.so (the C-ABI library) in-tree with nvcc for sm_100a.

`python -m flash_whisper_b200.build` compiles every csrc/*.cu to an object (in parallel) and links
them into flash_whisper_b200/libflashwhisper.so. The ptxas register / spill report of each file is
written to flash_whisper_b200/_build/ptxas_<name>.log. The reference built its extension with
torch.utils.cpp_extension at import time (custom/ext.py:13-18); this library is plain C ABI and is
built ahead of time so the .so travels with the source tree.
"""

import concurrent.futures
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / 'csrc'
BUILD = PKG / '_build'
LIB = PKG / 'libflashwhisper.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xptxas=-v,-warn-spills', '-Xcompiler', '-fPIC',
              '--expt-relaxed-constexpr', '-I', str(PKG.parent / 'include')]


def _nvcc():
    cuda = os.environ.get('CUDA_HOME', '/usr/local/cuda')
    path = Path(cuda) / 'bin' / 'nvcc'
    return str(path) if path.exists() else 'nvcc'


def _sources():
    return sorted(CSRC.glob('*.cu'))


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src, headers):
    obj = BUILD / (src.stem + '.o')
    if not _stale(obj, [src, *headers]):
        return obj, None
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, '-c', str(src), '-o', str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    (BUILD / f'ptxas_{src.stem}.log').write_text(proc.stdout + proc.stderr)
    if proc.returncode != 0:
        return obj, f'{" ".join(cmd)}\n{proc.stdout}\n{proc.stderr}'
    return obj, None


def build(verbose=False, force=False):
    """Compiles and links the library if any source is newer than it. Returns the .so path."""
    BUILD.mkdir(exist_ok=True)
    headers = [*CSRC.glob('*.cuh'), *CSRC.glob('*.h'), *(PKG.parent / 'include').glob('*.h')]
    srcs = _sources()
    if force:
        for o in BUILD.glob('*.o'):
            o.unlink()
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(srcs)) as pool:
        results = list(pool.map(lambda s: _compile(s, headers), srcs))
    errors = [err for _, err in results if err]
    if errors:
        raise RuntimeError('nvcc failed:\n' + '\n'.join(errors))
    objs = [obj for obj, _ in results]
    if _stale(LIB, objs) or force:
        cmd = [_nvcc(), *ARCH, '-shared', '-Xcompiler', '-fPIC', *map(str, objs), '-o', str(LIB)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f'link failed:\n{" ".join(cmd)}\n{proc.stdout}\n{proc.stderr}')
    if verbose:
        for src in srcs:
            log = BUILD / f'ptxas_{src.stem}.log'
            if log.exists():
                for line in log.read_text().splitlines():
                    if 'registers' in line or 'spill' in line.lower() or 'error' in line.lower():
                        print(f'{src.name}: {line.strip()}')
    return LIB


if __name__ == '__main__':
    build(verbose=True, force='--force' in sys.argv)
    print(f'built {LIB}')
