"""Builds the reference's own decode kernels for sm_100a into oracle/_ref/ (test infrastructure).

The reference compiles custom/kernels/whisper_kernels.cu at import time with
torch.utils.cpp_extension (custom/ext.py:13-18, flags :10). This recipe compiles the same single
source file, read in place from the reference checkout, with the same flags and
TORCH_CUDA_ARCH_LIST=10.0a, writing only into oracle/_ref/ (git-ignored, shipped to GPU boxes).
GPU tests load it with `load_ref()` to compare this package's kernels against the reference's on
identical inputs. Nothing is copied from the reference into the repository.

    python -m oracle.build_ref [/path/to/reference]

Without an argument the checkout is $FLASH_WHISPER_REFERENCE, else a directory named `reference` beside
this repository's directory.
"""

import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / '_ref'
SO_NAME = 'whisper_ext_ref'


def reference_checkout():
    """Path of the reference checkout ($FLASH_WHISPER_REFERENCE, else ../reference beside the repo)."""
    env = os.environ.get('FLASH_WHISPER_REFERENCE')
    return Path(env) if env else HERE.parent.parent / 'reference'


def build(reference=None):
    reference = reference_checkout() if reference is None else reference
    src = Path(reference) / 'custom' / 'kernels' / 'whisper_kernels.cu'
    if not src.exists():
        return None
    REF_DIR.mkdir(exist_ok=True)
    os.environ['TORCH_CUDA_ARCH_LIST'] = '10.0a'
    from torch.utils.cpp_extension import load
    try:
        load(name=SO_NAME, sources=[str(src)], build_directory=str(REF_DIR),
             extra_cuda_cflags=['-O3', '-lineinfo', '-Xptxas=-v,-warn-spills', '--expt-relaxed-constexpr'],
             extra_cflags=['-O3'], verbose=False)
    except Exception:
        pass  # importing may fail without a GPU; the built .so is what matters
    so = REF_DIR / f'{SO_NAME}.so'
    return so if so.exists() else None


def load_ref():
    """Imports the prebuilt reference kernel module (needs torch already imported), or None."""
    so = REF_DIR / f'{SO_NAME}.so'
    if not so.exists():
        return None
    import torch  # noqa: F401  (the extension links against libtorch)
    loader = importlib.machinery.ExtensionFileLoader(SO_NAME, str(so))
    spec = importlib.util.spec_from_file_location(SO_NAME, str(so), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == '__main__':
    out = build(Path(sys.argv[1]) if len(sys.argv) > 1 else None)
    print(f'built {out}' if out else 'reference source not found; nothing built')
