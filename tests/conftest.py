"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked `gpu` need a CUDA device (a B200 for the tcgen05 kernels); everything else runs on
the CPU. The oracle package is test infrastructure and may be imported here.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / 'tests' / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    return torch.device('cuda')


@pytest.fixture(scope='session')
def ext(cuda):
    from flash_whisper_b200.ext import load_ext
    return load_ext()


@pytest.fixture(scope='session')
def ref_ext(cuda):
    """The reference's own kernels (oracle/_ref), or skip if they were not built."""
    from oracle.build_ref import load_ref
    mod = load_ref()
    if mod is None:
        pytest.skip('oracle/_ref not built')
    return mod
