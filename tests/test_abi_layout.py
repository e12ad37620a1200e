"""The ctypes mirrors of the C-ABI descriptor structs (flash_whisper_b200/_lib.py) against the C
compiler's own layout of include/flash_whisper.h: a small C program built with the host compiler
prints sizeof and every field's offsetof, and each must equal the ctypes structure's."""

import shutil
import subprocess

import pytest

from flash_whisper_b200 import _lib

STRUCTS = {
    'fw_decoder_t': _lib.Decoder,
    'fw_batch_decoder_t': _lib.BatchDecoder,
    'fw_encoder_t': _lib.Encoder,
    'fw_decoder_layer_t': _lib.DecoderLayer,
    'fw_encoder_layer_t': _lib.EncoderLayer,
}


@pytest.fixture(scope='module')
def c_layout(tmp_path_factory):
    cc = shutil.which('gcc') or shutil.which('cc')
    if cc is None:
        pytest.skip('no C compiler')
    d = tmp_path_factory.mktemp('abi')
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "flash_whisper.h"', 'int main(void) {']
    for cname, cls in STRUCTS.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append('  return 0;\n}')
    src = d / 'layout.c'
    src.write_text('\n'.join(lines) + '\n')
    exe = d / 'layout'
    subprocess.run([cc, '-std=c11', '-I', str(_lib.HEADER.parent), str(src), '-o', str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    table = {}
    for line in out.splitlines():
        name, field, value = line.split()
        table[(name, field)] = int(value)
    return table


@pytest.mark.parametrize('cname', list(STRUCTS))
def test_ctypes_struct_matches_c_layout(c_layout, cname):
    cls = STRUCTS[cname]
    assert c_layout[(cname, 'sizeof')] == __import__('ctypes').sizeof(cls)
    for field, _ in cls._fields_:
        assert c_layout[(cname, field)] == getattr(cls, field).offset, f'{cname}.{field}'
