"""The C-ABI library: it builds for sm_100a, loads without a GPU, and exports every entry point the header
declares with the argument count the Python binding uses (no compute call is made here)."""
import os
import re

import pytest

from morj_b200 import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'include', 'morj_b200.h')


def declared():
    text = open(HEADER).read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    out = {}
    for m in re.finditer(r'\b(?:int|const char\*)\s+(morj_\w+)\(([^)]*)\);', text):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ('', 'void') else len(args.split(','))
    return out


def test_header_declares_the_entry_points():
    names = declared()
    assert {'morj_gemm_bf16', 'morj_tree_attention', 'morj_qkv_post', 'morj_label_head'} <= set(names)


def test_library_loads_and_exports_every_declared_symbol():
    from morj_b200.build import build
    build()
    lib = _native.lib()
    for name, argc in declared().items():
        assert hasattr(lib, name), name
        if name != 'morj_last_error':
            assert len(_native.SIGNATURES[name]) == argc, name
    assert set(_native.SIGNATURES) | {'morj_last_error'} == set(declared())
    assert lib.morj_version() == 100


def test_host_side_work_list_and_error_reporting():
    import ctypes
    import numpy as np
    lib = _native.lib()
    # segments of 130, 1, 0 and 69 queries over 130, 200, 5 and 69 keys; 64 queries per tile (2 heads per KV head)
    qo = np.array([0, 130, 131, 131, 200], dtype=np.int32)
    kv = np.array([0, 130, 330, 335, 404], dtype=np.int32)
    work = _native.attention_work(qo, kv, 0, 32, 16, 0)
    pairs = work.reshape(-1, 2).tolist()
    assert sorted(pairs) == [[0, 0], [0, 64], [0, 128], [1, 0], [3, 0], [3, 64]]
    # longest first: the segment-1 row sees 200 keys (4 chunks), segment 0's last tile 130 keys (3 chunks)
    assert pairs[0] == [1, 0] and pairs[1] == [0, 128]
    cap_fail = lib.morj_tree_attention_work(qo.ctypes.data_as(_native.IP), kv.ctypes.data_as(_native.IP), None, 4, 0,
                                            32, 16, 1, 0, work.ctypes.data_as(_native.IP), 2)
    assert cap_fail == -1 and b'exceed capacity' in lib.morj_last_error()
    # argument checks fail before any device access
    with pytest.raises(ValueError, match='multiples of 8'):
        _native.call('morj_gemm_bf16', 16, 7, 16, 7, 16, 16, 4, 16, 7, 0, None)
    with pytest.raises(ValueError, match='unknown epilogue'):
        _native.call('morj_gemm_bf16', 16, 64, 16, 64, 16, 64, 4, 16, 64, 9, None)
