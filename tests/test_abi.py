"""CPU: the C-ABI library builds, loads and exports every declared symbol."""
import ctypes
import os
import re

import oracle as O
import smoe_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "smoe_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(smoe_cuda_\w+)\s*\(", src)))


def test_library_exports_header():
    L = smoe_cuda.lib()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert sorted(smoe_cuda.EXPORTS) == names


def test_canonical_helper_matches_libstdcxx_rule():
    for w in [0, 1, 0x80000000, 0xFFFFFF00, 0xFFFFFFFF, 123456 << 8]:
        assert smoe_cuda.canonical_from_u32(w) == O.canonical_from_word(w)


def test_struct_layouts():
    assert ctypes.sizeof(smoe_cuda.SamplerRow) == 24
    assert ctypes.sizeof(smoe_cuda.MoeLayer) == 8 + 8 + 72 + 16 + 8


def test_init_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        return
    L = smoe_cuda.lib()
    a = smoe_cuda.InitArgs(0, 0, 0, 0, 0, 0, 0)
    assert not L.smoe_cuda_init_ex(ctypes.byref(a))
    assert smoe_cuda.last_error() != ""
