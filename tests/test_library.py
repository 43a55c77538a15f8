"""The C-ABI library loads and exports every entry point include/mllm.h declares (no GPU needed)."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, pkg


def _declared():
    src = open(os.path.join(ROOT, "include", "mllm.h")).read()
    return sorted(set(re.findall(r"\b(mllm_[a-z0-9_]+)\s*\(", src)))


def test_header_and_exports_agree():
    P = pkg()
    decl = _declared()
    assert set(decl) == set(P.EXPORTS)
    L = P.load_library()
    for name in decl:
        assert hasattr(L, name), name


def test_create_rejects_bad_files_before_touching_a_device():
    """Format errors come from the C++ parser (pgw.cpp) ahead of any CUDA call."""
    P = pkg()
    L = P.load_library()
    good = open(os.path.join(GOLDEN, "ref_llama.pgw"), "rb").read()
    h = ctypes.c_void_p()

    def create(data):
        buf = np.frombuffer(data, np.uint8)
        return L.mllm_create(0, buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes, 1, 0, ctypes.byref(h))

    assert create(b"PGW9" + good[4:]) == -1
    assert b"bad magic" in L.mllm_last_error(None)
    assert create(good[:200]) == -1
    bad_table = bytearray(good)
    bad_table[256] = ord("{")
    assert create(bytes(bad_table)) == -1
    q8 = bytearray(good)
    q8[4] = 3
    assert create(bytes(q8)) == -2
    # head_dim 128 is rejected as unsupported
    hd = bytearray(good)
    hd[20:24] = (1).to_bytes(4, "little")
    assert create(bytes(hd)) == -2
