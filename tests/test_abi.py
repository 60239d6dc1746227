"""CPU: the C-ABI library loads and exports every symbol include/std_b200.h declares."""
import ctypes
import os
import re

from std_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(REPO, "include", "std_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(std_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_all_declared_symbols():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in std_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_host_side_argument_checks_without_gpu():
    lib = _lib.load()
    assert lib.std_version() == 100
    # bad shapes are rejected on the host before any CUDA call
    assert lib.std_draft_attn(None, None, None, None, 0, 1, 28, 4, 64, 16, None, None, None, 0, 0, None) == 1
    assert lib.std_verify_attn(None, None, None, None, 0, 19, 1, 1, 28, 4, 128, 16, None, None, None, 0, None) == 1
    assert lib.std_topk_select(None, 10, 1, None, 5, 6, None, None) == 1
    assert lib.std_draft_attn_workspace_bytes(1, 28, 4, 128, 1024) == 0  # merged in DSMEM
    # split partials: B*Hkv*splits rows of 128 x (128 fp32 + m, l)
    assert lib.std_verify_attn_workspace_bytes(8, 4, 33000) >= 8 * 4 * 128 * 128 * 4
