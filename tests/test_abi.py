"""The C-ABI library loads and exports every function include/krystal_cuda.h declares.

No compute call runs here (there may be no GPU); the GPU tests call through it.
"""
import re
from pathlib import Path

from krystal_b200 import abi

HEADER = Path(__file__).resolve().parent.parent / "include" / "krystal_cuda.h"


def declared_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(kc_[a-z_]+)\s*\(", text))


def test_header_and_binding_agree():
    assert declared_functions() == set(abi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.kc_abi_version() == 1


def test_struct_sizes_match_the_c_layout():
    import ctypes as C
    assert C.sizeof(abi.KcConfig) == 13 * 4 + 4 + 8 + 4 + 4  # 13 u32, pad, pointer, u32, tail pad
    assert C.sizeof(abi.KcBatchView) == 8 + 8 + 8 * 8
    assert C.sizeof(abi.KcBatchOut) == 8 * 11
