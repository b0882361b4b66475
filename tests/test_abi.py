"""C ABI (include/dwarf_b200.h): the shared library loads on a machine without a
GPU, reports the header's ABI version and exports every function the header
declares; every declared entry point has a ctypes binding. No compute calls."""

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "dwarf_b200.h"


def _declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|void)\s+\**(dwarf_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "dwarf_abi_version" in names and "dwarf_dsqg_fwd" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    from dwarf_v2_b200 import _build

    path = _build.build()
    lib = ctypes.CDLL(str(path))
    missing = [name for name in _declared() if not hasattr(lib, name)]
    assert not missing, f"symbols declared in dwarf_b200.h but not exported: {missing}"
    version = int(re.search(r"#define DWARF_ABI_VERSION (\d+)", HEADER.read_text()).group(1))
    lib.dwarf_abi_version.restype = ctypes.c_int
    assert lib.dwarf_abi_version() == version


def test_every_args_entry_point_is_bound():
    from dwarf_v2_b200 import _lib

    text = HEADER.read_text()
    with_args = set(re.findall(r"^int (dwarf_\w+)\(const dwarf_\w+_args\*", text, flags=re.M))
    assert with_args <= set(_lib._ENTRY_POINTS), sorted(with_args - set(_lib._ENTRY_POINTS))
