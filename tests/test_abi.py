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


def _c_layouts(structs: dict[str, list[str]]) -> dict[str, list[int]]:
    """sizeof and offsetof of every named field of the header's structs, compiled by gcc."""
    import shutil
    import subprocess
    import tempfile

    import pytest

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stddef.h>", "#include <stdio.h>", f'#include "{HEADER}"', "int main(void) {"]
    for struct, fields in structs.items():
        parts = [f"(long)sizeof({struct})"] + [f"(long)offsetof({struct}, {f})" for f in fields]
        fmt = " ".join(["%ld"] * len(parts))
        lines.append(f'  printf("{struct} {fmt}\\n", {", ".join(parts)});')
    lines.append("  return 0;\n}")
    with tempfile.TemporaryDirectory() as tmp:
        src, exe = Path(tmp) / "layout.c", Path(tmp) / "layout"
        src.write_text("\n".join(lines))
        build = subprocess.run([cc, "-std=c11", str(src), "-o", str(exe)], capture_output=True, text=True)
        assert build.returncode == 0, build.stderr[-2000:]
        out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return {ln.split()[0]: [int(v) for v in ln.split()[1:]] for ln in out.splitlines()}


def test_ctypes_structs_match_the_header_layout():
    """Every args struct bound in Python has the C struct's size and the same offset
    for every field the binding names (explicit padding fields, named ``pad*``,
    stand for the compiler's implicit padding and are not compared)."""
    from dwarf_v2_b200 import _lib

    text = HEADER.read_text()
    struct_of = dict(re.findall(r"^int (dwarf_\w+)\(const (dwarf_\w+_args)\*", text, flags=re.M))
    bare = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    c_fields = {}
    for body, name in re.findall(r"typedef struct \{(.*?)\}\s*(dwarf_\w+_args);", bare, flags=re.S):
        names = set()
        for decl in body.split(";"):
            decl = re.sub(r"\[.*?\]", "", decl).strip()  # arrays: the name before [N]
            if decl:  # "type a, b" / "const void* p": the identifiers after the type
                head, *rest = decl.split(",")
                names.add(re.findall(r"\w+", head)[-1])
                names.update(r.strip().lstrip("*").strip() for r in rest)
        c_fields[name] = names
    structs, bindings, py_names = {}, {}, {}
    for entry, binding in _lib._ENTRY_POINTS.items():
        c_struct = struct_of[entry]
        pairs = []
        for name, _ in binding._fields_:
            if name.startswith("pad"):
                continue
            c_name = name if name in c_fields[c_struct] else name.rstrip("_")  # Python keywords: in_ -> in
            assert c_name in c_fields[c_struct], (c_struct, name)
            pairs.append((name, c_name))
        structs[c_struct] = [c for _, c in pairs]
        py_names[c_struct] = [n for n, _ in pairs]
        bindings[c_struct] = binding
    layouts = _c_layouts(structs)
    for c_struct, binding in bindings.items():
        got = [ctypes.sizeof(binding)] + [getattr(binding, f).offset for f in py_names[c_struct]]
        assert got == layouts[c_struct], (c_struct, list(zip(["sizeof"] + structs[c_struct], got, layouts[c_struct])))
