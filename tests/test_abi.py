"""The C ABI: the built library loads (no GPU needed) and exports every symbol include/*.h declares."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

from gs_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text):
            name = m.group(1)
            if name.startswith(("splat_", "gs2d_", "splat2d_", "gs3d_", "adam_")):
                names.add(name)
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_the_header():
    assert declared_functions() == set(_lib.exported_symbols())


def test_abi_version_and_error_channel():
    lib = _lib.load()
    assert lib.splat_abi_version() == _lib.ABI_VERSION
    # an argument error is reported without touching the GPU
    status = lib.splat_radix_sort_pairs(None, None, None, None, 10, 3, 0, 8, None, 0, None)
    assert status == 1
    assert b"key_bytes" in lib.splat_last_error()


def _prototypes() -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, [parameter types]) parsed from the header's prototypes."""
    out = {}
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"#[^\n]*", "", text)
        for m in re.finditer(r"([A-Za-z_][A-Za-z0-9_ \*]*?)\b([A-Za-z_][A-Za-z0-9_]*)\s*\(([^;{}]*?)\)\s*;", text):
            ret, name, params = m.group(1).strip(), m.group(2), m.group(3).strip()
            plist = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
            out[name] = (ret, plist)
    return out


def _kind(decl: str):
    if re.match(r"const char\s*\*", decl):
        return ctypes.c_char_p
    if "*" in decl:
        return ctypes.c_void_p
    if "size_t" in decl:
        return ctypes.c_size_t
    if "long long" in decl:
        return ctypes.c_longlong
    if re.search(r"\bdouble\b", decl):
        return ctypes.c_double
    if re.search(r"\bfloat\b", decl):
        return ctypes.c_float
    if re.search(r"\bint\b", decl):
        return ctypes.c_int
    raise AssertionError(f"unclassified parameter {decl!r}")


def test_ctypes_signatures_match_the_header():
    """Every argtypes list has the header's arity and kinds (a short list truncates the stream handle)."""
    protos = _prototypes()
    for name, (res, args) in _lib._SIGNATURES.items():
        ret, params = protos[name]
        want = [_kind(p) for p in params]
        assert args == want, f"{name}: ctypes {args} vs header {want}"
        if "*" in ret:
            assert res == ctypes.c_char_p, name
        elif "size_t" in ret:
            assert res == ctypes.c_size_t, name
        elif "long long" in ret:
            assert res == ctypes.c_longlong, name
        else:
            assert res == ctypes.c_int, name
