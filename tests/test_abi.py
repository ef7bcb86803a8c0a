"""CPU checks of the drop-in C ABI: the libraries load, export every symbol the
headers declare, and the ctypes argtypes agree with the header signatures.
No kernel is launched (no GPU needed)."""

import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO

INCLUDE = os.path.join(REPO, "include")


def _ctype_of(param: str):
    """ctypes type of one C parameter declaration (pointers and streams are
    c_void_p at this ABI)."""
    p = param.strip()
    if "*" in p or p.startswith("cudaStream_t"):
        return ctypes.c_void_p
    base = p.rsplit(None, 1)[0] if len(p.split()) > 1 else p
    base = base.replace("const ", "").strip()
    return {"int": ctypes.c_int, "float": ctypes.c_float, "unsigned long long": ctypes.c_ulonglong,
            "unsigned int": ctypes.c_uint, "size_t": ctypes.c_size_t}[base]


def header_functions(path):
    """{name: [ctypes type per parameter]} for every function prototype in a header."""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    funcs = {}
    for m in re.finditer(r"^\s*(?:void|int|size_t)\s+(\w+)\s*\(([^;{]*?)\)\s*;", src, flags=re.M | re.S):
        name, params = m.group(1), m.group(2).strip()
        funcs[name] = [] if params in ("", "void") else [_ctype_of(x) for x in params.split(",")]
    return funcs


HEADERS = {
    "qwen_fused.h": "libqwen_fused.so",
    "qwen_step.h": "libqwen_fused.so",
    "qwen_fp8.h": "libqwen_fp8.so",
}


@pytest.mark.parametrize("header", sorted(HEADERS))
def test_library_exports_every_declared_symbol(header):
    from qwen35_b200 import _lib
    lib = ctypes.CDLL(os.path.join(_lib.LIB_DIR, HEADERS[header]))
    funcs = header_functions(os.path.join(INCLUDE, header))
    assert len(funcs) >= 1
    missing = [f for f in funcs if not hasattr(lib, f)]
    assert not missing, f"{HEADERS[header]} lacks {missing}"


def test_ctypes_bindings_match_headers():
    """Every binding's argtypes equal the header's parameter types one by one
    (pointer and stream parameters as c_void_p)."""
    from qwen35_b200 import _lib
    fused = header_functions(os.path.join(INCLUDE, "qwen_fused.h"))
    fused.update(header_functions(os.path.join(INCLUDE, "qwen_step.h")))
    fp8 = header_functions(os.path.join(INCLUDE, "qwen_fp8.h"))
    for name, argtypes in _lib.REFERENCE_FUSED_ARGTYPES.items():
        assert fused[name] == list(argtypes), name
    for name, (_, argtypes) in _lib.NEW_FUSED.items():
        assert fused[name] == list(argtypes), name
    for name, argtypes in _lib.REFERENCE_FP8_ARGTYPES.items():
        assert fp8[name] == list(argtypes), name
    # every declared symbol is bound
    assert set(fused) == set(_lib.REFERENCE_FUSED_ARGTYPES) | set(_lib.NEW_FUSED)
    assert set(fp8) == set(_lib.REFERENCE_FP8_ARGTYPES) | set(_lib.NEW_FP8)


def test_bindings_load_through_loader():
    from qwen35_b200 import _lib
    assert _lib.fused().qwen_abi_version() == 1
    assert _lib.fp8() is not None


@pytest.mark.parametrize("header", sorted(HEADERS))
def test_headers_compile_as_c(header, tmp_path):
    src = tmp_path / "t.c"
    src.write_text(f'#include "{header}"\nint main(void) {{ return 0; }}\n')
    r = subprocess.run(["gcc", "-fsyntax-only", "-I", INCLUDE, "-I", "/usr/local/cuda/include", str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


REF_ROOT = os.environ.get("QWEN_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")
REF_MAIN = os.path.join(REF_ROOT, "main.py")


@pytest.mark.skipif(not os.path.exists(REF_MAIN), reason="reference checkout not present")
def test_reference_argtypes_are_mirrored():
    """Every argtypes list main.py declares has the same length here."""
    from qwen35_b200 import _lib
    src = open(REF_MAIN).read()
    for m in re.finditer(r"_(fused|fp8)_dll\.(\w+)\.argtypes\s*=\s*\[(.*?)\]", src, flags=re.S):
        which, name, body = m.groups()
        n = body.count("ctypes.c_")
        table = _lib.REFERENCE_FUSED_ARGTYPES if which == "fused" else _lib.REFERENCE_FP8_ARGTYPES
        assert name in table, name
        assert len(table[name]) == n, name
