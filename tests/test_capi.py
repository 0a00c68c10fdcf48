"""CPU checks of the C-ABI boundary: the header compiles as C, and the built library loads and
exports every symbol the header declares (no kernel is launched here)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mpq_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mpq_[a-z0-9_]+)\s*\(", text)))


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "mpq_b200.h"\nint main(void){return 0;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", f"-I{ROOT / 'include'}", str(src)],
                   check=True)


def test_library_exports_every_declared_symbol():
    from mpq_b200 import _lib
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.mpq_abi_version() == 1


def test_bindings_cover_header():
    from mpq_b200 import _lib
    names = set(declared_symbols()) - {"mpq_last_error", "mpq_abi_version"}
    assert names <= set(_lib.SIGNATURES), sorted(names - set(_lib.SIGNATURES))


def test_invalid_argument_reports_error_without_gpu():
    """Argument validation runs on the host before any launch."""
    from mpq_b200 import _lib
    lib = _lib.load()
    st = lib.mpq_gemm_f32(7, 1, 1, 1, ctypes.c_float(1.0), None, 1, None, 1, ctypes.c_float(0.0), None, 1, None)
    assert st == 10001
    assert b"null pointer" in lib.mpq_last_error() or b"layout" in lib.mpq_last_error()
