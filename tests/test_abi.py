"""The C-ABI library loads on a machine without a GPU and exports every symbol that
include/g4.h declares (no compute calls here)."""
import ctypes
import re

from g4pkg import PKG_DIR, g4

HEADER = PKG_DIR.parent / "include" / "g4.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?(?:int|size_t|const char\*|void)\s*\*?\s*(g4_\w+)\s*\(", text,
                                 re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "g4_w4g32_gemm" in syms and "g4_last_error" in syms
    assert len(syms) >= 7


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(g4.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"declared in g4.h but not exported: {missing}"


def test_binding_covers_header():
    assert set(declared_symbols()) <= set(g4.SIGNATURES), set(declared_symbols()) - set(g4.SIGNATURES)


def test_abi_version_and_error_string():
    lib = g4.lib()
    assert lib.g4_abi_version() >= 1
    # argument checks run on the host before any CUDA call, so they work without a GPU
    rc = lib.g4_w4g32_gemm(None, None, None, None, 1, 8, 32, None, 8, None)
    assert rc == -1
    assert b"null" in lib.g4_last_error()


def test_serve_binary_is_built_and_answers_help():
    """g4_serve (the reference engine's process interface) is built beside libg4.so; --help needs no GPU."""
    import subprocess
    b = PKG_DIR / "g4_serve"
    assert b.exists()
    r = subprocess.run([str(b), "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "ENGINE_SERVE" in r.stderr
