"""The C-ABI library loads on a CPU-only host and exports every symbol the
public header declares (no compute call without a GPU)."""
import ctypes
import os
import re

from fable5_llm_b200 import _lib

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_symbols():
    names = set()
    for fn in os.listdir(HDR):
        if fn.endswith(".h"):
            src = open(os.path.join(HDR, fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(f5_[a-z0-9_]+)\s*\(", src))
    return names


def test_header_symbols_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 10
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert declared_symbols() <= bound, sorted(declared_symbols() - bound)


def test_abi_version_without_gpu():
    assert _lib.lib().f5_abi_version() == 1
    assert _lib.lib().f5_status_string(-1) == b"invalid argument"
