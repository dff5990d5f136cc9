"""The C ABI library loads and exports every entry point include/katago_cuda.h declares (no GPU needed)."""

import ctypes
import os
import re

from katago_cuda import api


def declared():
    text = open(api.HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(kc_\w+)\s*\(", text, re.M)))


def test_header_parses():
    names = declared()
    assert "kc_model_load" in names and "kc_get_output" in names and len(names) >= 20


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(api.library_path())
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared()) <= set(api._SIGS)


def test_device_count_without_gpu_is_clean():
    # on a CPU-only machine the call succeeds with 0 usable devices
    n = api.device_count()
    assert n >= 0
