"""The C-ABI library loads and exports every function its public headers
declare (no GPU needed: nothing is called)."""
import ctypes
import glob
import os
import re

from conftest import ROOT, PKG

LIB = os.path.join(PKG, "libapus_gcuda.so")


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"typedef[^;]*;", "", src, flags=re.S)
        for m in re.finditer(r"\b(apus_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_header_symbols():
    assert os.path.exists(LIB), "libapus_gcuda.so not built"
    lib = ctypes.CDLL(LIB)
    names = declared_functions()
    assert len(names) > 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_mirror_binds_every_entry_point():
    """The host mirror (apus_gcuda.py) declares every C-ABI entry point with
    its argument types, except the hook-table filler, which only a C engine
    can use (it fills a struct of C function pointers)."""
    src = open(os.path.join(PKG, "apus_gcuda.py")).read()
    unbound = [n for n in declared_functions() if f'"{n}"' not in src and n != "apus_gcuda_fill_hooks"]
    assert not unbound, unbound
