"""The C-ABI library loads without a GPU and exports every function that
include/*.h declares (no compute calls are made here)."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT

DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(lcml_\w+)\s*\(", re.M)


def declared(header):
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    names = set(DECL.findall(src))
    return sorted(n for n in names if not n.endswith("_t"))


def test_fp8_header_symbols_exported():
    import luisaml_b200 as lb
    lib = lb.lib()
    names = declared(os.path.join(ROOT, "include", "lcml_fp8.h"))
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.lcml_abi_version() == 2  # 2: per-call `variant` fields in the GEMM and conv descriptors


def test_python_prototypes_cover_header():
    from luisaml_b200 import _capi
    names = declared(os.path.join(ROOT, "include", "lcml_fp8.h"))
    bound = set(_capi.PROTOTYPES) | {"lcml_last_error", "lcml_launch_count"}
    assert not [n for n in names if n not in bound]


@pytest.mark.parametrize("header", sorted(glob.glob(os.path.join(ROOT, "include", "*.h"))))
def test_every_header_resolves(header):
    libs = [ctypes.CDLL(p) for p in glob.glob(os.path.join(ROOT, "luisaml_b200", "lib", "*.so"))]
    names = declared(header)
    for n in names:
        assert any(hasattr(l, n) for l in libs), f"{n} declared in {os.path.basename(header)} but not exported"
