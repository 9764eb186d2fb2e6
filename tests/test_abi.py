"""The C-ABI library builds, loads and exports every entry point include/eps_b200.h
declares; without a GPU its calls fail loudly (no CPU fallback)."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT, gpu_available

HEADER = os.path.join(ROOT, "include", "eps_b200.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"EPS_B200_EXPORT\s+[\w\s\*]+?\b(eps_b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert "eps_b200_lookup" in names and "eps_b200_push" in names
    assert len(names) >= 12


def test_library_exports_every_declared_symbol(eps):
    so = eps.library_path()
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT\s+(eps_b200_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
    lib = ctypes.CDLL(so)
    for n in declared():
        assert hasattr(lib, n)


def test_python_binding_lists_entry_points(eps):
    assert set(eps.ENTRY_POINTS) == set(declared())


def test_abi_version(eps):
    assert eps.load_library().eps_b200_abi_version() == 3


def test_struct_sizes_match_header(eps):
    # sizes of the C structs as laid out by the C compiler
    src = r'''
#include <stdio.h>
#include "eps_b200.h"
int main(void){printf("%zu %zu %zu %zu %zu %zu\n", sizeof(EpsB200Status), sizeof(EpsB200Options),
 sizeof(EpsB200Table), sizeof(EpsB200Feature), sizeof(EpsB200Buffer), sizeof(EpsB200Stats));return 0;}
'''
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "s.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "s")
        subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe])
        sizes = [int(x) for x in subprocess.check_output([exe]).split()]
    py = [ctypes.sizeof(t) for t in (eps.Status, eps.Options, eps.Table, eps.Feature, eps.Buffer,
                                     eps.Stats)]
    assert sizes == py


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure path")
def test_no_gpu_fails_loudly(eps):
    with pytest.raises(eps.EpsError) as e:
        eps.ParameterStore(device=0)
    assert e.value.code in (eps.UNAVAILABLE, eps.RUN_FAILED)
