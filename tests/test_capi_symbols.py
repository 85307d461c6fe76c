"""The C-ABI library loads and exports every function include/*.h declares (no GPU
needed; nothing here launches work)."""
import ctypes
import glob
import os
import re

import pytest

from asicfortranai_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[\w\s\*]+?\b(\w+)\s*\(", txt, flags=re.M):
            nm = m.group(1)
            if nm not in ("if", "while", "for", "return", "sizeof", "defined"):
                names.add(nm)
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "matmul_3p5bit_awq" in names and "q35_gemm_dev" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    assert set(declared_functions()) <= set(_lib.SIGNATURES), \
        set(declared_functions()) - set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.q35_status_string(0) == b"ok"
    assert lib.q35_status_string(1) == b"invalid argument"
    assert lib.q35_version() >= 100


def test_invalid_sizes_rejected_before_any_device_work():
    lib = _lib.load()
    # K odd -> invalid argument, reported without touching the device
    st = lib.q35_matmul_3p5bit_awq(None, None, None, None, None, 1, 4, 3)
    assert st == 1
    assert "K must be even" in _lib.last_error() or "NULL" in _lib.last_error()
    st = lib.q35_matmul_int4_awq(None, None, None, None, 0, 4, 4)
    assert st == 1


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "q35.h"
int main(void) {
    /* argument checks answer before any device work */
    int st = q35_matmul_3p5bit_awq(0, 0, 0, 0, 0, 1, 4, 3);
    if (st != Q35_ERR_INVALID) return 1;
    if (strcmp(q35_status_string(Q35_OK), "ok") != 0) return 2;
    /* the reference's void signature reports a failure on stderr */
    int32_t c[4] = {7, 7, 7, 7};
    matmul_3p5bit_awq(0, 0, 0, 0, c, 1, 4, 3);
    if (c[0] != 7) return 3;   /* outputs untouched on failure */
    printf("%d %s\n", q35_version(), q35_last_error());
    return 0;
}
"""


@pytest.mark.parametrize("lang", ["c99", "c++11"])
def test_header_compiles_and_links_as_plain_c_and_cpp(tmp_path, lang):
    """include/q35.h is a plain C header: a C99 (and a C++11) program that includes it
    compiles warning-free, links against libq35 and calls entry points that need no GPU."""
    import shutil
    import subprocess
    cc = "gcc" if lang == "c99" else "g++"
    if shutil.which(cc) is None:
        pytest.skip(f"{cc} not installed")
    _lib.load()
    src = tmp_path / "prog.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "prog"
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    flags = ["-std=c99", "-pedantic"] if lang == "c99" else ["-std=c++11", "-x", "c++"]
    subprocess.run([cc, *flags, "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(src), "-L", lib_dir, "-lq35", "-Wl,-rpath," + lib_dir, "-o", str(exe)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split()[0] == str(_lib.load().q35_version())
    assert "matmul_3p5bit_awq: K must be even" in out.stderr, out.stderr
