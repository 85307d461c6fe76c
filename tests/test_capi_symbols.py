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
    st = lib.q35_matmul_int4_awq(None, None, None, None, -1, 4, 4)
    assert st == 1


def test_empty_operands_match_the_reference_loops():
    """M = 0 or N = 0: the reference's loops run no iterations -- success, nothing written.
    K = 0: every C(i,j) keeps its initial 0 and the dequantization follows from it
    (matmul_3p5bit_dynamic.f90:42-82, matmul_int4_groq.f90:33-69).  No device work."""
    import numpy as np
    from asicfortranai_b200.matmul_3p5bit_groq import dequantize_output_3p5bit, matmul_3p5bit_awq
    from asicfortranai_b200.matmul_int4_groq import dequantize_output, matmul_int4_awq
    lib = _lib.load()
    for M, N in ((0, 5), (3, 0), (0, 0)):
        assert lib.q35_matmul_3p5bit_awq(None, None, None, None, None, M, N, 8) == 0
        assert lib.q35_matmul_int4_awq(None, None, None, None, M, N, 8) == 0
        assert lib.q35_matmul_int4_fused(None, None, None, None, M, N, 8) == 0
        assert lib.q35_dequantize_output_3p5bit(None, None, None, None, M, N) == 0
        assert lib.q35_dequantize_output(None, None, None, M, N) == 0
    M, N = 3, 4
    s = np.array([0.5, -2.0, 1e-3, 3.0], np.float32)
    o = np.array([-7.0, 0.25, -0.0, 1.0], np.float32)
    A = np.zeros((M, 0), np.int8)
    W = np.zeros((0, N), np.int8)
    C = matmul_3p5bit_awq(A, W, s, o, M, N, 0)
    assert C.shape == (M, N) and (C == 0).all()
    C4 = matmul_int4_awq(A, W, s, M, N, 0)
    assert (C4 == 0).all()
    out = np.full((M, N), 9.0, np.float32, order="F")
    assert lib.q35_matmul_int4_fused(A.ctypes.data, W.ctypes.data, s.ctypes.data, out.ctypes.data, M, N, 0) == 0
    want = (np.float32(0) * s)[None, :].repeat(M, 0)          # -0.0 where the scale is negative
    np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))
    # an odd or negative K is still an error
    assert lib.q35_matmul_3p5bit_awq(None, None, None, None, None, 0, 4, 3) == 1
    assert lib.q35_matmul_3p5bit_awq(None, None, None, None, None, 2, 4, -2) == 1
    # zero-size arrays through the Python mirrors of the dequantization
    e = dequantize_output_3p5bit(np.zeros((0, N), np.int32), s, o, 0, N)
    assert e.shape == (0, N)
    assert dequantize_output(np.zeros((M, 0), np.int32), s[:0], M, 0).shape == (M, 0)


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


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """The Python mirrors of q35_model_config, q35_layer_weights and q35_sampling have the
    C header's size and field offsets (an ABI drift would pass garbage silently)."""
    import ctypes
    import json
    import shutil
    import subprocess
    from asicfortranai_b200.llama_model import LayerWeights, ModelConfig, Sampling
    if shutil.which("gcc") is None:
        pytest.skip("gcc not installed")
    structs = {"q35_model_config": ModelConfig, "q35_layer_weights": LayerWeights, "q35_sampling": Sampling}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "q35.h"', "int main(void) {", 'printf("{");']
    first = True
    for cname, py in structs.items():
        for f, _ in py._fields_:
            sep = "" if first else ","
            first = False
            lines.append(f'printf("{sep}\\"{cname}.{f}\\": %zu", offsetof({cname}, {f}));')
        lines.append(f'printf(",\\"{cname}.__size__\\": %zu", sizeof({cname}));')
    lines += ['printf("}\\n");', "return 0; }"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    got = json.loads(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    for cname, py in structs.items():
        assert got[f"{cname}.__size__"] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[f"{cname}.{f}"] == getattr(py, f).offset, (cname, f)


def _prototypes():
    """name -> (return type, [parameter types]) of every function include/*.h declares."""
    out = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        txt = re.sub(r"^\s*#.*$", "", txt, flags=re.M)
        for m in re.finditer(r"([\w\s\*]+?)\b(\w+)\s*\(([^;{}]*?)\)\s*;", txt):
            ret, name, params = m.group(1).strip(), m.group(2), m.group(3).strip()
            if name in ("if", "while", "for", "return", "sizeof") or ret.startswith("typedef"):
                continue
            plist = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
            out[name] = (" ".join(ret.split()), plist)
    return out


_OPAQUE = ("q35_ctx", "q35_weights", "q35_graph", "q35_tp", "q35_model")


def _kind_c(decl: str) -> str:
    """the ABI class of a C declaration: ptr, i32 (4-byte integer), i64 (8-byte integer),
    f32, f64 or void"""
    decl = " ".join(decl.replace("const", " ").split())
    if "*" in decl or decl.split()[0] in _OPAQUE:
        return "ptr"
    base = decl.split()[0]
    return {"int": "i32", "int32_t": "i32", "uint32_t": "i32", "int64_t": "i64", "uint64_t": "i64",
            "size_t": "i64", "float": "f32", "double": "f64", "void": "void"}[base]


def _kind_py(t) -> str:
    import ctypes
    if t is None:
        return "void"
    if t in (ctypes.c_void_p, ctypes.c_char_p) or isinstance(t, type) and issubclass(t, ctypes._Pointer):
        return "ptr"
    if t is ctypes.c_float:
        return "f32"
    if t is ctypes.c_double:
        return "f64"
    return "i64" if ctypes.sizeof(t) == 8 else "i32"


def test_python_signatures_match_the_prototypes():
    """Every ctypes binding has the C prototype's argument count and argument / return
    classes (pointer, 4- or 8-byte integer, float, double): a float passed where the
    C side takes a double, or a missing argument, would otherwise go unnoticed."""
    protos = _prototypes()
    assert set(protos) == set(declared_functions())
    for name, (ret, params) in protos.items():
        rt, at = _lib.SIGNATURES[name]
        assert len(at) == len(params), (name, params, at)
        assert _kind_py(rt) == _kind_c(ret + " x"), (name, ret, rt)
        for p, a in zip(params, at):
            assert _kind_c(p) == _kind_py(a), (name, p, a)
