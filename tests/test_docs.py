"""The integration guide's code agrees with the library: every libq35 function its C, Go
and Fortran snippets call exists in include/q35.h with that many arguments, the Fortran
interface block binds existing symbols with the right argument counts, and the Python
snippet's calls name existing functions and methods."""
import os
import re

from tests.test_capi_symbols import _prototypes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _blocks(lang):
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return re.findall(r"```" + lang + r"\n(.*?)```", text, flags=re.S)


def _calls(code):
    """(name, argument count) of each call of a q35_* / matmul_* function in code"""
    out = []
    for m in re.finditer(r"\b((?:C\.)?(?:q35_\w+|matmul_3p5bit_awq))\s*\(", code):
        depth, i, args, cur = 1, m.end(), [], ""
        while depth:
            ch = code[i]
            if ch in "([{":
                depth += 1
            elif ch in ")]}":
                depth -= 1
            if depth == 1 and ch == ",":
                args.append(cur)
                cur = ""
            elif depth:
                cur += ch
            i += 1
        if cur.strip():
            args.append(cur)
        out.append((m.group(1).replace("C.", ""), len(args)))
    return out


def test_c_and_go_snippets_call_existing_functions():
    protos = _prototypes()
    calls = [c for lang in ("c", "go") for b in _blocks(lang) for c in _calls(b)]
    assert len(calls) >= 6
    for name, n in calls:
        assert name in protos, name
        assert n == len(protos[name][1]), (name, n, protos[name][1])


def test_fortran_interface_block_binds_existing_symbols():
    protos = _prototypes()
    (block,) = _blocks("fortran")
    heads = re.findall(r"function\s+(\w+)\s*\(([^)]*)\)\s*bind\(C\)", block)
    assert len(heads) >= 3
    for name, args in heads:
        assert name in protos, name
        assert len([a for a in args.split(",") if a.strip()]) == len(protos[name][1]), name


def test_python_snippet_names_existing_api():
    import importlib
    (block,) = _blocks("python")
    for mod, names in re.findall(r"from (asicfortranai_b200[\w.]*) import ([\w, ]+)", block):
        m = importlib.import_module(mod)
        for n in names.split(","):
            assert hasattr(m, n.strip()), (mod, n)
    from asicfortranai_b200.llama_model import LLaMAModel
    from asicfortranai_b200.quantized import Context, QuantizedMatrix
    for obj, meth in re.findall(r"\b(m|W|ctx|g)\.(\w+)\(", block):
        cls = {"m": LLaMAModel, "W": QuantizedMatrix, "ctx": Context}.get(obj)
        if cls is not None:
            assert hasattr(cls, meth), (obj, meth)
