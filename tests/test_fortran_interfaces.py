"""The Fortran drop-in modules (asicfortranai_b200/fortran/*.f90) bind libq35 through
bind(C) interface blocks.  No Fortran compiler exists in this image, so this test reads
the interfaces as text and checks each against the C prototype of include/q35.h: the
symbol exists, the argument count matches, and every dummy argument has the C
parameter's class (a `value` integer/real of the same width, or a pointer for a dummy
passed by reference or a `type(c_ptr), value`); the result matches the C return type.
It also checks that the modules' public procedures keep the reference's names."""
import glob
import os
import re

from tests.test_capi_symbols import _kind_c, _prototypes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FDIR = os.path.join(ROOT, "asicfortranai_b200", "fortran")

_FKIND = {"c_int": "i32", "c_int32_t": "i32", "c_int64_t": "i64", "c_size_t": "i64",
          "c_float": "f32", "c_double": "f64"}


def _logical_lines(path):
    """free-form source with comments removed and & continuations joined"""
    out, cur = [], ""
    for raw in open(path):
        line = raw.split("!", 1)[0].rstrip() if '"' not in raw.split("!", 1)[0] else raw.rstrip()
        if not line.strip():
            continue
        s = line.strip()
        if s.startswith("&"):
            s = s[1:].strip()
        if s.endswith("&"):
            cur += s[:-1] + " "
            continue
        out.append(cur + s)
        cur = ""
    return out


def _split_top(s):
    parts, depth, cur = [], 0, ""
    for ch in s:
        if ch == "(":
            depth += 1
        elif ch == ")":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        parts.append(cur.strip())
    return parts


def _interfaces():
    """bind name -> (result class, [dummy classes in order], file)"""
    found = {}
    for path in sorted(glob.glob(os.path.join(FDIR, "*.f90"))):
        lines = _logical_lines(path)
        i = 0
        while i < len(lines):
            m = re.match(r"(?i)\s*(?:(.+?)\s+)?(function|subroutine)\s+(\w+)\s*\(([^)]*)\)\s*"
                         r"bind\s*\(\s*C\s*,\s*name\s*=\s*\"(\w+)\"\s*\)", lines[i])
            if not m:
                i += 1
                continue
            rtype, kind, fname, args, cname = m.groups()
            dummies = [a.strip().lower() for a in args.split(",") if a.strip()]
            decl = {}
            j = i + 1
            while not re.match(r"(?i)\s*end\s+(function|subroutine)", lines[j]):
                d = re.match(r"(?i)\s*(integer|real|type|character)\s*\(([^)]*)\)\s*(.*?)::\s*(.*)$", lines[j])
                if d:
                    base, kindsel, attrs, ents = d.groups()
                    is_value = "value" in attrs.lower()
                    for e in _split_top(ents):
                        nm = re.match(r"(\w+)", e).group(1).lower()
                        if not is_value or base.lower() == "type":
                            cls = "ptr"
                        else:
                            cls = _FKIND[kindsel.split("=")[-1].strip().lower()]
                        decl[nm] = cls
                j += 1
            if kind.lower() == "subroutine":
                rcls = "void"
            else:
                rm = re.match(r"(?i)(integer|real|type)\s*\(([^)]*)\)", rtype.strip())
                rcls = "ptr" if rm.group(1).lower() == "type" else _FKIND[rm.group(2).strip().lower()]
            found[cname] = (rcls, [decl[d] for d in dummies], os.path.basename(path))
            i = j + 1
    return found


def test_every_interface_matches_its_prototype():
    protos = _prototypes()
    ifaces = _interfaces()
    assert len(ifaces) >= 10
    for cname, (rcls, dcls, fname) in ifaces.items():
        assert cname in protos, (fname, cname)
        ret, params = protos[cname]
        assert len(dcls) == len(params), (fname, cname, dcls, params)
        assert rcls == _kind_c(ret + " x"), (fname, cname, rcls, ret)
        for d, p in zip(dcls, params):
            assert d == _kind_c(p), (fname, cname, d, p)


def test_modules_keep_the_reference_procedure_names():
    want = {
        "matmul_3p5bit_groq.f90": ("matmul_3p5bit_groq", {"matmul_3p5bit_awq", "dequantize_output_3p5bit"}),
        "matmul_int4_groq.f90": ("matmul_int4_groq", {"matmul_int4_awq", "dequantize_output"}),
        "sampling.f90": ("sampling", {"sample_greedy", "sample_top_k", "sample_top_p", "sample_temperature",
                                      "apply_temperature", "softmax"}),
        "weight_loader.f90": ("weight_loader", {"load_layer_weights"}),
    }
    for fname, (module, procs) in want.items():
        lines = _logical_lines(os.path.join(FDIR, fname))
        assert any(re.match(rf"(?i)\s*module\s+{module}\s*$", l) for l in lines), fname
        public = set()
        for l in lines:
            m = re.match(r"(?i)\s*public\s*::\s*(.*)$", l)
            if m:
                public |= {p.strip().lower() for p in m.group(1).split(",")}
        assert procs <= public, (fname, procs - public)
        for p in procs:   # each public procedure is defined in the module
            assert any(re.match(rf"(?i)\s*(?:pure\s+)?(?:\w+\s+)?(subroutine|function)\s+{p}\s*\(", l)
                       for l in lines), (fname, p)
