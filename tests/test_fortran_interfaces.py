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
        # transformer_layer.f90:16-18, llama_model.f90:11, matmul_cublas.f90:16-18,
        # matmul_cuda_fortran.cuf:21, matmul_openacc.f90:20, transformer_layer_gpu.f90:23-24,
        # llama_model_gpu.f90:19
        "transformer_layer.f90": ("transformer_layer", {"apply_transformer_layer", "init_rope_freqs",
                                                        "init_kv_cache", "reset_kv_cache", "rms_norm"}),
        "llama_model.f90": ("llama_model", {"init_llama_model", "forward_llama", "cleanup_llama_model"}),
        "matmul_cublas.f90": ("matmul_cublas", {"matmul_int4_cublas", "matmul_int4_cublas_cached", "cublas_init",
                                                "cublas_shutdown", "dequantize_weights_gpu", "allocate_gpu_memory"}),
        "matmul_cuda_fortran.f90": ("matmul_cuda_fortran", {"matmul_int4_cuda", "matmul_int4_cuda_fused"}),
        "matmul_openacc.f90": ("matmul_openacc", {"matmul_int4_openacc", "dequantize_output_openacc"}),
        "transformer_layer_gpu.f90": ("transformer_layer_gpu", {"init_gpu_layer", "apply_transformer_layer_gpu",
                                                                "cleanup_gpu_layer"}),
        "llama_model_gpu.f90": ("llama_model_gpu", {"init_llama_model_gpu", "forward_llama_gpu",
                                                    "cleanup_llama_model_gpu"}),
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


def test_module_types_and_constants_keep_the_reference_names():
    """The derived types and the dimension constants of transformer_layer.f90:16-18 and
    llama_model.f90:11 / llama_model_gpu.f90:19 are public under the same names, and the
    types keep every reference component."""
    want = {
        "transformer_layer.f90": ("TransformerLayer", {"HIDDEN_DIM", "INTERMEDIATE_DIM", "NUM_HEADS", "NUM_KV_HEADS",
                                                       "HEAD_DIM"},
                                  {"wq", "wk", "wv", "wo", "wq_scales", "wk_scales", "wv_scales", "wo_scales",
                                   "w_gate", "w_up", "w_down", "w_gate_scales", "w_up_scales", "w_down_scales",
                                   "attn_norm", "ffn_norm", "rope_freqs", "k_cache", "v_cache", "cache_pos"}),
        "llama_model.f90": ("LLaMAModel", set(), {"token_embeddings", "layers", "final_norm", "output_weights",
                                                  "num_layers", "max_seq_len"}),
        "llama_model_gpu.f90": ("LLaMAModelGPU", set(), {"token_embeddings", "layers", "final_norm",
                                                         "output_weights", "num_layers", "max_seq_len",
                                                         "gpu_initialized"}),
    }
    for fname, (tname, consts, comps) in want.items():
        lines = _logical_lines(os.path.join(FDIR, fname))
        public = set()
        for l in lines:
            m = re.match(r"(?i)\s*public\s*::\s*(.*)$", l)
            if m:
                public |= {p.strip().lower() for p in m.group(1).split(",")}
        assert {tname.lower()} | {c.lower() for c in consts} <= public, fname
        i = next(i for i, l in enumerate(lines) if re.match(rf"(?i)\s*type\s*::\s*{tname}\s*$", l))
        got = set()
        while not re.match(r"(?i)\s*end\s+type", lines[i]):
            m = re.match(r"(?i)\s*[^:]*::\s*(.*)$", lines[i])
            if m and i > 0:
                got |= {re.match(r"(\w+)", e).group(1).lower() for e in _split_top(m.group(1))}
            i += 1
        assert comps <= got, (fname, comps - got)


def _bind_c_type(path, tname):
    """[(component, class)] of a bind(C) derived type, in order"""
    lines = _logical_lines(path)
    i = next(i for i, l in enumerate(lines) if re.match(rf"(?i)\s*type\s*,\s*bind\s*\(\s*C\s*\)\s*::\s*{tname}\s*$", l))
    out = []
    i += 1
    while not re.match(r"(?i)\s*end\s+type", lines[i]):
        d = re.match(r"(?i)\s*(integer|real|type)\s*\(([^)]*)\)\s*::\s*(.*)$", lines[i])
        cls = "ptr" if d.group(1).lower() == "type" else _FKIND[d.group(2).strip().lower()]
        for e in _split_top(d.group(3)):
            out.append((re.match(r"(\w+)", e).group(1).lower(), cls))
        i += 1
    return out


def test_fortran_struct_mirrors_match_the_header():
    """q35_model_config_t and q35_layer_weights_t (q35_model_api.f90) have the C structs'
    fields in order with the same classes; the ctypes mirrors they are compared with are
    checked against the header's offsets in test_capi_symbols."""
    import ctypes
    from asicfortranai_b200.llama_model import LayerWeights, ModelConfig
    path = os.path.join(FDIR, "q35_model_api.f90")

    def cls(t):
        if t is ctypes.c_void_p:
            return "ptr"
        if t is ctypes.c_float:
            return "f32"
        return "i64" if ctypes.sizeof(t) == 8 else "i32"

    for tname, py in (("q35_model_config_t", ModelConfig), ("q35_layer_weights_t", LayerWeights)):
        assert _bind_c_type(path, tname) == [(f, cls(t)) for f, t in py._fields_], tname
