"""ctypes wrapper of the CPU oracle (q35_oracle.c).

TEST INFRASTRUCTURE ONLY: the tests, the smoke check and bench.py's CPU-baseline leg
use this module to produce expected results.  The product library never imports it.

Arrays follow the reference's Fortran layout; numpy arrays are passed in Fortran order
(``A`` of shape (M, K) with ``order='F'``, ``W_Q`` of shape (K//2, N), ...).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_i8p = np.ctypeslib.ndpointer(np.int8, flags="F_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="F_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="F_CONTIGUOUS")


def build(native: bool = False) -> str:
    """Compile the oracle (make -C oracle); returns the path of the shared library."""
    target = "native" if native else "all"
    subprocess.run(["make", "-s", "-C", _HERE, target], check=True)
    return os.path.join(_HERE, "liborc_native.so" if native else "liborc.so")


def lib(native: bool = False):
    global _LIB
    if _LIB is not None and not native:
        return _LIB
    path = os.path.join(_HERE, "liborc_native.so" if native else "liborc.so")
    src = os.path.join(_HERE, "q35_oracle.c")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        build(native)
    L = C.CDLL(path)
    L.orc_rng_u64.restype = C.c_uint64
    L.orc_rng_u64.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
    L.orc_gen_int8.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_uint64]
    L.orc_gen_normal.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_uint64, C.c_double]
    L.orc_gen_tokens.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_uint64, C.c_int32]
    L.orc_quantize_3p5bit_asym.argtypes = [_f32p, _i8p, _f32p, _f32p, C.c_int32, C.c_int32]
    L.orc_quantize_int4_sym.argtypes = [_f32p, _i8p, _f32p, C.c_int32, C.c_int32]
    L.orc_matmul_3p5bit_awq.argtypes = [_i8p, _i8p, _f32p, _f32p, _i32p, C.c_int32, C.c_int32,
                                        C.c_int32, C.c_int32]
    L.orc_dequantize_output_3p5bit.argtypes = [_i32p, _f32p, _f32p, _f32p, C.c_int32, C.c_int32]
    L.orc_matmul_int4_awq.argtypes = [_i8p, _i8p, _f32p, _i32p, C.c_int32, C.c_int32, C.c_int32]
    L.orc_dequantize_output.argtypes = [_i32p, _f32p, _f32p, C.c_int32, C.c_int32]
    L.orc_matmul_int4_simd.argtypes = [_i8p, _i8p, _f32p, _i32p, C.c_int32, C.c_int32, C.c_int32]
    L.orc_quantize_activations.argtypes = [_f32p, _i8p, C.c_int64]
    L.orc_q35_linear.argtypes = [_f32p, _i8p, _f32p, _f32p, _f32p, C.c_int32, C.c_int32,
                                 C.c_int32, C.c_int32]
    L.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, C.c_int32, C.c_int32, C.c_float]
    L.orc_rms_norm_tree.argtypes = [_f32p, _f32p, _f32p, C.c_int32, C.c_int32, C.c_float]
    L.orc_q35_expf.restype = C.c_float
    L.orc_q35_expf.argtypes = [C.c_float]
    L.orc_swish.restype = C.c_float
    L.orc_swish.argtypes = [C.c_float]
    L.orc_rope_freqs.argtypes = [_f32p, C.c_int32, C.c_int32, C.c_float]
    L.orc_sample_greedy.restype = C.c_int32
    L.orc_sample_greedy.argtypes = [_f32p, C.c_int32]
    L.orc_model_create.restype = C.c_void_p
    L.orc_model_create.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    L.orc_model_destroy.argtypes = [C.c_void_p]
    L.orc_model_reset.argtypes = [C.c_void_p]
    L.orc_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p]
    L.orc_layer_forward.argtypes = [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32]
    L.orc_generate_greedy.restype = C.c_int32
    L.orc_generate_greedy.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                      C.c_void_p, C.c_void_p]
    L.orc_sample.restype = C.c_int32
    L.orc_sample.argtypes = [_f32p, C.c_int32, C.c_int32, C.c_float, C.c_int32, C.c_float, C.c_float,
                             C.c_int32]
    L.orc_sample_uniform.restype = C.c_float
    L.orc_sample_uniform.argtypes = [C.c_uint64, C.c_int32, C.c_int32]
    L.orc_generate.restype = C.c_int32
    L.orc_generate.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                               C.c_int32, C.c_void_p, C.c_void_p]
    L.orc_set_threads.argtypes = [C.c_int32]
    L.orc_get_threads.restype = C.c_int32
    if not native:
        _LIB = L
    return L


def _F(a, dt):
    return np.asfortranarray(a, dtype=dt)


# ---- generator -------------------------------------------------------------------
def gen_int8(shape, seed, tensor_id, order="F"):
    n = int(np.prod(shape))
    out = np.empty(n, np.int8)
    lib().orc_gen_int8(out.ctypes.data, n, seed, tensor_id)
    return out.reshape(shape, order=order)


def gen_normal(shape, seed, tensor_id, sigma=0.02, order="F"):
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    lib().orc_gen_normal(out.ctypes.data, n, seed, tensor_id, sigma)
    return out.reshape(shape, order=order)


def gen_tokens(n, seed, tensor_id, vocab):
    out = np.empty(n, np.int32)
    lib().orc_gen_tokens(out.ctypes.data, n, seed, tensor_id, vocab)
    return out


# ---- quantizers ------------------------------------------------------------------
def quantize_3p5bit(W):
    """W float32 (K, N) -> (W_Q int8 (K/2, N), scales (N,), offsets (N,)), Fortran order."""
    W = _F(W, np.float32)
    K, N = W.shape
    assert K % 2 == 0
    wq = np.zeros((K // 2, N), np.int8, order="F")
    s = np.zeros(N, np.float32)
    o = np.zeros(N, np.float32)
    lib().orc_quantize_3p5bit_asym(W, wq, s, o, K, N)
    return wq, s, o


def quantize_int4(W):
    W = _F(W, np.float32)
    K, N = W.shape
    assert K % 2 == 0
    wq = np.zeros((K // 2, N), np.int8, order="F")
    s = np.zeros(N, np.float32)
    lib().orc_quantize_int4_sym(W, wq, s, K, N)
    return wq, s


# ---- kernels ---------------------------------------------------------------------
def matmul_3p5bit_awq(A, W_Q, scales, offsets, mode=0):
    A = _F(A, np.int8)
    W_Q = _F(W_Q, np.int8)
    M, K = A.shape
    N = W_Q.shape[1]
    C_ = np.zeros((M, N), np.int32, order="F")
    lib().orc_matmul_3p5bit_awq(A, W_Q, _F(scales, np.float32), _F(offsets, np.float32), C_,
                                M, N, K, mode)
    return C_


def dequantize_output_3p5bit(C_, scales, offsets):
    C_ = _F(C_, np.int32)
    M, N = C_.shape
    out = np.zeros((M, N), np.float32, order="F")
    lib().orc_dequantize_output_3p5bit(C_, _F(scales, np.float32), _F(offsets, np.float32), out,
                                       M, N)
    return out


def matmul_int4_awq(A, W_Q, scales):
    A = _F(A, np.int8)
    W_Q = _F(W_Q, np.int8)
    M, K = A.shape
    N = W_Q.shape[1]
    C_ = np.zeros((M, N), np.int32, order="F")
    lib().orc_matmul_int4_awq(A, W_Q, _F(scales, np.float32), C_, M, N, K)
    return C_


def matmul_int4_simd(A, W_Q, scales):
    """matmul_simd_optimized.f90:24-112 (same sums as matmul_int4_awq, the reference's
    SIMD/OpenMP loop form; a timed CPU stand-in)."""
    A = _F(A, np.int8)
    W_Q = _F(W_Q, np.int8)
    M, K = A.shape
    N = W_Q.shape[1]
    C_ = np.zeros((M, N), np.int32, order="F")
    lib().orc_matmul_int4_simd(A, W_Q, _F(scales, np.float32), C_, M, N, K)
    return C_


def dequantize_output(C_, scales):
    C_ = _F(C_, np.int32)
    M, N = C_.shape
    out = np.zeros((M, N), np.float32, order="F")
    lib().orc_dequantize_output(C_, _F(scales, np.float32), out, M, N)
    return out


def quantize_activations(x):
    x = _F(x, np.float32)
    out = np.zeros(x.shape, np.int8, order="F")
    lib().orc_quantize_activations(x, out, x.size)
    return out


def rms_norm(x, w, eps=1e-5):
    x = _F(x, np.float32)
    S, dim = x.shape
    out = np.zeros_like(x, order="F")
    lib().orc_rms_norm(x, _F(w, np.float32), out, S, dim, eps)
    return out


def rope_freqs(max_seq, head_dim, theta=10000.0):
    f = np.zeros((max_seq, head_dim // 2), np.float32, order="F")
    lib().orc_rope_freqs(f, max_seq, head_dim, theta)
    return f


def sample_greedy(logits):
    return int(lib().orc_sample_greedy(_F(logits, np.float32), len(logits)))


SAMPLE_GREEDY, SAMPLE_TEMPERATURE, SAMPLE_TOP_K, SAMPLE_TOP_P = 0, 1, 2, 3


def sample(logits, mode, u, temperature=0.0, top_k=0, top_p=0.0, order=1):
    """sampling.f90:88-259 with the uniform draw u; order 0 = the source's sequential sums
    with expf, 1 = the device sampler's blocked order with q35_expf.  1-based token."""
    lg = _F(logits, np.float32)
    return int(lib().orc_sample(lg, len(lg), int(mode), float(temperature), int(top_k), float(top_p),
                                float(u), int(order)))


def sample_uniform(seed, seq, n):
    return float(lib().orc_sample_uniform(int(seed), int(seq), int(n)))


class OrcSampling(C.Structure):
    _fields_ = [("mode", C.c_int32), ("temperature", C.c_float), ("top_k", C.c_int32),
                ("top_p", C.c_float), ("seed", C.c_uint64)]


def set_threads(n):
    lib().orc_set_threads(int(n))


# ---- model -----------------------------------------------------------------------
class OrcConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("max_seq", C.c_int32), ("rms_eps", C.c_float),
                ("rope_theta", C.c_float), ("rope_mode", C.c_int32), ("wformat", C.c_int32),
                ("order", C.c_int32)]


_LW_NAMES = (["wq", "wk", "wv", "wo", "wg", "wu", "wd"] + ["sq", "sk", "sv", "so", "sg", "su", "sd"]
             + ["oq", "ok", "ov", "oo", "og", "ou", "od"] + ["attn_norm", "ffn_norm"])


class OrcLayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _LW_NAMES]


class OracleModel:
    """forward_llama / generation restated on the CPU over a weights dict.

    ``weights`` is the dict made by tests' model builder: per layer l, keys
    ``f"{l}.{name}"`` for packed matrices (K/2,N) int8, scales/offsets (N,) float32 and
    norms (hidden,) float32, plus ``embed`` (vocab, hidden), ``final_norm``, ``lm_head``
    (hidden, vocab), all Fortran order.
    """

    def __init__(self, cfg: dict, weights: dict):
        self.cfg = cfg
        self._keep = []
        c = OrcConfig(cfg["n_layers"], cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"],
                      cfg["head_dim"], cfg["ffn"], cfg["vocab"], cfg["max_seq"],
                      cfg.get("rms_eps", 1e-5), cfg.get("rope_theta", 10000.0),
                      cfg.get("rope_mode", 0), cfg.get("wformat", 0), cfg.get("order", 1))
        layers = (OrcLayerWeights * cfg["n_layers"])()
        for l in range(cfg["n_layers"]):
            for nm in _LW_NAMES:
                key = f"{l}.{nm}"
                if key in weights:
                    arr = weights[key]
                    assert arr.flags.f_contiguous
                    self._keep.append(arr)
                    setattr(layers[l], nm, arr.ctypes.data)
        for k in ("embed", "final_norm", "lm_head"):
            assert weights[k].flags.f_contiguous
            self._keep.append(weights[k])
        self._cfg = c
        self._layers = layers
        self.h = lib().orc_model_create(C.byref(c), layers, weights["embed"].ctypes.data,
                                        weights["final_norm"].ctypes.data,
                                        weights["lm_head"].ctypes.data)

    def reset(self):
        lib().orc_model_reset(self.h)

    def forward(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        S = len(ids)
        out = np.zeros((S, self.cfg["vocab"]), np.float32, order="F")
        lib().orc_forward(self.h, ids.ctypes.data, S, out.ctypes.data)
        return out

    def layer_forward(self, layer, x):
        x = _F(x, np.float32)
        out = np.zeros_like(x, order="F")
        lib().orc_layer_forward(self.h, layer, x.ctypes.data, out.ctypes.data, x.shape[0])
        return out

    def generate(self, prompt, n_steps, stop_at_eos=False, want_logits=False, sampling=None, seq=0):
        """sampling: None (greedy) or dict(mode, temperature, top_k, top_p, seed); the draws
        are those of sequence ``seq`` of a model run."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(n_steps, np.int32)
        lg = np.zeros((self.cfg["vocab"], n_steps), np.float32, order="F") if want_logits else None
        smp = None
        if sampling is not None:
            smp = OrcSampling(int(sampling.get("mode", 0)), float(sampling.get("temperature", 0.0)),
                              int(sampling.get("top_k", 0)), float(sampling.get("top_p", 0.0)),
                              int(sampling.get("seed", 0)))
        n = lib().orc_generate(self.h, prompt.ctypes.data, len(prompt), n_steps, int(stop_at_eos),
                               C.byref(smp) if smp is not None else None, int(seq), toks.ctypes.data,
                               lg.ctypes.data if want_logits else None)
        return (toks[:n], lg) if want_logits else toks[:n]

    def __del__(self):
        try:
            lib().orc_model_destroy(self.h)
        except Exception:
            pass
