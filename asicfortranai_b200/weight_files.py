"""Writers of the reference's weight-file formats (host tooling, numpy only); the readers
live in libq35 (``LLaMAModel.load_layer_weights`` / ``LLaMAModel.load_safetensors``).

* ``write_layer_file``: the stream-binary layer file of weight_loader.f90 /
  generate_test_weights.f90:154-183 -- wq, wk, wv, wo, w_gate, w_up, w_down, each W_Q(K/2,N)
  INT4 bytes column-major then scales[N] fp32, optionally attn_norm and ffn_norm
  (scripts/convert_weights_to_fortran.py:94-121).
* ``write_safetensors``: a safetensors file (8-byte little-endian header length, JSON
  header of dtype / shape / data_offsets, then the raw little-endian data).
* ``llama_3p5bit_tensors``: the tensors of a 3.5-bit LLaMA checkpoint in the layout of
  convert_weights_3p5bit.py:105-139 (``key.weight_q`` int8 [K/2][N], ``key.scales``,
  ``key.offsets``; norms and embeddings in floating point, or embeddings quantized too).
"""
from __future__ import annotations

import json

import numpy as np

_PROJ = [("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"), ("v", "self_attn.v_proj"),
         ("o", "self_attn.o_proj"), ("g", "mlp.gate_proj"), ("u", "mlp.up_proj"), ("d", "mlp.down_proj")]

_DTYPES = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int8): "I8",
           np.dtype(np.uint8): "U8", np.dtype(np.int32): "I32", np.dtype(np.int64): "I64",
           np.dtype(np.float64): "F64", np.dtype(np.int16): "I16"}


def write_layer_file(path, layer: dict, norms: bool = False) -> int:
    """layer: ``w{q,k,v,o,g,u,d}`` W_Q(K/2,N) int8 and ``s{...}`` scales (N,) float32 in the
    reference layout (INT4), plus ``attn_norm`` / ``ffn_norm`` when norms.  Returns bytes."""
    n = 0
    with open(path, "wb") as f:
        for nm, _ in _PROJ:
            w = np.asfortranarray(layer["w" + nm], np.int8)
            s = np.ascontiguousarray(layer["s" + nm], np.float32)
            f.write(w.tobytes(order="F"))
            f.write(s.astype("<f4").tobytes())
            n += w.nbytes + s.nbytes
        if norms:
            for k in ("attn_norm", "ffn_norm"):
                v = np.ascontiguousarray(layer[k], np.float32)
                f.write(v.astype("<f4").tobytes())
                n += v.nbytes
    return n


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Write tensors (name -> numpy array, C order) as one safetensors file."""
    header = {}
    off = 0
    blobs = []
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        if a.dtype not in _DTYPES:
            raise ValueError(f"{name}: unsupported dtype {a.dtype}")
        b = a.astype(a.dtype.newbyteorder("<")).tobytes()
        header[name] = {"dtype": _DTYPES[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_safetensors_header(path) -> dict:
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        return json.loads(f.read(n))


def llama_3p5bit_tensors(cfg: dict, w: dict, float_dtype=np.float16, quantized_embeddings=None) -> dict:
    """Checkpoint tensors from a weights dict in the reference layouts (keys ``{l}.w{q..d}``
    W_Q(K/2,N), ``{l}.s..``/``{l}.o..``, ``{l}.attn_norm``/``{l}.ffn_norm``, ``embed``
    (vocab,hidden), ``final_norm``, ``lm_head`` (hidden,vocab)).  quantized_embeddings: None,
    or a dict with ``embed`` / ``lm_head`` each a (weight_q [vocab/2][hidden], scales,
    offsets) triple written in place of the floating-point tensor."""
    t = {}
    for l in range(cfg["n_layers"]):
        pre = f"model.layers.{l}."
        for nm, key in _PROJ:
            base = pre + key + ".weight"
            t[base + ".weight_q"] = np.ascontiguousarray(w[f"{l}.w{nm}"], np.int8)   # [K/2][N]
            t[base + ".scales"] = np.ascontiguousarray(w[f"{l}.s{nm}"], np.float32)
            t[base + ".offsets"] = np.ascontiguousarray(w[f"{l}.o{nm}"], np.float32)
        t[pre + "input_layernorm.weight"] = np.asarray(w[f"{l}.attn_norm"]).astype(float_dtype)
        t[pre + "post_attention_layernorm.weight"] = np.asarray(w[f"{l}.ffn_norm"]).astype(float_dtype)
    q = quantized_embeddings or {}
    for name, key, arr in (("embed", "model.embed_tokens.weight", np.asarray(w["embed"])),
                           ("lm_head", "lm_head.weight", np.asarray(w["lm_head"]).T)):
        if name in q:
            wq, s, o = q[name]
            t[key + ".weight_q"] = np.ascontiguousarray(wq, np.int8)
            t[key + ".scales"] = np.ascontiguousarray(s, np.float32)
            t[key + ".offsets"] = np.ascontiguousarray(o, np.float32)
        else:
            t[key] = np.ascontiguousarray(arr).astype(float_dtype)                  # [vocab][hidden]
    t["model.norm.weight"] = np.asarray(w["final_norm"]).astype(float_dtype)
    return t


def expand_3p5bit(wq, scales, offsets) -> np.ndarray:
    """[K/2][N] pair bytes -> [K][N] floats as code * scale + zero_point (the quantizer's
    inverse, convert_weights_3p5bit.py:59-60), code the 4-bit field for even k and the
    3-bit field for odd k, in float32 arithmetic."""
    raw = np.asarray(wq).astype(np.int32) & 0x7F
    n1 = raw >> 3
    n1 = np.where(n1 >= 8, n1 - 16, n1)
    n2 = raw & 7
    n2 = np.where(n2 >= 4, n2 - 8, n2)
    K2, N = raw.shape
    out = np.empty((2 * K2, N), np.float32)
    s = np.asarray(scales, np.float32)[None, :]
    o = np.asarray(offsets, np.float32)[None, :]
    out[0::2] = (n1.astype(np.float32) * s) + o
    out[1::2] = (n2.astype(np.float32) * s) + o
    return out
