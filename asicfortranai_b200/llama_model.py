"""Host mirror of the reference modules ``llama_model`` (llama_model.f90),
``transformer_layer`` (transformer_layer.f90) and the generation loop of
``llama_generate.f90`` over libq35.so.  All compute runs on the GPU.

    model = LLaMAModel(ctx, config)          # init_llama_model
    model.set_layer(l, weights)              # TransformerLayer fields, reference layouts
    model.set_embeddings(E, final_norm, W)   # token_embeddings / final_norm / output_weights
    logits = model.forward_llama(ids, S)     # (S, vocab), Fortran order
    out = model.apply_transformer_layer(l, x, S)
    model.set_sampling("top_p", top_p=0.95, seed=1)   # llama_generate.f90:94-98 (default greedy)
    toks = model.generate(prompts, n_steps)  # all sequences of the batch
    model.cleanup_llama_model()
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("max_seq", C.c_int32), ("rms_eps", C.c_float),
                ("rope_theta", C.c_float), ("rope_mode", C.c_int32), ("wformat", C.c_int32),
                ("max_batch", C.c_int32)]


_LW = ["wq", "wk", "wv", "wo", "wg", "wu", "wd", "sq", "sk", "sv", "so", "sg", "su", "sd",
       "oq", "ok", "ov", "oo", "og", "ou", "od", "attn_norm", "ffn_norm"]


class LayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _LW]


# LLaMA-70B constants of transformer_layer.f90:21-27 and llama_model.f90:14-16
LLAMA70B = dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672,
                vocab=32000, max_seq=2048, rms_eps=1e-5, rope_theta=10000.0)
LLAMA13B = dict(n_layers=40, hidden=5120, n_heads=40, n_kv_heads=40, head_dim=128, ffn=13824,
                vocab=32000, max_seq=2048, rms_eps=1e-5, rope_theta=10000.0)


def make_config(d: dict) -> ModelConfig:
    return ModelConfig(d["n_layers"], d["hidden"], d["n_heads"], d["n_kv_heads"], d["head_dim"],
                       d["ffn"], d["vocab"], d["max_seq"], d.get("rms_eps", 1e-5),
                       d.get("rope_theta", 10000.0), d.get("rope_mode", 0), d.get("wformat", 0),
                       d.get("max_batch", 1))


class Sampling(C.Structure):
    _fields_ = [("mode", C.c_int32), ("temperature", C.c_float), ("top_k", C.c_int32),
                ("top_p", C.c_float), ("seed", C.c_uint64)]


SAMPLE_MODES = {"greedy": 0, "temperature": 1, "top_k": 2, "top_p": 3}


class LLaMAModel:
    def __init__(self, ctx, cfg: dict, tp=None):
        """tp: an asicfortranai_b200.tp.TPGroup to shard the model over (None: one GPU)."""
        L = _lib.load()
        self.ctx, self.cfg, self.tp = ctx, dict(cfg), tp
        self._c = make_config(cfg)
        h = C.c_void_p()
        _lib.check(L.q35_model_create_tp(ctx.h, C.byref(self._c), tp.h if tp is not None else None, C.byref(h)),
                   "init_llama_model")
        self.h = h
        ctx.adopt(self)

    # -- loading -------------------------------------------------------------------
    def set_layer(self, layer: int, w: dict):
        """w: wq..wd (K/2,N) int8, sq..sd scales, oq..od offsets (3.5-bit), attn_norm,
        ffn_norm -- Fortran-order numpy arrays as in TransformerLayer."""
        keep = []
        lw = LayerWeights()
        for n in _LW:
            if n in w and w[n] is not None:
                a = np.asfortranarray(w[n])
                keep.append(a)
                setattr(lw, n, a.ctypes.data)
        _lib.check(_lib.load().q35_model_set_layer(self.h, layer, C.byref(lw)), f"set_layer({layer})")

    def load_layer_weights(self, layer: int, filename: str):
        """weight_loader.f90 load_layer_weights: one layer from the stream-binary INT4 file
        (INT4 model); the two norms are taken when the file carries them."""
        _lib.check(_lib.load().q35_model_load_layer_file(self.h, layer, str(filename).encode()),
                   f"load_layer_weights({layer})")

    def load_safetensors(self, paths):
        """The 3.5-bit safetensors checkpoint (convert_weights_3p5bit.py format), one path
        or a list of shard paths (3.5-bit model)."""
        if isinstance(paths, (str, bytes)) or hasattr(paths, "__fspath__"):
            paths = [paths]
        enc = [str(p).encode() for p in paths]
        arr = (C.c_char_p * len(enc))(*enc)
        _lib.check(_lib.load().q35_model_load_safetensors(self.h, arr, len(enc)), "load_safetensors")

    def set_embeddings(self, embed, final_norm, lm_head):
        e = np.asfortranarray(embed, np.float32)
        f = np.ascontiguousarray(final_norm, np.float32)
        w = np.asfortranarray(lm_head, np.float32)
        _lib.check(_lib.load().q35_model_set_embeddings(self.h, e.ctypes.data, f.ctypes.data, w.ctypes.data),
                   "set_embeddings")

    def init_random(self, seed: int = 0, sigma: float = 0.02):
        _lib.check(_lib.load().q35_model_init_random(self.h, seed, sigma), "init_random")

    # -- the reference procedures ------------------------------------------------------
    def reset_kv_cache(self):
        _lib.check(_lib.load().q35_model_reset(self.h), "reset_kv_cache")

    def forward_llama(self, token_ids, seq_len: int | None = None, seq: int = 0):
        ids = np.ascontiguousarray(token_ids, np.int32)
        S = len(ids) if seq_len is None else seq_len
        out = np.zeros((S, self.cfg["vocab"]), np.float32, order="F")
        _lib.check(_lib.load().q35_model_forward(self.h, seq, ids.ctypes.data, S, out.ctypes.data),
                   "forward_llama")
        return out

    def forward_next_token(self, token_ids, seq: int = 0) -> int:
        ids = np.ascontiguousarray(token_ids, np.int32)
        _lib.check(_lib.load().q35_model_forward(self.h, seq, ids.ctypes.data, len(ids), None), "forward")
        return int(self.last_tokens()[seq])

    def apply_transformer_layer(self, layer: int, x, seq_len: int | None = None, seq: int = 0,
                                advance: bool = True):
        x = np.asfortranarray(x, np.float32)
        S = x.shape[0] if seq_len is None else seq_len
        out = np.zeros_like(x, order="F")
        _lib.check(_lib.load().q35_model_layer_forward(self.h, layer, seq, x.ctypes.data, S,
                                                       out.ctypes.data, int(advance)),
                   "apply_transformer_layer")
        return out

    def last_tokens(self):
        t = np.zeros(self.cfg.get("max_batch", 1), np.int32)
        _lib.check(_lib.load().q35_model_last_tokens(self.h, t.ctypes.data), "last_tokens")
        return t

    def decode_step(self, ids=None, want_logits=False):
        B = self.cfg.get("max_batch", 1)
        nxt = np.zeros(B, np.int32)
        lg = np.zeros((B, self.cfg["vocab"]), np.float32, order="F") if want_logits else None
        i = np.ascontiguousarray(ids, np.int32) if ids is not None else None
        _lib.check(_lib.load().q35_model_decode_step(self.h, i.ctypes.data if i is not None else None,
                                                     nxt.ctypes.data, lg.ctypes.data if want_logits else None),
                   "decode_step")
        return (nxt, lg) if want_logits else nxt

    def generate(self, prompts, n_steps: int, stop_at_eos: bool = False):
        """prompts: [max_batch][prompt_len] 1-based ids.  Returns a list of token arrays."""
        p = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        B, P = p.shape
        assert B == self.cfg.get("max_batch", 1)
        out = np.zeros((B, n_steps), np.int32)
        n = np.zeros(B, np.int32)
        _lib.check(_lib.load().q35_model_generate(self.h, p.ctypes.data, P, n_steps, int(stop_at_eos),
                                                  out.ctypes.data, n.ctypes.data), "generate")
        return [out[b, :n[b]] for b in range(B)]

    def set_sampling(self, mode="greedy", temperature: float = 0.0, top_k: int = 0, top_p: float = 0.0,
                     seed: int = 0):
        """Next-token rule of forward/decode/generate: "greedy" (default), "temperature",
        "top_k" or "top_p" (sampling.f90), drawn on the GPU.  Sequence b's n-th draw comes
        from the counter-based generator (seed, b, n); reset_kv_cache and this call restart
        the draws.  Under tensor parallelism every rank calls it with the same arguments."""
        m = SAMPLE_MODES[mode] if isinstance(mode, str) else int(mode)
        smp = Sampling(m, temperature, top_k, top_p, seed)
        _lib.check(_lib.load().q35_model_set_sampling(self.h, C.byref(smp)), "set_sampling")

    def debug_buffer(self, name: str, shape, dtype=np.float32):
        """Copy of an internal buffer (row-major): x, yqkv, q, ygu, xi8, kc, vc."""
        out = np.zeros(shape, dtype)
        _lib.check(_lib.load().q35_model_debug_buffer(self.h, name.encode(), out.ctypes.data, out.nbytes),
                   "debug_buffer")
        return out

    @property
    def weight_bytes(self) -> int:
        return int(_lib.load().q35_model_weight_bytes(self.h))

    def cleanup_llama_model(self):
        if self.h:
            _lib.load().q35_model_destroy(self.h)
            self.h = None

    close = cleanup_llama_model

    def __del__(self):
        try:
            self.cleanup_llama_model()
        except Exception:
            pass
