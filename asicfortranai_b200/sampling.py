"""Host mirror of the reference module ``sampling`` (sampling.f90) over libq35.so: every
draw runs on the GPU in one fused kernel (q35_sample.cu).

    tok = sample_greedy(logits, vocab_size)               # sampling.f90:64-83
    tok = sample_temperature(logits, vocab_size, 0.8)     # :88-118
    tok = sample_top_k(logits, vocab_size, 40)            # :123-176
    tok = sample_top_p(logits, vocab_size, 0.95)          # :181-259
    toks = sample_rows(ctx, "top_p", logits_dev, u_dev, top_p=0.95)   # device rows

Tokens are 1-based, as in the reference.  ``random_number`` is replaced by the uniform
draw ``u`` in [0, 1): pass it for a reproducible draw, or leave it None to take one from
``rng`` (a numpy Generator; numpy's default generator when None).  Vocabularies up to
32,768.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib

MODES = {"greedy": 0, "temperature": 1, "top_k": 2, "top_p": 3}


def _row(logits, vocab_size):
    lg = np.ascontiguousarray(np.asarray(logits, np.float32).reshape(-1))
    n = len(lg) if vocab_size is None else int(vocab_size)
    if n > len(lg):
        raise ValueError("vocab_size exceeds the logits")
    return lg, n


def _u(u, rng):
    if u is not None:
        return float(u)
    g = rng if rng is not None else np.random.default_rng()
    return float(g.integers(0, 1 << 24)) * 2.0 ** -24       # exactly representable, < 1


def _draw(fn, lg, n, *args, ctx=None):
    """ctx: a quantized.Context, or None for the library's context of the current device."""
    tok = C.c_int32()
    _lib.check(fn(ctx.h if ctx is not None else None, lg.ctypes.data, n, *args, C.byref(tok)), fn.__name__)
    return tok.value


def sample_greedy(logits, vocab_size=None, ctx=None) -> int:
    lg, n = _row(logits, vocab_size)
    return _draw(_lib.load().q35_sample_greedy, lg, n, ctx=ctx)


def sample_temperature(logits, vocab_size=None, temperature: float = 1.0, u=None, rng=None, ctx=None) -> int:
    lg, n = _row(logits, vocab_size)
    return _draw(_lib.load().q35_sample_temperature, lg, n, float(temperature), _u(u, rng), ctx=ctx)


def sample_top_k(logits, vocab_size=None, k: int = 40, u=None, rng=None, ctx=None) -> int:
    lg, n = _row(logits, vocab_size)
    return _draw(_lib.load().q35_sample_top_k, lg, n, int(k), _u(u, rng), ctx=ctx)


def sample_top_p(logits, vocab_size=None, p: float = 0.95, u=None, rng=None, ctx=None) -> int:
    lg, n = _row(logits, vocab_size)
    return _draw(_lib.load().q35_sample_top_p, lg, n, float(p), _u(u, rng), ctx=ctx)


def sample_rows(ctx, mode, logits_ptr: int, rows: int, vocab: int, u_ptr: int, tokens_ptr: int,
                temperature: float = 0.0, top_k: int = 0, top_p: float = 0.0) -> None:
    """Device rows: logits[rows][vocab] fp32, u[rows] fp32, tokens[rows] int32 (device
    pointers, e.g. torch tensors' data_ptr()); enqueued on ctx's stream."""
    m = MODES[mode] if isinstance(mode, str) else int(mode)
    _lib.check(_lib.load().q35_sample_dev(ctx.h, m, logits_ptr, rows, vocab, temperature, top_k, top_p,
                                          u_ptr, tokens_ptr), "q35_sample_dev")
