"""Writers of the reference's weight-file formats (host side, no GPU)."""
import json

import numpy as np

from asicfortranai_b200 import weight_files as wf
from oracle import oracle as orc
from tests.model_util import TINY, layer_dict, make_weights


def test_safetensors_layout(tmp_path):
    t = {"a": np.arange(6, dtype=np.float32).reshape(2, 3), "b": np.array([-1, 2, 3], np.int8),
         "c": np.array([1.5, -2.0], np.float16)}
    p = tmp_path / "x.safetensors"
    wf.write_safetensors(p, t, metadata={"format": "pt"})
    raw = p.read_bytes()
    n = int.from_bytes(raw[:8], "little")
    assert n % 8 == 0
    h = json.loads(raw[8:8 + n])
    assert h["a"] == {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}
    assert h["b"] == {"dtype": "I8", "shape": [3], "data_offsets": [24, 27]}
    assert h["c"] == {"dtype": "F16", "shape": [2], "data_offsets": [27, 31]}
    data = raw[8 + n:]
    np.testing.assert_array_equal(np.frombuffer(data[0:24], "<f4").reshape(2, 3), t["a"])
    np.testing.assert_array_equal(np.frombuffer(data[24:27], np.int8), t["b"])
    np.testing.assert_array_equal(np.frombuffer(data[27:31], "<f2"), t["c"])
    assert wf.read_safetensors_header(p)["__metadata__"] == {"format": "pt"}


def test_layer_file_layout(tmp_path):
    cfg = dict(TINY, wformat=1)
    w = make_weights(cfg, seed=1)
    ld = layer_dict(w, 0)
    p = tmp_path / "layer0.bin"
    n = wf.write_layer_file(p, ld, norms=True)
    hid, QN, KN, F = cfg["hidden"], cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"], cfg["ffn"]
    need = sum(K // 2 * N + 4 * N for K, N in ((hid, QN), (hid, KN), (hid, KN), (QN, hid), (hid, F), (hid, F), (F, hid)))
    assert n == need + 8 * hid == p.stat().st_size
    raw = p.read_bytes()
    # wq column-major (K/2, N), then its scales (weight_loader.f90:78-84)
    wq = np.frombuffer(raw[:hid // 2 * QN], np.int8).reshape((hid // 2, QN), order="F")
    np.testing.assert_array_equal(wq, ld["wq"])
    sq = np.frombuffer(raw[hid // 2 * QN: hid // 2 * QN + 4 * QN], "<f4")
    np.testing.assert_array_equal(sq, ld["sq"])
    np.testing.assert_array_equal(np.frombuffer(raw[-4 * hid:], "<f4"), ld["ffn_norm"])


def test_checkpoint_keys_and_shapes():
    cfg = dict(TINY, n_layers=2)
    w = make_weights(cfg, seed=2)
    t = wf.llama_3p5bit_tensors(cfg, w)
    hid, V = cfg["hidden"], cfg["vocab"]
    assert t["model.layers.1.mlp.down_proj.weight.weight_q"].shape == (cfg["ffn"] // 2, hid)
    assert t["model.layers.0.self_attn.k_proj.weight.scales"].shape == (cfg["n_kv_heads"] * cfg["head_dim"],)
    assert t["model.embed_tokens.weight"].shape == (V, hid) and t["model.embed_tokens.weight"].dtype == np.float16
    np.testing.assert_array_equal(t["lm_head.weight"], w["lm_head"].T.astype(np.float16))
    # [K/2][N] row-major holds the reference's W_Q(K/2,N) element (p, j) at p*N + j
    wq = t["model.layers.0.self_attn.q_proj.weight.weight_q"]
    assert wq.flags.c_contiguous
    np.testing.assert_array_equal(wq, w["0.wq"])


def test_expand_inverts_the_quantizer_where_codes_fit():
    W = orc.gen_normal((64, 40), 3, 9, 0.02)
    wq, s, o = orc.quantize_3p5bit(W)
    x = wf.expand_3p5bit(np.ascontiguousarray(wq), s, o)
    # code = round((w - zp)/scale) in [-8,7]; odd rows keep 3 bits (codes outside [-4,3] wrap)
    q = np.clip(np.round((W - o[None, :]) / s[None, :]), -8, 7)
    fits = np.ones_like(W, bool)
    fits[1::2] = (q[1::2] >= -4) & (q[1::2] <= 3)
    assert fits.mean() > 0.5
    np.testing.assert_allclose(x[fits], (q * s[None, :] + o[None, :]).astype(np.float32)[fits], rtol=0, atol=1e-6)
    assert np.all(np.abs(x - W)[fits] <= s[None, :].repeat(64, 0)[fits] * 0.5001 + 1e-7)
