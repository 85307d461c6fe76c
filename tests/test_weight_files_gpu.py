"""Weight-file readers of libq35 (weight_loader.f90's stream-binary layer file and the
3.5-bit safetensors checkpoint of convert_weights_3p5bit.py): a model loaded from files
gives logits bit-identical to the oracle over the same weights."""
import numpy as np
import pytest

from asicfortranai_b200 import weight_files as wf
from oracle import oracle as orc
from tests.model_util import TINY, layer_dict, make_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from asicfortranai_b200.quantized import Context
    c = Context(0)
    yield c
    c.close()


def same(a, b):
    np.testing.assert_array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def _model(ctx, cfg):
    from asicfortranai_b200.llama_model import LLaMAModel
    return LLaMAModel(ctx, cfg)


def test_stream_layer_files_int4(ctx, tmp_path):
    cfg = dict(TINY, wformat=1, n_layers=2)
    w = make_weights(cfg, seed=3)
    wf.write_layer_file(tmp_path / "weights_layer0.bin", layer_dict(w, 0), norms=True)
    wf.write_layer_file(tmp_path / "weights_layer1.bin", layer_dict(w, 1), norms=False)
    ref_w = dict(w)                               # layer 1 keeps the initial norms, 1.0
    ref_w["1.attn_norm"] = np.ones(cfg["hidden"], np.float32)
    ref_w["1.ffn_norm"] = np.ones(cfg["hidden"], np.float32)
    gm = _model(ctx, cfg)
    gm.load_layer_weights(0, tmp_path / "weights_layer0.bin")
    gm.load_layer_weights(1, str(tmp_path / "weights_layer1.bin"))
    gm.set_embeddings(w["embed"], w["final_norm"], w["lm_head"])
    ids = orc.gen_tokens(6, 3, 7, cfg["vocab"])
    same(gm.forward_llama(ids), orc.OracleModel(cfg, ref_w).forward(ids))
    gm.cleanup_llama_model()


def test_stream_layer_file_errors(ctx, tmp_path):
    from asicfortranai_b200 import Q35Error
    cfg = dict(TINY, wformat=1, n_layers=1)
    w = make_weights(cfg, seed=4)
    p = tmp_path / "l0.bin"
    wf.write_layer_file(p, layer_dict(w, 0))
    raw = p.read_bytes()
    (tmp_path / "short.bin").write_bytes(raw[:-4])
    gm = _model(ctx, cfg)
    with pytest.raises(Q35Error, match="bytes"):
        gm.load_layer_weights(0, tmp_path / "short.bin")
    with pytest.raises(Q35Error, match="cannot open"):
        gm.load_layer_weights(0, tmp_path / "missing.bin")
    with pytest.raises(Q35Error):
        gm.load_layer_weights(1, p)                                   # layer out of range
    gm.cleanup_llama_model()
    g35 = _model(ctx, dict(cfg, wformat=0))
    with pytest.raises(Q35Error, match="INT4"):
        g35.load_layer_weights(0, p)
    g35.cleanup_llama_model()


@pytest.mark.parametrize("float_dtype", [np.float32, np.float16])
def test_safetensors_checkpoint_3p5bit(ctx, tmp_path, float_dtype):
    cfg = dict(TINY, n_layers=2)
    w = make_weights(cfg, seed=5)
    t = wf.llama_3p5bit_tensors(cfg, w, float_dtype=float_dtype)
    keys = sorted(t)
    half = len(keys) // 2                          # two shard files
    wf.write_safetensors(tmp_path / "a.safetensors", {k: t[k] for k in keys[:half]})
    wf.write_safetensors(tmp_path / "b.safetensors", {k: t[k] for k in keys[half:]})
    ref_w = dict(w)
    for k in ("embed", "final_norm", "lm_head", "0.attn_norm", "0.ffn_norm", "1.attn_norm", "1.ffn_norm"):
        ref_w[k] = np.asfortranarray(np.asarray(w[k]).astype(float_dtype).astype(np.float32))
    gm = _model(ctx, cfg)
    gm.load_safetensors([tmp_path / "a.safetensors", tmp_path / "b.safetensors"])
    ids = orc.gen_tokens(9, 5, 8, cfg["vocab"])
    same(gm.forward_llama(ids), orc.OracleModel(cfg, ref_w).forward(ids))
    gm.cleanup_llama_model()


def test_safetensors_quantized_embeddings(ctx, tmp_path):
    """The reference converter quantizes every 2-D tensor: embeddings and LM head arrive as
    weight_q/scales/offsets and are expanded as code * scale + zero_point."""
    cfg = dict(TINY, n_layers=1)
    w = make_weights(cfg, seed=6)
    E = np.asfortranarray(w["embed"])                         # [vocab][hidden] = [K][N]
    H = np.asfortranarray(np.asarray(w["lm_head"]).T)         # [vocab][hidden]
    qe, qh = orc.quantize_3p5bit(E), orc.quantize_3p5bit(H)
    t = wf.llama_3p5bit_tensors(cfg, w, float_dtype=np.float32, quantized_embeddings={"embed": qe, "lm_head": qh})
    wf.write_safetensors(tmp_path / "m.safetensors", t)
    ref_w = dict(w)
    ref_w["embed"] = np.asfortranarray(wf.expand_3p5bit(*qe))
    ref_w["lm_head"] = np.asfortranarray(wf.expand_3p5bit(*qh).T)
    gm = _model(ctx, cfg)
    gm.load_safetensors(tmp_path / "m.safetensors")
    ids = orc.gen_tokens(5, 6, 9, cfg["vocab"])
    same(gm.forward_llama(ids), orc.OracleModel(cfg, ref_w).forward(ids))
    gm.cleanup_llama_model()


def test_safetensors_errors(ctx, tmp_path):
    from asicfortranai_b200 import Q35Error
    cfg = dict(TINY, n_layers=1)
    w = make_weights(cfg, seed=7)
    t = wf.llama_3p5bit_tensors(cfg, w)
    bad = dict(t)
    del bad["model.layers.0.mlp.up_proj.weight.offsets"]
    wf.write_safetensors(tmp_path / "missing.safetensors", bad)
    gm = _model(ctx, cfg)
    with pytest.raises(Q35Error, match="up_proj.weight.offsets"):
        gm.load_safetensors(tmp_path / "missing.safetensors")
    wrong = dict(t)
    wrong["model.layers.0.self_attn.q_proj.weight.weight_q"] = t["model.layers.0.self_attn.q_proj.weight.weight_q"][:-2]
    wf.write_safetensors(tmp_path / "shape.safetensors", wrong)
    with pytest.raises(Q35Error, match="shape"):
        gm.load_safetensors(tmp_path / "shape.safetensors")
    (tmp_path / "junk.safetensors").write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json}      ")
    with pytest.raises(Q35Error, match="header"):
        gm.load_safetensors(tmp_path / "junk.safetensors")
    gm.cleanup_llama_model()
