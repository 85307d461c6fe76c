"""Tiny LLaMA configurations and random weights for model parity tests: one weights
dict (Fortran-order numpy arrays, the reference's layouts) drives both the CPU oracle
and the GPU model."""
import numpy as np

from oracle import oracle as orc

TINY = dict(n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, vocab=1000,
            max_seq=96, rms_eps=1e-5, rope_theta=10000.0, rope_mode=0, wformat=0, max_batch=1)


def make_weights(cfg, seed=0, sigma=0.02, norm_mean=1.0):
    """Quantized layer matrices from N(0, sigma^2); norms around norm_mean (the
    reference initialises them to 1.0, llama_model.f90:74-75); embeddings and LM head
    N(0, sigma^2) scaled so that activations stay O(1)."""
    fmt = cfg.get("wformat", 0)
    hid, H, KVH, D, F, V = (cfg[k] for k in ("hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab"))
    QN, KN = H * D, KVH * D
    w = {}
    tid = 10
    for l in range(cfg["n_layers"]):
        for nm, (K, N) in zip(("q", "k", "v", "o", "g", "u", "d"),
                              ((hid, QN), (hid, KN), (hid, KN), (QN, hid), (hid, F), (hid, F), (F, hid))):
            W = orc.gen_normal((K, N), seed, tid, sigma)
            tid += 1
            if fmt == 0:
                wq, s, o = orc.quantize_3p5bit(W)
                w[f"{l}.o{nm}"] = o
            else:
                wq, s = orc.quantize_int4(W)
            w[f"{l}.w{nm}"] = wq
            w[f"{l}.s{nm}"] = s
        for nm in ("attn_norm", "ffn_norm"):
            w[f"{l}.{nm}"] = (norm_mean + orc.gen_normal((hid,), seed, tid, sigma)).astype(np.float32)
            tid += 1
    w["embed"] = orc.gen_normal((V, hid), seed, 1, 1.0)
    w["final_norm"] = (norm_mean + orc.gen_normal((hid,), seed, 2, sigma)).astype(np.float32)
    w["lm_head"] = orc.gen_normal((hid, V), seed, 3, 0.05)
    return w


def layer_dict(w, l):
    d = {}
    for nm in ("q", "k", "v", "o", "g", "u", "d"):
        d["w" + nm] = w[f"{l}.w{nm}"]
        d["s" + nm] = w[f"{l}.s{nm}"]
        if f"{l}.o{nm}" in w:
            d["o" + nm] = w[f"{l}.o{nm}"]
    d["attn_norm"] = w[f"{l}.attn_norm"]
    d["ffn_norm"] = w[f"{l}.ffn_norm"]
    return d


def gpu_model(ctx, cfg, w, tp=None):
    from asicfortranai_b200.llama_model import LLaMAModel
    m = LLaMAModel(ctx, cfg, tp)
    for l in range(cfg["n_layers"]):
        m.set_layer(l, layer_dict(w, l))
    m.set_embeddings(w["embed"], w["final_norm"], w["lm_head"])
    return m


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def random_init_weights(cfg, seed=0, sigma=0.02):
    """The weights q35_model_init_random(seed, sigma) builds on the device, made on the
    host with the oracle's copy of the same counter-based generator: per layer l the
    fused (hidden, q|k|v) matrix draws tensor 1000+16l, o 1000+16l+1, the fused
    (hidden, gate|up) matrix +2, down +3, the norms +4 and +5 (N(0, sigma^2), no unit
    mean); the embedding table tensor 1 ([vocab][hidden] row-major), the final norm 2,
    the LM head 3 ([vocab][hidden] row-major, i.e. the reference's (hidden, vocab)
    column-major).  Quantized per column with the model's format; column slices of a
    per-column quantization equal the quantization of the slices."""
    fmt = cfg.get("wformat", 0)
    hid, H, KVH, D, F, V = (cfg[k] for k in ("hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab"))
    QN, KN = H * D, KVH * D
    w = {}

    def quant(K, N, tid):
        W = orc.gen_normal((K, N), seed, tid, sigma)
        if fmt == 0:
            wq, s, o = orc.quantize_3p5bit(W)
        else:
            (wq, s), o = orc.quantize_int4(W), None
        return wq, s, o

    def put(l, nm, q, c0, c1):
        wq, s, o = q
        w[f"{l}.w{nm}"] = np.asfortranarray(wq[:, c0:c1])
        w[f"{l}.s{nm}"] = np.ascontiguousarray(s[c0:c1])
        if o is not None:
            w[f"{l}.o{nm}"] = np.ascontiguousarray(o[c0:c1])

    for l in range(cfg["n_layers"]):
        t0 = 1000 + 16 * l
        q = quant(hid, QN + 2 * KN, t0)
        put(l, "q", q, 0, QN)
        put(l, "k", q, QN, QN + KN)
        put(l, "v", q, QN + KN, QN + 2 * KN)
        put(l, "o", quant(QN, hid, t0 + 1), 0, hid)
        gu = quant(hid, 2 * F, t0 + 2)
        put(l, "g", gu, 0, F)
        put(l, "u", gu, F, 2 * F)
        put(l, "d", quant(F, hid, t0 + 3), 0, hid)
        del q, gu
        w[f"{l}.attn_norm"] = orc.gen_normal((hid,), seed, t0 + 4, sigma)
        w[f"{l}.ffn_norm"] = orc.gen_normal((hid,), seed, t0 + 5, sigma)
    w["embed"] = np.asfortranarray(orc.gen_normal((V * hid,), seed, 1, sigma).reshape(V, hid))
    w["final_norm"] = orc.gen_normal((hid,), seed, 2, sigma)
    w["lm_head"] = orc.gen_normal((V * hid,), seed, 3, sigma).reshape((hid, V), order="F")
    return w
