"""The decode path at the benchmarked model widths, against the CPU oracle.

The LLaMA-70B shape (hidden 8192, 64 query / 8 KV heads, FFN 28672) and the LLaMA-13B
shape (hidden 5120, 40 / 40 heads, FFN 13824), both with vocabulary 32000 and RoPE in the
reference's position-in-call mode, with two layers instead of 80 / 40 (every layer runs
the same kernels; the widths, head counts and the 32000-row LM head are what change the
launch shapes).  The weights are the ones q35_model_init_random builds for the benchmark
(N(0, 0.02^2), 3.5-bit), reproduced on the host by the oracle's copy of the generator, so
this checks the benchmarked model itself (llama_model.f90:105-147, transformer_layer.f90
:527-565, the generation loop of llama_generate.f90:76-123):

  * prefill logits of a 16-token prompt and 64 greedy decode steps: every step's logits
    and token bit-identical to the oracle in the kernels' reduction order;
  * batched decode (70B: 16 sequences, 13B: 8, the benchmark's batch sizes) on the
    tensor-core matmuls and the several-row attention, per sequence against the oracle;
  * the oracle in the source's own order (sequential fp32 sums, libm expf) against the
    GPU: logit error and greedy-token agreement over the 64 steps, and beside it the same
    source loops as an 8-lane vectorising build runs them against the sequential order,
    reported (written to $Q35_REPORT_DIR/model_widths_source_order.json when that is set)."""
import functools
import json
import os

import numpy as np
import pytest

from oracle import oracle as orc
from tests.model_util import random_init_weights, rel_err

pytestmark = pytest.mark.gpu

SHAPES = {
    "llama70b": dict(n_layers=2, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=32000),
    "llama13b": dict(n_layers=2, hidden=5120, n_heads=40, n_kv_heads=40, head_dim=128, ffn=13824, vocab=32000),
}
BATCH = {"llama70b": (16, 3, 3), "llama13b": (8, 4, 4)}   # sequences, prompt, tokens
PROMPT, STEPS = 16, 64
_results = {}


def cfg_of(name, max_batch=1, order=1):
    return dict(SHAPES[name], max_seq=96, rms_eps=1e-5, rope_theta=10000.0, rope_mode=0, wformat=0,
                max_batch=max_batch, order=order)


@functools.lru_cache(maxsize=2)
def host_weights(name):
    return random_init_weights(cfg_of(name), seed=0, sigma=0.02)


@pytest.fixture(scope="module")
def ctx():
    from asicfortranai_b200.quantized import Context
    c = Context(0)
    yield c
    c.close()


def same(a, b, what):
    np.testing.assert_array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32), err_msg=what)


@pytest.mark.parametrize("name", list(SHAPES))
def test_prefill_and_64_greedy_steps_bit_exact(ctx, name):
    from asicfortranai_b200.llama_model import LLaMAModel
    cfg = cfg_of(name)
    w = host_weights(name)
    prompt = orc.gen_tokens(PROMPT, 11, 1, cfg["vocab"])
    om = orc.OracleModel(cfg, w)
    ref_prefill = om.forward(prompt)
    om.reset()
    ref_tokens, ref_logits = om.generate(prompt, STEPS + 1, want_logits=True)
    gm = LLaMAModel(ctx, cfg)
    gm.init_random(0, 0.02)
    lg = gm.forward_llama(prompt)
    same(lg, ref_prefill, "prefill logits")
    toks = [int(gm.last_tokens()[0])]
    assert toks[0] == ref_tokens[0]
    for t in range(1, STEPS + 1):
        nxt, lgt = gm.decode_step(want_logits=True)
        same(lgt[0], ref_logits[:, t], f"decode step {t} logits")
        assert nxt[0] == ref_tokens[t], f"decode step {t} token"
        toks.append(int(nxt[0]))
    gm.cleanup_llama_model()
    _results[name] = (prompt, lg, np.array(toks, np.int32))


@pytest.mark.parametrize("name", list(SHAPES))
def test_batched_decode_bit_exact(ctx, name):
    from asicfortranai_b200.llama_model import LLaMAModel
    B, P, T = BATCH[name]
    cfg = cfg_of(name, max_batch=B)
    w = host_weights(name)
    prompts = np.stack([orc.gen_tokens(P, 12, 100 + b, cfg["vocab"]) for b in range(B)])
    gm = LLaMAModel(ctx, cfg)
    gm.init_random(0, 0.02)
    got = gm.generate(prompts, T)
    gm.cleanup_llama_model()
    om = orc.OracleModel(cfg_of(name), w)
    for b in range(B):
        om.reset()
        np.testing.assert_array_equal(got[b], om.generate(prompts[b], T), err_msg=f"sequence {b}")


@pytest.mark.parametrize("name", list(SHAPES))
def test_source_order_agreement_reported(name):
    """The source-order oracle (what transformer_layer.f90 says, with sequential sums and
    libm expf) against the GPU's prefill logits and 64 greedy steps.  The reference's
    -ffast-math build fixes no order, so this is a measurement, reported.  Where the two
    orders differ, they differ sparsely: a rounding difference moves one re-quantized
    activation (trunc(x*127), no rescale) across a step and the rows that attend to it
    follow; the other rows agree to ~1e-5.  Asserted: most prefill rows within 1e-3."""
    if name not in _results:
        pytest.skip("needs the bit-exact run of the same shape first")
    prompt, lg, toks = _results[name]
    om0 = orc.OracleModel(cfg_of(name, order=0), host_weights(name))
    ref0 = om0.forward(prompt)
    om0.reset()
    toks0 = om0.generate(prompt, STEPS + 1)
    err = rel_err(lg, ref0)
    rows = [rel_err(lg[r], ref0[r]) for r in range(PROMPT)]
    close = sum(e <= 1e-3 for e in rows)
    agree = int(np.sum(toks0 == toks))
    first = int(np.argmax(toks0 != toks)) if agree < len(toks) else len(toks)
    # the same source loops as an 8-lane vectorising build runs them (another order the
    # reference's -ffast-math build permits) against the sequential source order
    om2 = orc.OracleModel(cfg_of(name, order=2), host_weights(name))
    ref2 = om2.forward(prompt)
    om2.reset()
    toks2 = om2.generate(prompt, STEPS + 1)
    agree2 = int(np.sum(toks0 == toks2))
    rep_vec = {"prefill_rows_within_1e-3": sum(rel_err(ref2[r], ref0[r]) <= 1e-3 for r in range(PROMPT)),
               "prefill_logits_rel_err_max": rel_err(ref2, ref0), "greedy_tokens_equal": agree2,
               "first_divergence": int(np.argmax(toks0 != toks2)) if agree2 < len(toks0) else len(toks0),
               "gpu_vs_vectorised_rel_err_max": rel_err(lg, ref2)}
    rep = {"shape": name, "layers": SHAPES[name]["n_layers"], "prompt": PROMPT, "greedy_steps": STEPS,
           "vectorised_build_vs_source": rep_vec,
           "prefill_logits_rel_err_max": err, "prefill_rows_within_1e-3": close,
           "prefill_rows_rel_err": [float(f"{e:.2e}") for e in rows],
           "prefill_argmax_equal": int(sum(np.argmax(lg[r]) == np.argmax(ref0[r]) for r in range(PROMPT))),
           "greedy_tokens_equal": agree, "greedy_tokens_total": len(toks), "first_divergence": first}
    print(json.dumps(rep))
    d = os.environ.get("Q35_REPORT_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        p = os.path.join(d, "model_widths_source_order.json")
        prev = json.load(open(p)) if os.path.exists(p) else {}
        prev[name] = rep
        json.dump(prev, open(p, "w"), indent=1)
    assert close >= PROMPT // 2, rep
