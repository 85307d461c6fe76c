"""Device sampler (q35_sample.cu) against the oracle's order-1 restatement of
sampling.f90: identical 1-based tokens for every mode, parameter edge and draw; the
model's sampled generation against the oracle's generation with the same draws."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.model_util import TINY, gpu_model, make_weights

pytestmark = pytest.mark.gpu

F = np.float32
ONE_MINUS = float(np.nextafter(F(1), F(0)))
UNIFORMS = [0.0, 1e-7, 0.25, 0.5, 0.7316, 0.9, 0.999, ONE_MINUS]


@pytest.fixture(scope="module")
def ctx():
    from asicfortranai_b200.quantized import Context
    c = Context(0)
    yield c
    c.close()


def _rows(V, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "peaked":
        return rng.normal(0, 3.0, V).astype(F)
    if kind == "flat":
        return rng.normal(0, 0.05, V).astype(F)
    return (np.round(rng.normal(0, 1.0, V) * 4) / 4).astype(F)     # many ties


def _device_tokens(ctx, lg, mode, us, **kw):
    import torch
    from asicfortranai_b200 import sampling
    V = len(lg)
    R = len(us)
    t_lg = torch.from_numpy(np.tile(lg, (R, 1))).cuda()
    t_u = torch.tensor(us, dtype=torch.float32, device="cuda")
    t_tok = torch.zeros(R, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    sampling.sample_rows(ctx, mode, t_lg.data_ptr(), R, V, t_u.data_ptr(), t_tok.data_ptr(), **kw)
    ctx.synchronize()
    return t_tok.cpu().numpy()


CASES = []
for V in (1, 2, 31, 32, 33, 1000, 4097, 32000, 32768):
    for kind in ("peaked", "flat", "ties"):
        CASES.append((V, kind))


@pytest.mark.parametrize("V,kind", CASES)
def test_modes_match_oracle(ctx, V, kind):
    lg = _rows(V, kind, V * 7 + len(kind))
    params = [("greedy", 0, {})]
    params += [("temperature", 1, dict(temperature=t)) for t in (-1.0, 0.0, 0.1, 0.8, 2.0)]
    params += [("top_k", 2, dict(top_k=k)) for k in sorted({-1, 0, 1, 5, 40, max(V - 1, 1), V, V + 1})]
    params += [("top_p", 3, dict(top_p=p)) for p in (0.0, 0.5, 0.9, 0.95, 1.0, 1.5)]
    for name, mode, kw in params:
        got = _device_tokens(ctx, lg, name, UNIFORMS, **kw)
        want = [orc.sample(lg, mode, u, order=1, **kw) for u in UNIFORMS]
        np.testing.assert_array_equal(got, want, err_msg=f"V={V} {kind} {name} {kw}")


def test_reference_test_program_logits(ctx):
    """test_sampling.f90:22-28 logits: greedy 4, top-k 5 within tokens 4..8, top-p 0.9
    never 1..3 -- each draw equal to the oracle's."""
    from asicfortranai_b200 import sampling
    V = 32000
    lg = np.array([(V - i) / 1000.0 for i in range(1, V + 1)], F)
    lg[0], lg[1], lg[2], lg[99] = 5.0, 4.0, 3.0, 2.5
    assert sampling.sample_greedy(lg, V) == 4
    rng = np.random.default_rng(5)
    us = [float(x) for x in (rng.integers(0, 1 << 24, 40) * 2.0 ** -24)]
    for u in us:
        k = sampling.sample_top_k(lg, V, 5, u=u)
        assert 4 <= k <= 8 and k == orc.sample(lg, 2, u, top_k=5, order=1)
        p = sampling.sample_top_p(lg, V, 0.9, u=u)
        assert p >= 4 and p == orc.sample(lg, 3, u, top_p=0.9, order=1)
        for t in (0.1, 2.0):
            assert sampling.sample_temperature(lg, V, t, u=u) == orc.sample(lg, 1, u, temperature=t, order=1)


def test_host_entry_points_on_a_context(ctx):
    from asicfortranai_b200 import sampling
    lg = _rows(777, "peaked", 1)
    for u in UNIFORMS:
        assert sampling.sample_top_p(lg, None, 0.95, u=u, ctx=ctx) == orc.sample(lg, 3, u, top_p=0.95, order=1)
        assert sampling.sample_top_k(lg, None, 40, u=u, ctx=ctx) == orc.sample(lg, 2, u, top_k=40, order=1)
    # vocab_size shorter than the array: the first vocab_size logits (reference: logits(vocab_size))
    assert sampling.sample_greedy(lg, 10, ctx=ctx) == int(np.argmax(lg[:10])) + 1


def test_bad_arguments(ctx):
    from asicfortranai_b200 import Q35Error, sampling
    lg = np.zeros(40000, F)
    with pytest.raises(Q35Error):
        sampling.sample_top_p(lg, None, 0.9, u=0.5, ctx=ctx)          # vocabulary above 32,768
    with pytest.raises(Q35Error):
        sampling.sample_top_k(lg[:100], None, 5, u=1.0, ctx=ctx)      # u outside [0,1)
    with pytest.raises(Q35Error):
        sampling.sample_rows(ctx, 7, 0, 1, 100, 0, 0)                 # unknown mode


@pytest.mark.parametrize("mode,kw", [("top_p", dict(top_p=0.95)), ("top_k", dict(top_k=40)),
                                     ("temperature", dict(temperature=0.8))])
def test_model_generation_with_sampling_matches_oracle(ctx, mode, kw):
    cfg = dict(TINY, max_batch=2)
    w = make_weights(cfg, seed=6)
    gm = gpu_model(ctx, cfg, w)
    gm.set_sampling(mode, seed=99, **kw)
    prompts = np.stack([orc.gen_tokens(9, 6, 40 + b, cfg["vocab"]) for b in range(2)])
    got = gm.generate(prompts, 32)
    smp = dict(mode={"temperature": 1, "top_k": 2, "top_p": 3}[mode], seed=99, **kw)
    for b in range(2):
        om = orc.OracleModel(dict(TINY, max_batch=1), w)
        want = om.generate(prompts[b], 32, sampling=smp, seq=b)
        np.testing.assert_array_equal(got[b], want, err_msg=f"sequence {b}")
    # a second run restarts the draws: the same tokens again
    again = gm.generate(prompts, 32)
    for b in range(2):
        np.testing.assert_array_equal(again[b], got[b])
    # back to greedy: the oracle's greedy tokens
    gm.set_sampling("greedy")
    g = gm.generate(prompts, 16)
    om = orc.OracleModel(dict(TINY, max_batch=1), w)
    np.testing.assert_array_equal(g[0], om.generate(prompts[0], 16))
    gm.cleanup_llama_model()


def test_decode_step_sampling_after_graph(ctx):
    """Changing the rule after the decode graph was captured re-captures it."""
    cfg = dict(TINY)
    w = make_weights(cfg, seed=8)
    gm = gpu_model(ctx, cfg, w)
    prompt = orc.gen_tokens(7, 8, 3, cfg["vocab"])
    gm.forward_next_token(prompt)
    gm.decode_step()                       # greedy graph
    gm.reset_kv_cache()
    gm.set_sampling("top_p", top_p=0.9, seed=3)
    got = gm.generate(prompt[None, :], 12)[0]
    om = orc.OracleModel(cfg, w)
    want = om.generate(prompt, 12, sampling=dict(mode=3, top_p=0.9, seed=3), seq=0)
    np.testing.assert_array_equal(got, want)
    gm.cleanup_llama_model()
