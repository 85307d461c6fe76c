"""The oracle's reduction orders (CPU only): the source's sequential loops with the C
library's expf (order 0), the GPU kernels' tree order with q35_expf (order 1), and the
source loops as an 8-lane vectorising build runs them (order 2).  Documents how far they
drift apart; the GPU is held bit-exact to order 1."""
import numpy as np

from oracle import oracle as orc
from tests.model_util import TINY, make_weights, rel_err


def test_tree_rmsnorm_close_to_sequential():
    x = orc.gen_normal((5, 8192), 3, 1, 1.0)
    w = (1.0 + orc.gen_normal((8192,), 3, 2, 0.02)).astype(np.float32)
    a = orc.rms_norm(x, w)
    b = np.zeros_like(a, order="F")
    orc.lib().orc_rms_norm_tree(np.asfortranarray(x), w, b, 5, 8192, 1e-5)
    assert rel_err(b, a) < 1e-6


def test_q35_expf_accuracy():
    xs = np.linspace(-100, 88, 200001, dtype=np.float32)
    L = orc.lib()
    got = np.array([L.orc_q35_expf(float(x)) for x in xs[::40]], np.float32)
    ref = np.exp(xs[::40].astype(np.float64))
    ulp = np.abs(got - ref) / np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert ulp.max() < 1.0


def test_orders_agree_without_boundary_crossings():
    cfg = dict(TINY, hidden=256, n_heads=2, n_kv_heads=1, ffn=512)
    w = make_weights(cfg, seed=2)
    ids = orc.gen_tokens(7, 2, 5, cfg["vocab"])
    a = orc.OracleModel(dict(cfg, order=0), w).forward(ids)
    b = orc.OracleModel(dict(cfg, order=1), w).forward(ids)
    assert rel_err(a, b) < 1e-3


def test_orders_drift_with_int8_boundary_crossings():
    """hidden 512: one sum of squares differs by a few ulps between the orders, one int8
    activation lands a step apart, and every later value moves -- the reason the GPU is
    held to one fixed order rather than to a tolerance."""
    cfg = dict(TINY, wformat=1)
    w = make_weights(cfg, seed=2)
    ids = orc.gen_tokens(7, 2, 5, cfg["vocab"])
    a = orc.OracleModel(dict(cfg, order=0), w).forward(ids)
    b = orc.OracleModel(dict(cfg, order=1), w).forward(ids)
    assert rel_err(a, b) > 1e-3


def test_a_vectorised_build_of_the_source_moves_as_far_as_the_gpu_order():
    """The hidden-512 model of the test above: reading the same source loops the way an
    8-lane -ffast-math build does (order 2) lands as far from the sequential order as the
    GPU's order does, and close to the GPU's order -- the sequential order is one of
    several the reference's own build may take."""
    cfg = dict(TINY, wformat=1)
    w = make_weights(cfg, seed=2)
    ids = orc.gen_tokens(7, 2, 5, cfg["vocab"])
    a, b, c = (orc.OracleModel(dict(cfg, order=o), w).forward(ids) for o in (0, 1, 2))
    assert rel_err(c, a) > 1e-3
    assert rel_err(c, b) < 1e-5
