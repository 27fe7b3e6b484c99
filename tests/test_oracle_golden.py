"""Pins the CPU oracle (oracle/psgd_oracle.py) to the reference: the golden vectors in tests/golden/ were made by
running the reference itself (tests/golden/make_golden.py) on seeded inputs; here the oracle replays the same
parameters, gradients and random draws and must land on the same Q, L, parameters and preconditioned gradients."""
import numpy as np
import pytest

from oracle import psgd_oracle as O
from scenario_util import SCEN, Scenario, load, rel


def replay(name, dtype=np.float64):
    sc = Scenario(name)
    opt = O.KronWhitenOracle(sc.params, dtype=dtype, **sc.meta["kw"])
    pre = None
    for step in range(1, sc.meta["steps"] + 1):
        G = sc.grads()
        if opt.QL is None:
            opt._init_on_the_fly([np.squeeze(x).astype(dtype) for x in G])
        pre = opt.step(G, sc.draws(step, opt.QL, G))
    return sc.g, opt, pre


@pytest.mark.parametrize("name", SCEN)
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_oracle_matches_reference(name, dtype):
    g, opt, pre = replay(name, dtype)
    tol = 1e-5  # measured: Q ~1e-7, Pg ~7e-7 (fp32 rounding of the reference run)
    worst = 0.0
    for k, (Q, L) in enumerate(opt.QL):
        for i, q in enumerate(Q):
            e = rel(q, g[f"Q_{k}_{i}"])
            worst = max(worst, e)
            assert e < tol, (name, k, i, e)
            assert abs(L[i] - float(g[f"L_{k}_{i}"])) <= tol * abs(float(g[f"L_{k}_{i}"])) + 1e-30
        assert rel(opt.params[k], g[f"param_{k}"]) < 1e-5
        assert rel(pre[k], g[f"pre_{k}"]) < tol, (name, k, rel(pre[k], g[f"pre_{k}"]))


def test_oracle_matches_reference_at_benchmark_sizes():
    """The benchmarked path's sizes (llama_block_bf16: factors of 2048, 256 and 5632, a 1-D 2048 parameter, a
    32000 x 2048 embedding with a diagonal factor; bf16 gradient values; init scale on the fly): the fp32 oracle
    against the reference's own outputs, stored as sketches (tests/golden/sketch.py). About a minute of CPU."""
    import sys
    import os
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    from sketch import sketch
    g, opt, pre = replay("llama_block_bf16", np.float32)
    errs = {}
    for k, (Q, L) in enumerate(opt.QL):
        for i, q in enumerate(Q):
            errs[f"Q_{k}_{i}"] = rel(sketch(q), g[f"Q_{k}_{i}"])
            assert abs(L[i] - float(g[f"L_{k}_{i}"])) <= 1e-5 * abs(float(g[f"L_{k}_{i}"]))
        errs[f"pre_{k}"] = rel(sketch(pre[k]), g[f"pre_{k}"])
    assert max(errs.values()) < 1e-5, errs  # measured: Q ~1e-7, Pg ~1.5e-6


def test_fast_r2_paths():
    """oracle update_precond (r2 False/True) against psgd_pro_fast.update_2d on the same draws."""
    g = load("fast_r2")
    for r2, tag in ((False, "p2"), (True, "r2")):
        rng = np.random.default_rng(77)
        Q, L = [np.eye(48) * 0.7, np.eye(80) * 0.7], [0.0, 0.0]
        for _ in range(3):
            G = (rng.standard_normal((48, 80), dtype=np.float32) * np.float32(0.02)).astype(np.float64)
            rnd = [rng.standard_normal((48, 80), dtype=np.float32)]
            for n in (48, 80):
                rnd += [rng.standard_normal((32, n), dtype=np.float32) for _ in range(2)]
            Q, L, _ = O.update_precond(Q, L, G, rnd, lr=0.1, betaL=0.9, damping=1e-9, r2=r2)
        for i in range(2):
            assert rel(Q[i], g[f"{tag}_Q_{i}"]) < 1e-4
            assert abs(L[i] - float(g[f"{tag}_L_{i}"])) < 1e-4 * abs(float(g[f"{tag}_L_{i}"]))


def test_units():
    g = load("units")
    for n in (65, 200):
        assert abs(O.norm_lower_bound_spd(g[f"spd_A_{n}"].astype(np.float64), g[f"spd_V_{n}"]) /
                   float(g[f"spd_out_{n}"]) - 1) < 1e-5
        assert abs(O.norm_lower_bound_skh(g[f"skh_A_{n}"].astype(np.float64), g[f"skh_V_{n}"]) /
                   float(g[f"skh_out_{n}"]) - 1) < 1e-5
    Q, V = g["proc_Q_in"].astype(np.float64), g["proc_V"]
    assert rel(O.procrustes_step2(Q, V), g["proc_Q_out"]) < 1e-6
    assert rel(O.procrustes_step_r2(Q, V), g["procr2_Q_out"]) < 1e-6
    bal = O.balance_kron_precond([g[f"bal_in_{i}"].astype(np.float64) for i in range(3)])
    for i in range(3):
        assert rel(bal[i], g[f"bal_out_{i}"]) < 1e-6


def test_init_rule():
    """psgd_pro.py:189 dense/diagonal rule and the scale^(1/order) identity init (:181, :191, :210)."""
    Q, L = O.init_kron((256, 512), 1.0, max_skew=1.0)
    assert Q[0].ndim == 2 and Q[1].ndim == 1  # 512^2 > 131072: diagonal under the default skew
    Q, L = O.init_kron((256, 512), 4.0, max_skew=float("inf"))
    assert Q[0].shape == (256, 256) and np.allclose(np.diag(Q[1]), 2.0)
    Q, _ = O.init_kron((3, 200), 1.0, max_size=100, max_skew=float("inf"))
    assert Q[0].ndim == 2 and Q[1].ndim == 1
    Q, _ = O.init_kron((), 9.0)
    assert Q[0].ndim == 0 and float(Q[0]) == 9.0
