"""Pins the CPU oracle (oracle/psgd_oracle.py) to the reference: the golden vectors in tests/golden/ were made by
running the reference itself (tests/golden/make_golden.py) on seeded inputs; here the oracle replays the same
parameters, gradients and random draws and must land on the same Q, L, parameters and preconditioned gradients."""
import json
import os

import numpy as np
import pytest

from oracle import psgd_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SCEN = ["config1", "mixed_inf", "mixed_skew1", "whiten_momentum", "prob_half"]


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a - b))


def load(name):
    z = np.load(os.path.join(GOLD, name + ".npz"))
    return {k: z[k] for k in z.files}


def reference_order_draws(rng, opt, srcs, forced):
    """One step's draws in the order psgd_pro.KronWhiten.step asks for them: the update coin (psgd_pro.py:345),
    then per parameter randn_like(G) (:123), randn(32, n) for each dense factor's two norm bounds (:35, :59) and
    the balancing coin (:138)."""
    u = float(rng.random(dtype=np.float32))
    d = {"update": u, "coins": [], "normals": []}
    if not u < opt.preconditioner_update_probability:
        return d
    for k, (QL, g) in enumerate(zip(opt.QL, srcs)):
        nd = [np.asarray(rng.standard_normal(g.shape, dtype=np.float32))]
        for q in QL[0]:
            if q.ndim == 2:
                nd += [rng.standard_normal((O.K_SUBSPACE, q.shape[0]), dtype=np.float32) for _ in range(2)]
        c = float(rng.random(dtype=np.float32))
        d["normals"].append(nd)
        d["coins"].append(0.0 if k in forced else c)
    return d


def replay(name, dtype=np.float64):
    g = load(name)
    meta = json.loads(str(g["meta"]))
    kw = {k: (float("inf") if v == "inf" else v) for k, v in meta["kw"].items()}
    rng_params = np.random.default_rng(1000 + meta["seed"])
    rng_grads = np.random.default_rng(2000 + meta["seed"])
    rng_draws = np.random.default_rng(3000 + meta["seed"])
    params = [np.asarray(rng_params.standard_normal(tuple(s), dtype=np.float32)) for s in meta["shapes"]]
    opt = O.KronWhitenOracle(params, dtype=dtype, **kw)
    pre = None
    for step in range(1, meta["steps"] + 1):
        G = [np.asarray(rng_grads.standard_normal(tuple(s), dtype=np.float32) * np.float32(sc), dtype=np.float32)
             for s, sc in zip(meta["shapes"], meta["grad_scale"])]
        Gs = [np.squeeze(x).astype(dtype) for x in G]
        if opt.QL is None:
            opt._init_on_the_fly(Gs)
        # the update source (gradient or momentum) decides the noise shapes; both have the gradient's shape
        forced = meta["force_balance"].get(str(step), [])
        draws = reference_order_draws(rng_draws, opt, Gs, forced)
        pre = opt.step(G, draws)
    return g, opt, pre


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
