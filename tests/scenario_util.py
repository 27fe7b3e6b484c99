"""Shared helpers for the parity tests: golden fixture loading and the reference-order random draw stream
(the same stream tests/golden/make_golden.py served to the reference)."""
import json
import os

import numpy as np

from oracle import psgd_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SCEN = ["config1", "mixed_inf", "mixed_skew1", "whiten_momentum", "prob_half", "nd_momentum"]


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a - b))


def load(name):
    z = np.load(os.path.join(GOLD, name + ".npz"))
    return {k: z[k] for k in z.files}


def meta_of(g):
    meta = json.loads(str(g["meta"]))
    meta["kw"] = {k: (float("inf") if v == "inf" else v) for k, v in meta["kw"].items()}
    return meta


def reference_order_draws(rng, QL, shapes, prob, forced):
    """One step's draws in the order psgd_pro.KronWhiten.step asks for them: the update coin (psgd_pro.py:345),
    then per parameter randn_like(G) (:123), randn(32, n) for each dense factor's two norm bounds (:35, :59) and
    the balancing coin (:138). QL: the oracle's per-parameter (Q list, L list), which fixes dense/diagonal."""
    u = float(rng.random(dtype=np.float32))
    d = {"update": u, "coins": [], "normals": []}
    if not u < prob:
        return d
    for k, (ql, shp) in enumerate(zip(QL, shapes)):
        nd = [np.asarray(rng.standard_normal(shp, dtype=np.float32))]
        for q in ql[0]:
            if q.ndim == 2:
                nd += [rng.standard_normal((O.K_SUBSPACE, q.shape[0]), dtype=np.float32) for _ in range(2)]
        c = float(rng.random(dtype=np.float32))
        d["normals"].append(nd)
        d["coins"].append(0.0 if k in forced else c)
    return d


class _FactorShape:
    """Stands in for a Q factor where only its kind matters (ndim 2: dense n x n, ndim 1: diagonal)."""

    def __init__(self, n, dense):
        self.ndim, self.shape = (2 if dense else 1), ((n, n) if dense else (n,))


def factor_layout(shapes, max_size, max_skew):
    """(Q list, L list) stand-ins with the dense / diagonal kinds of psgd_pro.py:189, for drawing the reference-order
    random stream without building the factors (the oracle's init_kron would allocate every n x n identity)."""
    out = []
    for shp in shapes:
        shp = tuple(shp)
        if len(shp) == 0:
            out.append(([_FactorShape(1, False)], [0.0]))
            continue
        numel = int(np.prod(shp))
        out.append(([_FactorShape(n, O.is_dense(n, numel, max_size, max_skew)) for n in shp], [0.0] * len(shp)))
    return out


def to_bf16_values(x):
    """float32 array rounded to the nearest bf16 value (round to nearest even), still float32; the rounding
    tests/golden/make_golden.py applies to the gradients of its grad_bf16 scenarios."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return r.view(np.float32)


class Scenario:
    """Parameters, per-step gradients and draws of a golden scenario, in the reference order."""

    def __init__(self, name):
        self.g = load(name)
        self.meta = meta_of(self.g)
        m = self.meta
        self.rng_params = np.random.default_rng(1000 + m["seed"])
        self.rng_grads = np.random.default_rng(2000 + m["seed"])
        self.rng_draws = np.random.default_rng(3000 + m["seed"])
        self.params = [np.asarray(self.rng_params.standard_normal(tuple(s), dtype=np.float32)) for s in m["shapes"]]

    def grads(self):
        m = self.meta
        out = [np.asarray(self.rng_grads.standard_normal(tuple(s), dtype=np.float32) * np.float32(sc),
                          dtype=np.float32) for s, sc in zip(m["shapes"], m["grad_scale"])]
        return [to_bf16_values(g) for g in out] if m.get("grad_bf16") else out

    def draws(self, step, QL, grads):
        shapes = [np.squeeze(x).shape for x in grads]
        forced = self.meta["force_balance"].get(str(step), [])
        prob = self.meta["kw"].get("preconditioner_update_probability", 1.0)
        return reference_order_draws(self.rng_draws, QL, shapes, prob, forced)
