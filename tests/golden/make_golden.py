"""Generates the golden vectors in tests/golden/*.npz by running the reference implementation itself.

Run here, where the reference checkout exists (it does not travel to GPU boxes):
    python tests/golden/make_golden.py /path/to/reference      (or PSGD_REFERENCE=/path/to/reference)
The reference imports the third-party opt_einsum, which is absent; tests/golden/standin provides the three names
it uses (see that package's docstring). Every Gaussian and uniform draw the reference makes through torch
(randn_like(G) for the damping noise, randn(32, n) for the norm-bound starts, rand([]) for the update and
balancing coins) is served from a numpy Generator seeded per scenario, in the order the reference asks for them.
tests/test_oracle_golden.py replays the same stream into the oracle (oracle/psgd_oracle.py).

Scenario parameters, gradients and draws are all derived from the seed; each .npz stores the scenario metadata
(json) and the reference's state after the last step: Q factors, L, parameters and the last preconditioned
gradients (before clipping). Scenarios marked "sketch" (the large bf16 case of the benchmarked path) store
two-sided sketches of the matrices instead (tests/golden/sketch.py), and the parameter change instead of the
parameter; "grad_bf16" scenarios round every gradient to bf16 values, which the reference then sees as fp32.

    python tests/golden/make_golden.py /path/to/reference [scenario names ...]   (default: all)"""
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PSGD_REFERENCE", "")
ONLY = set(sys.argv[2:])
sys.path.insert(0, HERE)
from sketch import sketch  # noqa: E402

SCENARIOS = [
    # config 1 of the benchmark plan: one fp32 256 x 512 weight, both factors dense, 10 steps
    dict(name="config1", shapes=[[256, 512]], steps=10, grad_scale=[0.01], seed=0,
         kw=dict(preconditioner_init_scale=1.0, preconditioner_max_skew=float("inf"), lr_params=1e-3)),
    # every factor kind with max_skew = inf: dense 2-D, 1-D dense, size-1 dim, 0-d scalar, squeezed (1, 33)
    dict(name="mixed_inf", shapes=[[48, 80], [10, 65], [65], [1], [], [1, 33]], steps=4,
         grad_scale=[1e-2, 3e-2, 1e-3, 0.5, 0.2, 1e-2], seed=1, force_balance={2: [0, 1], 3: [3]},
         kw=dict(preconditioner_max_skew=float("inf"), lr_params=1e-2)),
    # the reference default max_skew = 1 and a max_size: diagonal factors on 2-D and 1-D, momentum, update last
    dict(name="mixed_skew1", shapes=[[48, 80], [100, 20], [65], [30, 30]], steps=3,
         grad_scale=[1e-2, 1e-2, 1e-2, 1e-1], seed=2,
         kw=dict(preconditioner_max_size=64, momentum=0.9, update_preconditioner_first=False,
                 preconditioner_init_scale=0.5)),
    # whitening the momentum instead of the gradient
    dict(name="whiten_momentum", shapes=[[40, 24], [24]], steps=3, grad_scale=[1e-2, 1e-2], seed=3,
         kw=dict(whiten_grad=False, momentum=0.5, preconditioner_max_skew=float("inf"))),
    # preconditioner updated with probability 1/2 (the coin decides per step)
    dict(name="prob_half", shapes=[[32, 16]], steps=6, grad_scale=[1e-2], seed=4,
         kw=dict(preconditioner_update_probability=0.5, preconditioner_max_skew=float("inf"),
                 preconditioner_init_scale=1.0)),
    # the benchmarked path at its own sizes: the factor sizes of the Llama-style set (2048, 256, 5632), a 1-D 2048
    # parameter and an embedding whose 32000 dim exceeds max size 8192 (a diagonal factor); gradients N(0, 1e-3^2)
    # rounded to bf16 values, the init scale taken on the fly, max_skew = inf
    # order-3 and order-4 parameters (a conv-shaped 16 x 12 x 3 x 3 weight, a squeezed (20, 1, 7, 4), a 3-D
    # parameter whose 70 dim exceeds max size 64 and gets a diagonal factor) beside a matrix, momentum 0.9
    dict(name="nd_momentum", shapes=[[16, 12, 3, 3], [20, 1, 7, 4], [70, 6, 5], [24, 10]], steps=3,
         grad_scale=[1e-2, 2e-2, 1e-2, 1e-2], seed=6, force_balance={2: [0], 3: [2]},
         kw=dict(preconditioner_max_skew=float("inf"), preconditioner_max_size=64, momentum=0.9, lr_params=1e-2)),
    dict(name="llama_block_bf16", shapes=[[2048, 2048], [256, 2048], [5632, 2048], [2048, 5632], [2048],
                                          [32000, 2048]], steps=3,
         grad_scale=[1e-3] * 6, seed=5, sketch=True, grad_bf16=True,
         kw=dict(preconditioner_max_size=8192, preconditioner_max_skew=float("inf"))),
]


class DrawServer:
    """Serves the reference's torch random calls from a numpy Generator, checking shapes."""

    def __init__(self, rng, torch):
        self.rng, self.torch, self.log = rng, torch, []
        self.force = set()  # indices (into the coin sequence) of balancing coins forced to 0.0
        self.coin_count = -1

    def randn_like(self, G):
        x = np.asarray(self.rng.standard_normal(tuple(G.shape), dtype=np.float32))
        self.log.append(("n", tuple(G.shape)))
        return self.torch.from_numpy(x).to(G.dtype)

    def randn(self, *shape, dtype=None, device=None):
        x = self.rng.standard_normal(tuple(shape), dtype=np.float32)
        self.log.append(("n", tuple(shape)))
        return self.torch.from_numpy(x).to(dtype or self.torch.float32)

    def rand(self, shape):
        assert list(shape) == []
        x = float(self.rng.random(dtype=np.float32))
        self.log.append(("u", ()))
        return self.torch.tensor(x)


def torch_proxy(real, server):
    mod = types.ModuleType("torch_proxy")
    for name in dir(real):
        if not name.startswith("__"):
            try:
                setattr(mod, name, getattr(real, name))
            except Exception:
                pass
    mod.randn_like, mod.randn, mod.rand = server.randn_like, server.randn, server.rand
    return mod


def grads_for(rng, shapes, scales, bf16=False):
    out = [np.asarray(rng.standard_normal(tuple(s), dtype=np.float32) * np.float32(sc), dtype=np.float32)
           for s, sc in zip(shapes, scales)]
    return [to_bf16_values(g) for g in out] if bf16 else out


def to_bf16_values(x):
    """float32 array rounded to the nearest bf16 value (round to nearest even), still float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return r.view(np.float32)


def run_scenario(sc, torch, psgd_pro):
    rng_params = np.random.default_rng(1000 + sc["seed"])
    rng_grads = np.random.default_rng(2000 + sc["seed"])
    rng_draws = np.random.default_rng(3000 + sc["seed"])
    params = [torch.nn.Parameter(torch.from_numpy(np.asarray(rng_params.standard_normal(tuple(s), dtype=np.float32))))
              for s in sc["shapes"]]
    server = DrawServer(rng_draws, torch)
    real_torch = psgd_pro.torch
    psgd_pro.torch = torch_proxy(real_torch, server)
    # balancing coins: the reference draws torch.rand([]) after each parameter's update; force some to 0.0
    forced = sc.get("force_balance", {})
    step_box = [0]
    orig_rand = server.rand
    state = {"param_idx": 0}

    orig_update = psgd_pro.update_precond_kron_whiten_q0p5eq1p5

    def update_wrapped(QL, exprs, G, **kw):
        k = state["param_idx"]
        state["param_idx"] += 1
        if k in forced.get(step_box[0], []):
            def rand_forced(shape):
                orig_rand(shape)  # consume the draw, return 0.0
                return torch.tensor(0.0)
            server_rand_prev = psgd_pro.torch.rand
            psgd_pro.torch.rand = rand_forced
            try:
                return orig_update(QL, exprs, G, **kw)
            finally:
                psgd_pro.torch.rand = server_rand_prev
        return orig_update(QL, exprs, G, **kw)

    opt = psgd_pro.KronWhiten(params, **sc["kw"])
    opt._update_precond = update_wrapped
    captured = {}
    orig_pg = opt._precond_grad

    def pg_wrapped(*a):
        out = orig_pg(*a)
        captured.setdefault("pre", []).append(out.detach().clone())
        return out
    opt._precond_grad = pg_wrapped

    try:
        for step in range(1, sc["steps"] + 1):
            step_box[0] = step
            state["param_idx"] = 0
            captured["pre"] = []
            G = grads_for(rng_grads, sc["shapes"], sc["grad_scale"], sc.get("grad_bf16", False))

            def closure():
                return sum((p * torch.from_numpy(g)).sum() for p, g in zip(params, G))
            opt.step(closure)
    finally:
        psgd_pro.torch = real_torch
    out = {}
    sk = sc.get("sketch", False)
    keep = (lambda x: sketch(x)) if sk else (lambda x: np.asarray(x, dtype=np.float32))
    rng_p0 = np.random.default_rng(1000 + sc["seed"])
    for k, (QL, _) in enumerate(opt._QLs_exprs):
        Q, L = QL
        for i, q in enumerate(Q):
            out[f"Q_{k}_{i}"] = keep(q.detach().numpy())
            out[f"L_{k}_{i}"] = np.float32(L[i].item())
        p0 = np.asarray(rng_p0.standard_normal(tuple(sc["shapes"][k]), dtype=np.float32))
        if sk:
            out[f"dparam_{k}"] = sketch(params[k].detach().numpy().astype(np.float64) - p0)
        else:
            out[f"param_{k}"] = params[k].detach().numpy().astype(np.float32)
        out[f"pre_{k}"] = keep(captured["pre"][k].numpy())
    meta = dict(sc)
    meta["kw"] = {k: (v if v != float("inf") else "inf") for k, v in sc["kw"].items()}
    meta["force_balance"] = {str(k): v for k, v in sc.get("force_balance", {}).items()}
    meta["draw_log_len"] = len(server.log)
    out["meta"] = np.array(json.dumps(meta))
    return out


def run_fast_r2(torch, fast):
    """psgd_pro_fast.update_2d (the P-cached 2-D path) with r2 = False and True, 3 steps on a 48 x 80 gradient."""
    out = {}
    for r2 in (False, True):
        rng = np.random.default_rng(77)
        q1, q2 = torch.eye(48) * 0.7, torch.eye(80) * 0.7
        Q, L = [q1, q2], [torch.zeros([]), torch.zeros([])]
        P = [fast.gram_2d(q, fast.EagerOps) for q in Q]
        for _ in range(3):
            G = torch.from_numpy(rng.standard_normal((48, 80), dtype=np.float32) * np.float32(0.02))
            rnd = [torch.from_numpy(rng.standard_normal((48, 80), dtype=np.float32))]
            for n in (48, 80):
                rnd += [torch.from_numpy(rng.standard_normal((32, n), dtype=np.float32)) for _ in range(2)]
            fast.update_2d([Q, L], P, G, rnd, lr=0.1, betaL=0.9, damping=1e-9, r2=r2)
        tag = "r2" if r2 else "p2"
        for i in range(2):
            out[f"{tag}_Q_{i}"] = Q[i].numpy().astype(np.float32)
            out[f"{tag}_L_{i}"] = np.float32(L[i].item())
    return out


def run_units(torch, psgd_pro, fast):
    rng = np.random.default_rng(5)
    out = {}
    for n in (65, 200):
        X = torch.from_numpy(rng.standard_normal((n, n + 7), dtype=np.float32))
        A = X @ X.T
        S = torch.from_numpy(rng.standard_normal((n, n), dtype=np.float32))
        Sk = S - S.T
        V1 = torch.from_numpy(rng.standard_normal((32, n), dtype=np.float32))
        V2 = torch.from_numpy(rng.standard_normal((32, n), dtype=np.float32))
        out[f"spd_A_{n}"], out[f"spd_V_{n}"] = A.numpy(), V1.numpy()
        out[f"spd_out_{n}"] = np.float32(fast.norm_lower_bound_spd(A, V1).item())
        out[f"skh_A_{n}"], out[f"skh_V_{n}"] = Sk.numpy(), V2.numpy()
        out[f"skh_out_{n}"] = np.float32(fast.norm_lower_bound_skh(Sk, V2).item())
    Q = torch.eye(50) + 0.05 * torch.from_numpy(rng.standard_normal((50, 50), dtype=np.float32))
    V = torch.from_numpy(rng.standard_normal((32, 50), dtype=np.float32))
    out["proc_Q_in"], out["proc_V"] = Q.numpy().copy(), V.numpy()
    Q2 = Q.clone()
    fast.procrustes_step2(Q2, V)
    out["proc_Q_out"] = Q2.numpy()
    Qr = Q.clone()
    fast.procrustes_step_r2(Qr, V)
    out["procr2_Q_out"] = Qr.numpy()
    Qs = [torch.from_numpy(rng.standard_normal((n, n), dtype=np.float32)) * s for n, s in ((5, 3.0), (7, 0.01))]
    Qs.append(torch.from_numpy(rng.standard_normal(9, dtype=np.float32)) * 40.0)
    for i, q in enumerate(Qs):
        out[f"bal_in_{i}"] = q.numpy().copy()
    psgd_pro.balance_kron_precond(Qs)
    for i, q in enumerate(Qs):
        out[f"bal_out_{i}"] = q.numpy()
    return out


def main():
    if not REF or not os.path.isdir(REF):
        sys.exit("usage: make_golden.py /path/to/reference (the psgd_pro checkout; or set PSGD_REFERENCE)")
    sys.path.insert(0, os.path.join(HERE, "standin"))
    sys.path.insert(0, REF)
    import torch
    torch.set_num_threads(8)
    torch.backends.opt_einsum.enabled = False  # torch would otherwise route einsum through the stand-in
    import psgd_pro
    import psgd_pro_fast as fast
    for sc in SCENARIOS:
        if ONLY and sc["name"] not in ONLY:
            continue
        out = run_scenario(sc, torch, psgd_pro)
        np.savez_compressed(os.path.join(HERE, sc["name"] + ".npz"), **out)
        print("wrote", sc["name"], sum(v.size for v in out.values()), "values")
    if not ONLY or "fast_r2" in ONLY:
        np.savez_compressed(os.path.join(HERE, "fast_r2.npz"), **run_fast_r2(torch, fast))
    if not ONLY or "units" in ONLY:
        np.savez_compressed(os.path.join(HERE, "units.npz"), **run_units(torch, psgd_pro, fast))
    print("done")


if __name__ == "__main__":
    main()
