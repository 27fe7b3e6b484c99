"""End-to-end parity of psgd_pro_b200.KronWhiten (the sm_100a step) with the CPU oracle and the reference's golden
outputs, on the golden scenarios with identical parameters, gradients and random draws.

Tolerances (relative Frobenius error after the scenario's steps): precision="fp32" 1e-3 on every Q factor and the
preconditioned gradient; precision="bf16" (one bf16 MMA per product, fp32 accumulation) 2e-2."""
import numpy as np
import pytest
import torch

from oracle import psgd_oracle as O
from psgd_pro_b200 import KronWhiten
from scenario_util import SCEN, Scenario, rel

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-3, "bf16": 2e-2}


def run_pair(name, precision, cuda):
    sc = Scenario(name)
    kw = sc.meta["kw"]
    ora = O.KronWhitenOracle(sc.params, dtype=np.float64, **kw)
    params = [torch.nn.Parameter(torch.from_numpy(p.copy()).to(cuda)) for p in sc.params]
    opt = KronWhiten(params, precision=precision, **kw)
    pre = None
    for step in range(1, sc.meta["steps"] + 1):
        G = sc.grads()
        if ora.QL is None:
            ora._init_on_the_fly([np.squeeze(x).astype(np.float64) for x in G])
        draws = sc.draws(step, ora.QL, G)
        pre = ora.step(G, draws)
        opt.step_math([torch.from_numpy(x).to(cuda) for x in G], draws=draws)
    torch.cuda.synchronize()
    opt.check_errors()
    return sc, ora, opt, pre


@pytest.mark.parametrize("name", SCEN)
@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_step_matches_oracle_and_reference(cuda, name, precision):
    sc, ora, opt, pre = run_pair(name, precision, cuda)
    tol = TOL[precision]
    st = opt.state_dict()["state"]
    for k, ((Qo, Lo), s) in enumerate(zip(ora.QL, st)):
        for i, (qo, qg) in enumerate(zip(Qo, s["Q"])):
            qg = qg.detach().cpu().numpy()
            assert np.isfinite(qg).all()
            e_ora = rel(qg, qo)
            e_ref = rel(qg, sc.g[f"Q_{k}_{i}"])
            assert e_ora < tol and e_ref < tol, (name, k, i, e_ora, e_ref)
            lg = float(s["L"][i])
            assert abs(lg - Lo[i]) <= tol * abs(Lo[i]) + 1e-30, (name, k, i, lg, Lo[i])
        pg = opt._plan.params[k].pg32.detach().cpu().numpy().reshape(np.shape(pre[k]))
        assert rel(pg, pre[k]) < tol, (name, k, rel(pg, pre[k]))
        assert rel(pg, sc.g[f"pre_{k}"]) < tol
        assert rel(opt._params_with_grad[k].detach().cpu().numpy(), sc.g[f"param_{k}"]) < tol


def test_graphs_match_eager(cuda):
    """Device-drawn noise: the captured CUDA-graph step gives bitwise the eager result from the same seed."""
    torch.manual_seed(0)
    shapes = [(96, 200), (300,), (64, 64), (5000, 48)]
    base = [torch.randn(s) * 0.1 for s in shapes]
    grads = [[torch.randn(s).to(cuda) * 1e-2 for s in shapes] for _ in range(4)]
    out = []
    for graphs in (False, True):
        params = [torch.nn.Parameter(b.clone().to(cuda)) for b in base]
        opt = KronWhiten(params, preconditioner_init_scale=1.0, preconditioner_max_skew=float("inf"),
                         preconditioner_max_size=4096, cuda_graphs=graphs)
        torch.manual_seed(123)
        torch.cuda.manual_seed(123)
        for g in grads:
            opt.step_math(g)
        torch.cuda.synchronize()
        opt.check_errors()
        out.append([p.detach().clone() for p in params] + [q for s in opt.state_dict()["state"] for q in s["Q"]])
    for a, b in zip(*out):
        assert torch.equal(a, b)


def test_state_dict_roundtrip(cuda):
    """Save after 2 steps, load into a fresh optimizer, continue: same result as an uninterrupted run."""
    sc = Scenario("mixed_inf")
    kw = dict(sc.meta["kw"], preconditioner_init_scale=0.8)
    ora = O.KronWhitenOracle(sc.params, dtype=np.float64, **kw)
    G_all = [sc.grads() for _ in range(4)]
    D_all = []
    for step, G in enumerate(G_all, 1):
        d = sc.draws(step, ora.QL, G)
        D_all.append(d)
        ora.step(G, d)
    mk = lambda: [torch.nn.Parameter(torch.from_numpy(p.copy()).to(cuda)) for p in sc.params]
    pa = mk()
    a = KronWhiten(pa, **kw)
    for G, d in zip(G_all, D_all):
        a.step_math([torch.from_numpy(x).to(cuda) for x in G], draws=d)
    pb = mk()
    b = KronWhiten(pb, **kw)
    for G, d in zip(G_all[:2], D_all[:2]):
        b.step_math([torch.from_numpy(x).to(cuda) for x in G], draws=d)
    saved = {"state": [{"Q": [q.clone() for q in s["Q"]], "L": [l.clone() for l in s["L"]], "m": s["m"]}
                       for s in b.state_dict()["state"]], "counter_m": 0}
    pc = [torch.nn.Parameter(p.detach().clone()) for p in pb]
    c = KronWhiten(pc, **kw)
    c.load_state_dict(saved)
    for G, d in zip(G_all[2:], D_all[2:]):
        c.step_math([torch.from_numpy(x).to(cuda) for x in G], draws=d)
    torch.cuda.synchronize()
    for x, y in zip(a.state_dict()["state"], c.state_dict()["state"]):
        for qa, qc in zip(x["Q"], y["Q"]):
            assert rel(qc.cpu().numpy(), qa.cpu().numpy()) < 1e-5
    for x, y in zip(pa, pc):
        assert rel(y.detach().cpu().numpy(), x.detach().cpu().numpy()) < 1e-6


@pytest.mark.parametrize("whiten_grad,update_first,gdt", [(False, True, torch.float32), (False, False, torch.float32),
                                                          (True, True, torch.bfloat16), (False, True, torch.bfloat16)])
def test_momentum_in_the_staging_kernel(cuda, whiten_grad, update_first, gdt):
    """The momentum EMA (psgd_pro.py:334-343) runs inside the staging kernel, in whichever staging pass of the step
    reads the momentum first; with update probability 1/2 the preconditioner update is skipped on some steps, so
    the EMA moves between the update's pass and the apply's pass. Compared with the oracle on the same draws; with
    bf16 gradients the momentum is a bf16 tensor as in the reference (rounded at each in-place op), so the bar is
    the bf16 one."""
    rng = np.random.default_rng(21)
    shapes = [(48, 80), (65,), (100, 20), (30, 30)]
    kw = dict(momentum=0.9, whiten_grad=whiten_grad, update_preconditioner_first=update_first,
              preconditioner_update_probability=0.5, preconditioner_max_skew=float("inf"),
              preconditioner_init_scale=0.7, lr_params=1e-2)
    p0 = [rng.standard_normal(s, dtype=np.float32) for s in shapes]
    ora = O.KronWhitenOracle(p0, dtype=np.float64, **kw)
    params = [torch.nn.Parameter(torch.from_numpy(p.copy()).to(cuda)) for p in p0]
    opt = KronWhiten(params, precision="fp32", **kw)
    fired = set()
    for step in range(6):
        G = [(rng.standard_normal(s, dtype=np.float32) * np.float32(0.01)) for s in shapes]
        Gd = [torch.from_numpy(g).to(cuda).to(gdt) for g in G]
        G = [gd.float().cpu().numpy() for gd in Gd]  # the values the device sees
        d = ora.make_draws(rng, G)
        fired.add(d["update"] < 0.5)
        pre = ora.step(G, d)
        opt.step_math(Gd, draws=d)
    torch.cuda.synchronize()
    opt.check_errors()
    assert fired == {True, False}  # both orders of the EMA occurred
    tol = TOL["fp32"] if gdt == torch.float32 else TOL["bf16"]
    st = opt.state_dict()
    for k, ((Qo, _), s) in enumerate(zip(ora.QL, st["state"])):
        for qo, qg in zip(Qo, s["Q"]):
            assert rel(qg.cpu().numpy(), qo) < tol
        assert rel(s["m"].float().cpu().numpy(), ora.ms[k]) < tol
        pg = opt._plan.params[k].pg32.cpu().numpy().reshape(np.shape(pre[k]))
        assert rel(pg, pre[k]) < tol
    assert st["counter_m"] == 6


def test_order4_conv_weight_matches_oracle(cuda):
    """A conv-shaped 128 x 64 x 3 x 3 weight (four dense factors, the 3 x 3 ones included, max_skew = inf) and an
    order-3 parameter with a diagonal mode, in bf16 mode, two steps against the oracle on the same draws."""
    rng = np.random.default_rng(31)
    shapes = [(128, 64, 3, 3), (40, 300, 6)]
    kw = dict(preconditioner_max_skew=float("inf"), preconditioner_max_size=256, preconditioner_init_scale=0.9)
    p0 = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.05) for s in shapes]
    ora = O.KronWhitenOracle(p0, dtype=np.float64, **kw)
    params = [torch.nn.Parameter(torch.from_numpy(p.copy()).to(cuda)) for p in p0]
    opt = KronWhiten(params, precision="bf16", **kw)
    for _ in range(2):
        G = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.01) for s in shapes]
        d = ora.make_draws(rng, G, coins=[1.0, 1.0])
        d["update"] = 0.0
        pre = ora.step(G, d)
        opt.step_math([torch.from_numpy(g).to(cuda) for g in G], draws=d)
    torch.cuda.synchronize()
    opt.check_errors()
    for k, ((Qo, _), s) in enumerate(zip(ora.QL, opt.state_dict()["state"])):
        for qo, qg in zip(Qo, s["Q"]):
            assert rel(qg.cpu().numpy(), qo) < TOL["bf16"]
        pg = opt._plan.params[k].pg32.cpu().numpy().reshape(np.shape(pre[k]))
        assert rel(pg, pre[k]) < TOL["bf16"]
        assert rel(params[k].detach().cpu().numpy(), ora.params[k]) < TOL["bf16"]
