"""Parity of the benchmarked path itself: the factor sizes of the Llama-style set (2048, 256, 5632), a 1-D 2048
parameter and a 32000 x 2048 embedding whose 32000 dim is diagonal (the 16-range diagonal-factor kernel), bf16
gradients, three steps with the init scale taken on the fly, against golden values produced by the reference
itself (tests/golden/llama_block_bf16.npz, written by tests/golden/make_golden.py with the same parameters,
gradients and random draws).

The reference ran in fp32 on the bf16 gradient values; its matrices are stored as two-sided Gaussian sketches
(tests/golden/sketch.py), whose relative error estimates the relative Frobenius error of the whole matrix.

  * bf16 run (what bench.py times): bf16 parameters and gradients, precision="bf16" (one bf16 MMA per product,
    fp32 accumulation, fp32 Q), the groups with long reductions on the tcgen05 pair kernel. Q, L and the
    preconditioned gradient must match the reference within 2e-2. The parameter update is checked step by step
    against the reference's clip-and-apply arithmetic (psgd_pro.py:371-381, fp32 torch) on the B200's own
    preconditioned gradient: a bf16 parameter of magnitude ~1 has an ulp of 2^-7, larger than one update, so its
    stored change carries bf16 rounding that the fp32 reference run does not have.
  * fp32 run: fp32 parameters and the same gradient values as fp32 tensors, precision="fp32" (three-MMA split),
    the reference's exact configuration: Q, L, Pg and the parameter change within 1e-3."""
import numpy as np
import pytest
import torch

from psgd_pro_b200 import KronWhiten
from scenario_util import Scenario, factor_layout, rel

import os
import sys
sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from sketch import sketch  # noqa: E402

pytestmark = pytest.mark.gpu

NAME = "llama_block_bf16"
PAIR = 8  # the group flag of the pair kernel (include/psgd_b200.h, psgd_gemm_encode)


def reference_apply(p_prev, pg, lr, max_avg, max_elem):
    """psgd_pro.py:371-381 in fp32 torch, the parameter updated in fp32 and stored in its own dtype."""
    g = pg.clone()
    avg = torch.sqrt(torch.mean(g * g))
    if avg > max_avg:
        g *= max_avg / avg
    g.clamp_(min=-max_elem, max=max_elem)
    return (p_prev.float() - lr * g.reshape(p_prev.shape)).to(p_prev.dtype)


def run(cuda, precision):
    sc = Scenario(NAME)
    kw = sc.meta["kw"]
    layout = factor_layout(sc.meta["shapes"], kw["preconditioner_max_size"], kw["preconditioner_max_skew"])
    pdt = torch.bfloat16 if precision == "bf16" else torch.float32
    params = [torch.nn.Parameter(torch.from_numpy(p).to(cuda).to(pdt)) for p in sc.params]
    p0 = [p.detach().clone() for p in params]
    opt = KronWhiten(params, precision=precision, **kw)
    for step in range(1, sc.meta["steps"] + 1):
        G = sc.grads()
        draws = sc.draws(step, layout, G)
        prev = [p.detach().clone() for p in params]
        opt.step_math([torch.from_numpy(g).to(cuda).to(pdt) for g in G], draws=draws)
        torch.cuda.synchronize()
        opt.check_errors()
        for k, (p, pr, pp) in enumerate(zip(params, prev, opt._plan.params)):
            exp = reference_apply(pr, pp.pg32, opt.lr_params, *opt.grad_clip_max_amps).float()
            got, before = p.detach().float(), pr.float()
            # the stored results may differ by the rounding of the stored value (the two fp32 sums can straddle a
            # rounding boundary of the parameter dtype) plus a tiny share of the update (the clip scale's sum of
            # squares is reduced in another order)
            eps = torch.finfo(pdt).eps
            bound = 2 * eps * torch.maximum(before.abs(), exp.abs()) + 1e-5 * (exp - before).abs() + 1e-30
            assert bool(((got - exp).abs() <= bound).all()), (step, k)
    return sc, opt, params, p0


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_benchmarked_path_matches_reference(cuda, precision):
    sc, opt, params, p0 = run(cuda, precision)
    tol = 2e-2 if precision == "bf16" else 1e-3
    if precision == "bf16":
        # the long-reduction product groups run on the CTA-pair kernel, as in the benchmark (the one-row products of
        # the 1-D parameter form groups of their own, u1_r1 / a1_r1 / term1_r1, on the one-CTA kernel)
        kinds = {name: g.kind for name, g in opt._plan.phase_groups() if g is not None}
        for name in ("u1", "u2", "term1", "qupdate", "S", "procrustes", "gram", "a1", "a2"):
            assert kinds[name] & PAIR, (name, kinds[name])
        for name in ("u1_r1", "a1_r1"):
            assert not kinds[name] & PAIR, (name, kinds[name])
    st = opt.state_dict()["state"]
    errs = {}
    for k, s in enumerate(st):
        for i, q in enumerate(s["Q"]):
            e = rel(sketch(q.detach().double().cpu().numpy()), sc.g[f"Q_{k}_{i}"])
            errs[f"Q_{k}_{i}"] = e
            lg, lr_ = float(s["L"][i]), float(sc.g[f"L_{k}_{i}"])
            assert abs(lg - lr_) <= tol * abs(lr_), (k, i, lg, lr_)
        pg = opt._plan.params[k].pg32.detach().double().cpu().numpy().reshape(sc.meta["shapes"][k])
        errs[f"pre_{k}"] = rel(sketch(pg), sc.g[f"pre_{k}"])
        if precision == "fp32":
            d = params[k].detach().double().cpu().numpy() - sc.params[k].astype(np.float64)
            errs[f"dparam_{k}"] = rel(sketch(d), sc.g[f"dparam_{k}"])
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, (precision, bad, errs)
