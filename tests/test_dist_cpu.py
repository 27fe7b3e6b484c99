"""The multi-rank step (psgd_pro_b200.dist.ShardedKronWhiten) on CPU with the gloo backend, world size 2: each
rank runs the optimizer for the parameters the FLOP-balanced assignment gives it (here the CPU oracle stands in
for the GPU optimizer), and after the all-gather every rank holds exactly the parameters of a one-process run."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import psgd_oracle as O
from psgd_pro_b200.dist import ShardedKronWhiten, assignment_for, falg, lpt_assign, make_flat_params

SHAPES = [(48, 80), (10, 65), (65,), (30, 30), (7, 40), (100, 20)]
KW = dict(preconditioner_max_skew=float("inf"), preconditioner_init_scale=0.5, lr_params=0.01)


class OracleOptimizer:
    """CPU stand-in with KronWhiten's step_math(grads, draws): the oracle step, written back into the torch
    parameters (which may be views of a flat buffer)."""

    def __init__(self, params, **kw):
        self.params = params
        self.o = O.KronWhitenOracle([p.detach().numpy().copy() for p in params], dtype=np.float64, **kw)

    def set_init_scale(self, scale):
        self.o.QL = [O.init_kron(np.squeeze(p).shape, scale, self.o.max_size, self.o.max_skew, self.o.dtype)
                     for p in self.o.params]

    def step_math(self, grads, draws=None):
        self.o.step([g.numpy() for g in grads], draws)
        for p, new in zip(self.params, self.o.params):
            p.data.copy_(torch.from_numpy(np.asarray(new, dtype=np.float32)).reshape(p.shape))


KW_ONTHEFLY = dict(KW, preconditioner_init_scale=None)


def make_inputs(steps=3, kw=KW):
    rng = np.random.default_rng(0)
    p0 = [rng.standard_normal(s).astype(np.float32) for s in SHAPES]
    # gradient scales differ per parameter, so the on-the-fly init scale (a max over all gradients) depends on
    # which rank sees which gradient unless every rank takes the max over all of them
    G = [[(rng.standard_normal(s) * 0.02 * (1 + k)).astype(np.float32) for k, s in enumerate(SHAPES)]
         for _ in range(steps)]
    ora = O.KronWhitenOracle(p0, dtype=np.float64, **kw)
    D = [ora.make_draws(rng, g, coins=[1.0] * len(SHAPES)) for g in G]
    for d in D:
        d["update"] = 0.0
    return p0, G, D


def single_process_result(kw=KW):
    p0, G, D = make_inputs(kw=kw)
    ora = O.KronWhitenOracle(p0, dtype=np.float64, **kw)
    for g, d in zip(G, D):
        ora.step(g, d)
    return [np.asarray(p, dtype=np.float32) for p in ora.params]


def worker(rank, world, port, flat, out, kw=KW, buckets=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p0, G, D = make_inputs(kw=kw)
        owner = assignment_for(SHAPES, world, max_skew=float("inf"))
        if flat:
            it = iter(p0)
            params, buf, layout = make_flat_params(SHAPES, owner, world, torch.float32, "cpu",
                                                   init=lambda s: torch.from_numpy(next(it)), buckets=buckets,
                                                   max_skew=float("inf"))
            opt = ShardedKronWhiten(params, assignment=owner, flat=(buf, layout), optimizer_factory=OracleOptimizer,
                                    **kw)
        else:
            params = [torch.nn.Parameter(torch.from_numpy(p.copy())) for p in p0]
            opt = ShardedKronWhiten(params, assignment=owner, optimizer_factory=OracleOptimizer, buckets=buckets,
                                    **kw)
        assert 1 <= opt.nbuckets <= buckets
        for g, d in zip(G, D):
            opt.step_math([torch.from_numpy(x) for x in g], draws=d)
        out[rank] = [p.detach().numpy().copy() for p in params]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("flat,onthefly,buckets", [(False, False, 1), (True, False, 1), (True, True, 1),
                                                    (True, False, 3), (False, True, 2)])
def test_sharded_step_matches_one_process(flat, onthefly, buckets):
    """onthefly: no preconditioner_init_scale, so the first step sets it from max_i mean|g_i|^4 over every
    parameter's gradient (psgd_pro.py:329-332), on every rank alike. buckets: each rank's parameters stepped and
    all-gathered in that many buckets."""
    kw = KW_ONTHEFLY if onthefly else KW
    ref = single_process_result(kw)
    mgr = mp.Manager()
    out = mgr.dict()
    port = 29500 + (os.getpid() % 400) + (7 if flat else 0) + (13 if onthefly else 0) + 31 * buckets
    mp.spawn(worker, args=(2, port, flat, out, kw, buckets), nprocs=2, join=True)
    for r in range(2):
        for a, b in zip(out[r], ref):
            np.testing.assert_array_equal(a, b)


def rs_worker(rank, world, port, out, buckets):
    """reduce_scatter mode: rank r passes local gradients w_r * g with w = (4, -2), whose average over the two
    ranks is g exactly (sums of powers of two): every rank must end with the one-process result for g."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p0, G, D = make_inputs(kw=KW_ONTHEFLY)
        owner = assignment_for(SHAPES, world, max_skew=float("inf"))
        it = iter(p0)
        params, buf, layout = make_flat_params(SHAPES, owner, world, torch.float32, "cpu",
                                               init=lambda s: torch.from_numpy(next(it)), buckets=buckets,
                                               max_skew=float("inf"))
        opt = ShardedKronWhiten(params, assignment=owner, flat=(buf, layout), optimizer_factory=OracleOptimizer,
                                reduce_scatter=True, **KW_ONTHEFLY)
        w = 4.0 if rank == 0 else -2.0
        for step, (g, d) in enumerate(zip(G, D)):
            local = [torch.from_numpy(x) * w for x in g]
            if step == 1:  # the loop may also write straight into the optimizer's gradient buffer
                views = opt.local_grads()
                for v, x in zip(views, local):
                    v.copy_(x)
                local = views
            opt.step_math(local, draws=d)
        out[rank] = [p.detach().numpy().copy() for p in params]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("buckets", [1, 3])
def test_reduce_scatter_fused_into_the_sharded_step(buckets):
    ref = single_process_result(KW_ONTHEFLY)
    mgr = mp.Manager()
    out = mgr.dict()
    port = 29700 + (os.getpid() % 200) + buckets
    mp.spawn(rs_worker, args=(2, port, out, buckets), nprocs=2, join=True)
    for r in range(2):
        for a, b in zip(out[r], ref):
            np.testing.assert_array_equal(a, b)


def test_lpt_balance_and_determinism():
    costs = [falg(s, max_skew=float("inf")) for s in SHAPES]
    own = lpt_assign(costs, 4)
    assert own == lpt_assign(costs, 4)
    loads = [sum(c for c, o in zip(costs, own) if o == r) for r in range(4)]
    assert max(loads) <= max(costs) + sum(costs) / 4  # the LPT bound
    # the Llama-style set splits within a few percent across 8 ranks
    from psgd_pro_b200.workloads import llama_1b
    shp = [tuple(x for x in s if x != 1) for s in llama_1b()]
    c = [falg(s, 8192, float("inf")) for s in shp]
    own = lpt_assign(c, 8)
    loads = [sum(x for x, o in zip(c, own) if o == r) for r in range(8)]
    assert max(loads) / (sum(c) / 8) < 1.05
