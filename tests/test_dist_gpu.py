"""The sharded step on two B200s over NCCL (psgd_pro_b200.dist.ShardedKronWhiten with the real GPU optimizer, with
and without the fused gradient reduce-scatter),
against the same step run whole on one GPU: identical parameters and random draws (reference order, supplied),
bf16 parameters and gradients, the init scale taken on the fly from every parameter's gradient; after the
all-gather every rank must hold, bit for bit, the parameters of the one-GPU run, and each rank's Q factors must
equal the one-GPU run's factors of the parameters it owns. Skipped with fewer than two GPUs."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from scenario_util import factor_layout, reference_order_draws

pytestmark = pytest.mark.gpu

SHAPES = [(2048, 2048), (256, 2048), (2048,), (3000, 512), (48, 80), (65,), (4096, 64)]
KW = dict(preconditioner_max_size=8192, preconditioner_max_skew=float("inf"), precision="bf16")
STEPS = 2


def inputs():
    rng = np.random.default_rng(11)
    p0 = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.02) for s in SHAPES]
    G = [[rng.standard_normal(s, dtype=np.float32) * np.float32(1e-3 * (1 + k)) for k, s in enumerate(SHAPES)]
         for _ in range(STEPS)]
    layout = factor_layout(SHAPES, KW["preconditioner_max_size"], KW["preconditioner_max_skew"])
    drng = np.random.default_rng(12)
    D = [reference_order_draws(drng, layout, SHAPES, 1.0, []) for _ in range(STEPS)]
    return p0, G, D


def to_dev(x, dev):
    return torch.from_numpy(x).to(dev).to(torch.bfloat16)


def one_gpu(dev):
    from psgd_pro_b200 import KronWhiten
    p0, G, D = inputs()
    params = [torch.nn.Parameter(to_dev(p, dev)) for p in p0]
    opt = KronWhiten(params, **KW)
    for g, d in zip(G, D):
        opt.step_math([to_dev(x, dev) for x in g], draws=d)
    torch.cuda.synchronize()
    opt.check_errors()
    return [p.detach().float().cpu() for p in params], [[q.cpu() for q in s["Q"]] for s in opt.state_dict()["state"]]


def worker(rank, world, port, outdir, rs=False):
    import torch.distributed as dist
    from datetime import timedelta
    from psgd_pro_b200.dist import ShardedKronWhiten, assignment_for, make_flat_params
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        p0, G, D = inputs()
        owner = assignment_for([tuple(x for x in s if x != 1) for s in SHAPES], world, KW["preconditioner_max_size"],
                               KW["preconditioner_max_skew"])
        it = iter(p0)
        params, flat, seg = make_flat_params(SHAPES, owner, world, torch.bfloat16, dev,
                                             init=lambda s: to_dev(next(it), dev))
        opt = ShardedKronWhiten(params, assignment=owner, flat=(flat, seg), reduce_scatter=rs, **KW)
        w = (4.0 if rank == 0 else -2.0) if rs else 1.0  # local gradients whose average is the gradient exactly
        for g, d in zip(G, D):
            opt.step_math([to_dev(x, dev) * w for x in g], draws=d)
        torch.cuda.synchronize()
        if opt.inner is not None:
            opt.inner.check_errors()
        Q = {}
        if opt.inner is not None:
            for i, s in zip(opt.owned, opt.inner.state_dict()["state"]):
                Q[i] = [q.cpu() for q in s["Q"]]
        torch.save({"params": [p.detach().float().cpu() for p in params], "Q": Q, "owner": owner},
                   os.path.join(outdir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rs", [False, True])
def test_two_gpu_sharded_step_equals_one_gpu_step(cuda, rs):
    """rs: the ranks pass local gradients (4 g and -2 g) and the step reduce-scatters them itself (average g)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ref_p, ref_q = one_gpu(cuda)
    with tempfile.TemporaryDirectory() as d:
        port = 29600 + os.getpid() % 300 + (7 if rs else 0)
        mp.spawn(worker, args=(2, port, d, rs), nprocs=2, join=True)
        outs = [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(2)]
    owner = outs[0]["owner"]
    assert sorted(set(owner)) == [0, 1]  # both ranks own parameters
    for r, o in enumerate(outs):
        for k, (a, b) in enumerate(zip(o["params"], ref_p)):
            assert torch.equal(a, b), (r, k, (a - b).abs().max().item())
        for i, qs in o["Q"].items():
            assert owner[i] == r
            for qa, qb in zip(qs, ref_q[i]):
                assert torch.equal(qa, qb), (r, i)
