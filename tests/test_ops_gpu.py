"""psgd_pro_b200.ops, the reference's operator plug-in surface (psgd_pro_fast.EagerOps, kernels/ops.py custom ops)
on the tcgen05 GEMM, against fp64 torch products of the same inputs and the CPU oracle's norm bounds."""
import numpy as np
import pytest
import torch

from oracle import psgd_oracle as O
from psgd_pro_b200 import ops

pytestmark = pytest.mark.gpu
TOL = 1e-5  # bf16 hi/lo products with fp32 accumulation


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.fixture
def g():
    return torch.Generator().manual_seed(0)


@pytest.mark.parametrize("shape", [(96, 200), (65, 10), (256, 512), (3, 130), (640, 300)])
def test_syrk_both_orientations(cuda, g, shape):
    X = torch.randn(shape, generator=g).to(cuda)
    for trans in (False, True):
        C = ops.syrk(X, trans, True)
        ref = X.double().T @ X.double() if trans else X.double() @ X.double().T
        assert torch.equal(C, C.T) and rel(C, ref) < TOL
        assert rel(ops.syrk_cublas(X, trans), ref) < TOL
        assert rel(ops.syrk2(X, trans, False), ref) < TOL
        n = C.shape[0]
        P = ops.syrk2p(X, trans)
        assert P.numel() == n * (n + 1) // 2
        i, j = 3 % n, (n - 1)
        assert abs(P[i * n - i * (i - 1) // 2 + j - i].item() - ref[i, j].item()) <= 1e-4 * ref.abs().max().item()
        assert rel(ops.unpack(P, n), ref) < TOL
        # every packed entry (the fast epilogue writes interior tiles, the general one the edges and diagonal)
        iu = torch.triu_indices(n, n)
        assert rel(P.cpu(), ref[iu[0], iu[1]]) < TOL


@pytest.mark.parametrize("n,p", [(128, 64), (65, 33), (300, 7)])
def test_symm_reads_only_the_upper_triangle(cuda, g, n, p):
    A = torch.randn(n, n, generator=g)
    S = (A + A.T).to(cuda)
    X = torch.randn(n, p, generator=g).to(cuda)
    tri = S.clone()
    tri[torch.ones(n, n, dtype=torch.bool, device=cuda).tril(-1)] = float("nan")  # kernels/ops.py:190 poisoning
    ref = S.double() @ X.double()
    assert rel(ops.symm(tri, X), ref) < TOL
    assert rel(ops.symm_right(X.T.contiguous(), tri), (X.double().T @ S.double())) < TOL
    iu = torch.triu_indices(n, n, device=cuda)
    assert rel(ops.symm(S[iu[0], iu[1]].contiguous(), X), ref) < TOL  # packed storage


@pytest.mark.parametrize("sign", [1, -1])
def test_tri_vmm_and_rownorm(cuda, g, sign):
    n = 192
    A = torch.randn(n, n, generator=g)
    full = (A + A.T) if sign > 0 else (A - A.T)
    tri = full.clone()
    tri[torch.ones(n, n, dtype=torch.bool).tril(-1)] = float("nan")
    V = torch.randn(32, n, generator=g)
    W = ops.tri_vmm(V.to(cuda), tri.to(cuda), sign)
    assert rel(W, V.double() @ full.double()) < TOL
    r, m = ops.tri_rownorm2((A + A.T).triu().to(cuda))
    S = (A + A.T).double()
    assert rel(r, (S * S).sum(1)) < 1e-6 and abs(m.item() - S.abs().max().item()) < 1e-5


def test_norm_bounds_match_oracle(cuda, g):
    n = 200
    X = torch.randn(n, n + 7, generator=g)
    A = X @ X.T
    B = torch.randn(n, n, generator=g)
    Sk = B - B.T
    V = torch.randn(32, n, generator=g)
    spd = ops.B200Ops.norm_lower_bound_spd(A.to(cuda), V.to(cuda)).item()
    skh = ops.B200Ops.norm_lower_bound_skh(Sk.to(cuda), V.to(cuda)).item()
    assert abs(spd / O.norm_lower_bound_spd(A.double().numpy(), V.numpy()) - 1) < 1e-4
    assert abs(skh / O.norm_lower_bound_skh(Sk.double().numpy(), V.numpy()) - 1) < 1e-4


def test_eager_ops_contract(cuda, g):
    """The EagerOps method set (psgd_pro_fast.py:106-126) on a 2-D step's operands."""
    Ops = ops.make_ops({"k2t", "tri"})
    Pg = torch.randn(64, 96, generator=g).to(cuda)
    q = (torch.eye(64) + 0.01 * torch.randn(64, 64, generator=g)).to(cuda)
    assert rel(Ops.gram(Pg, 0, None), Pg.double() @ Pg.double().T) < TOL
    assert rel(Ops.gram(Pg, 1, None), Pg.double().T @ Pg.double()) < TOL
    assert rel(Ops.gram_q(q), q.double().T @ q.double()) < TOL
    T = Ops.sym(Pg, False)
    assert rel(Ops.symm(T, q), T.double() @ q.double()) < TOL
    assert rel(Ops.symm_r(Pg.T.contiguous(), T), Pg.double().T @ T.double()) < TOL
    assert rel(Ops.syrk(Pg, True), Pg.double().T @ Pg.double()) < TOL
    Pk = ops.make_ops({"packed"}).sym(Pg, False)
    assert Pk.dim() == 1 and rel(ops.unpack(Pk, 64), Pg.double() @ Pg.double().T) < TOL


def poison_lower(M):
    """The square form of kernels/ops.py:190: the lower triangle holds NaN, which no kernel may read."""
    T = M.clone()
    n = T.shape[0]
    T[torch.ones(n, n, dtype=torch.bool, device=T.device).tril(-1)] = float("nan")
    return T


def packed(M):
    n = M.shape[0]
    iu = torch.triu_indices(n, n, device=M.device)
    return M[iu[0], iu[1]].contiguous()


@pytest.mark.parametrize("n", [1, 64, 130, 513])
@pytest.mark.parametrize("sign", [1, -1])
def test_storage_forms_kernels(cuda, g, n, sign):
    """tri_vmm, tri_rownorm2, unpack and the norm bounds from the square-upper and packed forms, lower half
    poisoned; the skew form has a zero diagonal (kernels/k1.cu:41-50)."""
    A = torch.randn(n, n, generator=g)
    full = (A + A.T) if sign > 0 else (A - A.T)
    full = full.to(cuda)
    V = torch.randn(32, n, generator=g).to(cuda)
    for form in (poison_lower(full), packed(full)):
        W = ops.tri_vmm(V, form, sign)
        assert rel(W, V.double() @ full.double()) < TOL
        if sign > 0:
            r, m = ops.tri_rownorm2(form)
            F = full.double()
            assert rel(r, (F * F).sum(1)) < 1e-6 and abs(m.item() - F.abs().max().item()) <= 1e-6 * F.abs().max().item()
    assert torch.equal(ops.unpack(packed(full), n).cpu(), full.cpu()) if sign > 0 else True
    if n >= 2:
        bound = (ops.norm_lower_bound_spd if sign > 0 else ops.norm_lower_bound_skh)
        ora = (O.norm_lower_bound_spd if sign > 0 else O.norm_lower_bound_skh)
        M = full @ full.T if sign > 0 else full  # an spd matrix for the spd bound
        want = ora(M.double().cpu().numpy(), V.cpu().numpy())
        got_sq = bound(poison_lower(M), V).item()
        got_pk = bound(packed(M), V).item()
        assert abs(got_sq / want - 1) < 1e-4 and abs(got_pk / want - 1) < 1e-4
    ops.check_errors()


@pytest.mark.parametrize("n,p", [(128, 64), (300, 7), (1024, 512)])
def test_trmm_skips_the_zero_triangle(cuda, g, n, p):
    """triu(T) @ X (the triangular-times-dense product of the benchmark plan; oracle torch.triu(T) @ X in fp64)
    with the lower triangle of T poisoned: it is neither read nor multiplied."""
    T = torch.randn(n, n, generator=g) / n ** 0.5 + torch.eye(n)
    X = torch.randn(n, p, generator=g)
    ref = torch.triu(T).double() @ X.double()
    C = ops.trmm_impl(poison_lower(T.to(cuda)), X.to(cuda))
    assert rel(C, ref) < TOL
    ops.check_errors()
