"""Failure reporting on the device, tested without faulting, trapping or hanging the GPU:

  * the bounded wait runs out: psgd_wait_probe makes one thread wait, with the helper every GEMM wait uses, on a
    barrier that nothing arrives at; after its limit (here 1 ms) the error bit reaches the caller's device error
    word, and the next launches on the same device run normally;
  * the GEMM wait limit is host-settable (psgd_set_wait_limit_ns, default 2 s) and normal work stays well inside a
    shorter one;
  * a non-finite preconditioner (a NaN gradient makes term1, its norm bound and L NaN) raises
    PSGD_ERR_NONFINITE, which KronWhiten.check_errors reports, instead of going unnoticed."""
import pytest
import torch

from psgd_pro_b200 import KronWhiten, _capi, ops
from psgd_pro_b200 import kernels as K

pytestmark = pytest.mark.gpu


def test_wait_probe_runs_out_and_the_context_stays_usable(cuda):
    lib = _capi.lib()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert lib.psgd_wait_probe(err.data_ptr(), 1_000_000, K.stream_handle()) == 0
    torch.cuda.synchronize()
    assert int(err.item()) & 1, int(err.item())
    assert lib.psgd_wait_probe(err.data_ptr(), 0, K.stream_handle()) == _capi.c_int(-1).value  # no endless wait
    # the device still runs work: a product through the plug-in surface, checked against torch
    X = torch.randn(300, 200, device=cuda)
    C = ops.syrk_impl(X, False)
    ref = X.double() @ X.double().T
    assert ((C.double() - ref).norm() / ref.norm()).item() < 1e-5
    ops.check_errors()


def test_gemm_wait_limit_is_settable(cuda):
    lib = _capi.lib()
    old = lib.psgd_set_wait_limit_ns(200_000_000)  # 200 ms: far above any legitimate wait
    try:
        assert old == 2_000_000_000
        n = 2048
        A = torch.randn(n, n, device=cuda).to(torch.bfloat16)
        P = torch.empty(n * (n + 1) // 2, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        spec = K.make_spec((A, None), (A, None), n, n, n, bn=256, mode=K.PSGD_GEMM_SYRK, out_packed=P)
        g = K.GemmGroup([spec], 1, cuda)
        for _ in range(3):
            g.launch(err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        ref = (A.double() @ A.double().T)
        iu = torch.triu_indices(n, n, device=cuda)
        assert ((P.double() - ref[iu[0], iu[1]]).norm() / ref.norm()).item() < 1e-2
    finally:
        assert lib.psgd_set_wait_limit_ns(0) == 200_000_000  # 0 restores the default
    assert lib.psgd_set_wait_limit_ns(0) == 2_000_000_000


def test_nonfinite_factor_is_flagged(cuda):
    params = [torch.nn.Parameter(torch.randn(64, 96, device=cuda)), torch.nn.Parameter(torch.randn(40, device=cuda))]
    opt = KronWhiten(params, preconditioner_init_scale=1.0, preconditioner_max_skew=float("inf"), cuda_graphs=False)
    g = [torch.randn(64, 96, device=cuda) * 0.01, torch.randn(40, device=cuda) * 0.01]
    opt.step_math(g)
    opt.check_errors()  # a finite step reports nothing
    g[0][3, 5] = float("nan")
    opt.step_math(g)
    with pytest.raises(RuntimeError, match="NaN or infinite"):
        opt.check_errors()
    opt.clear_errors()
    opt.check_errors()
