"""The plug-in module imports on a host without a GPU and registers the reference's custom op names with fake
(meta) implementations, so tracing callers see the right output shapes."""
import torch

from psgd_pro_b200 import ops


def test_custom_ops_registered_with_fake_shapes():
    ns = getattr(torch.ops, ops.NS)
    for name in ("tri_vmm", "tri_rownorm2", "symm", "symm_right", "syrk_cublas", "syrk", "syrk2", "syrk2p", "unpack"):
        assert hasattr(ns, name), name
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        A = torch.empty(10, 7)
        assert ns.syrk(A, True, True).shape == (7, 7)
        assert ns.syrk2p(A, False).shape == (55,)
        assert ns.unpack(torch.empty(55), 10).shape == (10, 10)
        assert ns.symm(torch.empty(10, 10), torch.empty(10, 3)).shape == (10, 3)
        assert ns.symm_right(torch.empty(4, 10), torch.empty(55)).shape == (4, 10)
        assert ns.tri_vmm(torch.empty(32, 10), torch.empty(10, 10), 1).shape == (32, 10)


def test_make_ops_surface():
    O = ops.make_ops({"k1", "k2t", "tri", "nan"})
    for m in ("gram", "gram_q", "norm_lower_bound_spd", "norm_lower_bound_skh", "symm", "symm_r", "syrk", "sym"):
        assert callable(getattr(O, m))
    assert "b200" in O.flags and ops.side(torch.empty(55)) == 10


def test_kronwhiten_accepts_the_fast_class_keywords():
    """psgd_pro_fast.KronWhiten's constructor (psgd_pro_fast.py:245-264) takes these keywords beyond psgd_pro's;
    callers that pass them must drop in unchanged."""
    import inspect
    from psgd_pro_b200 import KronWhiten
    sig = inspect.signature(KronWhiten.__init__).parameters
    fast_kw = dict(preconditioner_max_size=float("inf"), preconditioner_max_skew=1.0, preconditioner_init_scale=None,
                   lr_params=0.001, lr_preconditioner=0.1, betaL=0.9, damping=1e-9, momentum=0.0,
                   grad_clip_max_amps=(2.0, 10.0), preconditioner_update_probability=1.0,
                   update_preconditioner_first=True, whiten_grad=True, compile=None, batch=False, cache_p=False,
                   graph_rng=False, p2d=False, r2=False)
    for k, v in fast_kw.items():
        assert k in sig, k
        assert sig[k].default == v, (k, sig[k].default, v)
    assert "ops" in sig
