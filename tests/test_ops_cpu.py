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
