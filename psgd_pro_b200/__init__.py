"""psgd_pro_b200: the PSGD-Kron optimizer step (dlyr3/psgd_pro's KronWhiten) on NVIDIA B200.

KronWhiten keeps the reference's constructor, attributes, step(closure) and step_math(grads); the arithmetic runs
in hand-written sm_100a kernels (libpsgd_b200.so, C ABI in include/psgd_b200.h). psgd_pro_b200.ops offers the
reference's operator plug-in surface (EagerOps-compatible methods and the psgd::* custom ops)."""
from .optimizer import KronWhiten

__all__ = ["KronWhiten"]
