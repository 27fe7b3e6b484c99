"""The reference's operator plug-in surface on B200 (psgd_pro_fast.py:106-126 EagerOps; kernels/ops.py:24-215).

B200Ops has the EagerOps method set (gram, gram_q, norm_lower_bound_spd / _skh, symm, symm_r, syrk, sym, flags),
so psgd_pro_fast.KronWhiten(ops=B200Ops) or make_ops(flags) callers keep working; the same contracts are also
registered as torch custom ops under the reference's names (psgd::tri_vmm, psgd::tri_rownorm2, psgd::symm,
psgd::symm_right, psgd::syrk_cublas, psgd::syrk, psgd::syrk2, psgd::syrk2p, psgd::unpack), each with a fake
implementation for tracing. When the reference's own kernels module has registered those names already, this
module registers under psgd_b200:: instead.

Every product runs in the tcgen05 GEMM of libpsgd_b200.so with bf16 hi/lo operands (three MMAs, fp32
accumulation; about 1e-6 relative to fp64 on random inputs), on the current stream. Inputs are fp32 CUDA tensors
as in the reference (kernels/k1.cu:275-278, kernels/blas.cpp:22); symmetric matrices may be given full, as an upper
triangle in a square (the lower triangle is never read, NaN allowed: kernels/ops.py:9) or packed (the row-major
upper triangle, element (i, j), i <= j, at i n - i (i - 1) / 2 + j - i: kernels/k2.py:78)."""
import torch
from torch import Tensor

from . import kernels as K

_KEEP = []  # staging buffers of the last calls (released once the stream has moved past them)


def _check(t, name):
    if not (t.is_cuda and t.dtype == torch.float32):
        raise RuntimeError(f"psgd_pro_b200.ops: {name} must be an fp32 CUDA tensor")


def side(S):
    """n of a symmetric matrix in storage form (square, or packed with n(n+1)/2 values); kernels/ops.py:119-121."""
    return S.shape[0] if S.dim() == 2 else int(((8 * S.shape[0] + 1) ** 0.5 - 1) / 2)


def _full(S, sign=1):
    """Full symmetric (sign 1) or skew-symmetric (sign -1) matrix from a storage form; only the upper triangle
    of a square input is read."""
    if S.dim() == 1:
        return unpack_impl(S, side(S), sign)
    up = torch.triu(S)
    low = torch.triu(S, 1).T
    return up + sign * low if sign > 0 else torch.triu(S, 1) - low


def _gemm(a_op, b_op, M, N, Kd, alpha=1.0, **out):
    """D = alpha * A B^T into fp32 outputs (out_f32=...)."""
    err = torch.zeros(1, dtype=torch.int32, device=out["out_f32"].device)
    spec = K.make_spec(a_op, b_op, M, N, Kd, bn=K_choose(N), alpha=alpha, **out)
    K.gemm(spec, 3, err)
    _KEEP.append((a_op, b_op, err))
    del _KEEP[:-8]


def K_choose(N):
    best = None
    for b in (128, 64, 32, 16):
        waste = -(-N // b) * b - N
        if best is None or waste < best[0]:
            best = (waste, b)
    return best[1]


def _op(X, transpose=False):
    op, keep = K.to_operand(X, transpose=transpose, split=True)
    _KEEP.append(keep)
    return op


# ---- the products ---------------------------------------------------------------------------------------------------
def syrk_impl(X, trans):
    """Full symmetric X^T X (trans) or X X^T, computed on the upper tiles only and mirrored (exactly symmetric)."""
    _check(X, "X")
    A = _op(X, transpose=trans)
    n, Kd = (X.shape[1], X.shape[0]) if trans else (X.shape[0], X.shape[1])
    C = torch.empty(n, n, device=X.device)
    err = torch.zeros(1, dtype=torch.int32, device=X.device)
    K.gemm(K.make_spec(A, A, n, n, Kd, bn=128, mode=K.PSGD_GEMM_SYRK, out_f32=C), 3, err)
    _KEEP.append((A, err))
    return C


def symm_impl(S, X):
    """S @ X with S symmetric in storage form (kernels/blas.cpp:35-49 cublasSsymm, side left)."""
    _check(X, "X")
    Sf = _full(S)
    n, p = X.shape
    C = torch.empty(n, p, device=X.device)
    _gemm(_op(Sf), _op(X, transpose=True), n, p, n, out_f32=C)
    return C


def symm_right_impl(X, S):
    """X @ S with S symmetric in storage form (kernels/blas.cpp:51-65, side right)."""
    _check(X, "X")
    Sf = _full(S)
    m, n = X.shape
    C = torch.empty(m, n, device=X.device)
    _gemm(_op(X), _op(Sf), m, n, n, out_f32=C)
    return C


def tri_vmm_impl(V, A, sign):
    """W = V @ A_sym for a symmetric (sign 1) or skew-symmetric (sign -1) A read from its upper triangle; the
    skew diagonal is taken as zero (kernels/k1.cu:1-3, :31-53)."""
    _check(V, "V")
    _check(A, "A")
    Af = _full(A, sign)
    m, n = V.shape
    W = torch.empty(m, n, device=V.device)
    # W[v, c] = sum_k V[v, k] A[k, c] = sum_k V[v, k] (sign A[c, k]): B operand = A itself, alpha = sign
    _gemm(_op(V), _op(Af), m, n, n, alpha=float(sign), out_f32=W)
    return W


def tri_rownorm2_impl(A):
    """(squared row norms, max |A_ij|) of the symmetric matrix held in the upper triangle (kernels/k1.cu:296-307)."""
    _check(A, "A")
    Af = _full(A)
    return (Af * Af).sum(1), Af.abs().amax()


def syrk_packed_impl(X, trans):
    """Row-major packed upper triangle of X^T X (trans) or X X^T, n(n+1)/2 values (kernels/k2.py:78-80)."""
    C = syrk_impl(X, trans)
    n = C.shape[0]
    iu = torch.triu_indices(n, n, device=C.device)
    return C[iu[0], iu[1]].contiguous()


def unpack_impl(Pk, n, sign=1):
    """Full symmetric n x n matrix from its row-major packed upper triangle (kernels/k2.py:88-103)."""
    iu = torch.triu_indices(n, n, device=Pk.device)
    C = torch.zeros(n, n, device=Pk.device, dtype=Pk.dtype)
    C[iu[0], iu[1]] = Pk
    low = torch.triu(C, 1).T
    return C + sign * low


def _norm_lower_bound(A, nf, V, sign, half_iters=2):
    """The subspace iteration of psgd_pro.py:19-41 with the random start V given (psgd_pro_fast.py:32-43); the
    products V A run on the tensor cores."""
    sn = torch.finfo(torch.float32).smallest_normal
    j = torch.argmax((A * A).sum(1))
    Aj = A.index_select(0, j.view(1)) / nf
    V = Aj + torch.sgn(torch.sum(Aj * V, dim=1, keepdim=True)) * V
    for _ in range(half_iters):
        V = tri_vmm_impl(V.contiguous(), A, sign) / nf
        V = V / (torch.linalg.vector_norm(V, dim=1, keepdim=True) + sn)
        V = tri_vmm_impl(V.contiguous(), A, sign) / nf
    return nf * torch.amax(torch.linalg.vector_norm(V, dim=1))


def norm_lower_bound_spd(A, V):
    """psgd_pro_fast.py:46-47 (A in storage form)."""
    Af = _full(A)  # exact for a full symmetric input; reads only the upper triangle of a triangle-stored one
    return _norm_lower_bound(Af, Af.diagonal().amax() + torch.finfo(torch.float32).smallest_normal, V, 1)


def norm_lower_bound_skh(A, V):
    """psgd_pro_fast.py:50-51 (A a full skew-symmetric matrix, as R = Q^T - Q)."""
    return _norm_lower_bound(A, A.abs().amax() + torch.finfo(torch.float32).smallest_normal, V, -1)


class B200Ops:
    """psgd_pro_fast.EagerOps (psgd_pro_fast.py:106-126) with the dense products on B200."""
    flags = frozenset({"b200"})

    @staticmethod
    def gram(Pg, i, expr):
        """term1 of factor i of a 2-D Pg (Pg Pg^T for i = 0, Pg^T Pg for i = 1); other orders use expr."""
        if Pg.dim() != 2:
            return expr(Pg, Pg)
        return syrk_impl(Pg.contiguous(), i == 1)

    @staticmethod
    def gram_q(q):
        return syrk_impl(q.contiguous(), True)

    norm_lower_bound_spd = staticmethod(norm_lower_bound_spd)
    norm_lower_bound_skh = staticmethod(norm_lower_bound_skh)

    @staticmethod
    def symm(A, q):
        return symm_impl(A, q.contiguous())

    @staticmethod
    def syrk(X, trans):
        return syrk_impl(X.contiguous(), trans)

    sym = syrk

    @staticmethod
    def symm_r(X, S):
        return symm_right_impl(X.contiguous(), S)


def make_ops(flags=()):
    """kernels/ops.py:142-215 compatibility: every flag combination maps to the B200 kernels (there is no size
    crossover: the tensor-core products serve every shape). "packed" keeps term1 and P as packed triangles."""
    flags = frozenset(flags)

    class Ops(B200Ops):
        pass

    if "packed" in flags:
        Ops.sym = staticmethod(lambda X, trans: syrk_packed_impl(X.contiguous(), trans))
    Ops.flags = flags | {"b200"}
    return Ops


# ---- custom ops under the reference's names ----------------------------------------------------------------------
def _namespace():
    try:
        torch.library.Library("psgd", "FRAGMENT")  # probe: does someone else own psgd::tri_vmm already?
        if hasattr(torch.ops, "psgd") and hasattr(torch.ops.psgd, "tri_vmm"):
            return "psgd_b200"
    except Exception:
        return "psgd_b200"
    return "psgd"


NS = _namespace()


@torch.library.custom_op(f"{NS}::tri_vmm", mutates_args=())
def tri_vmm(V: Tensor, A: Tensor, sign: int) -> Tensor:
    return tri_vmm_impl(V.contiguous(), A, sign)


@tri_vmm.register_fake
def _(V, A, sign):
    return V.new_empty(V.shape)


@torch.library.custom_op(f"{NS}::tri_rownorm2", mutates_args=())
def tri_rownorm2(A: Tensor) -> tuple[Tensor, Tensor]:
    r, m = tri_rownorm2_impl(A)
    return r, m.clone()


@tri_rownorm2.register_fake
def _(A):
    return A.new_empty(A.shape[0]), A.new_empty(())


@torch.library.custom_op(f"{NS}::symm", mutates_args=())
def symm(S: Tensor, B: Tensor) -> Tensor:
    return symm_impl(S, B.contiguous())


@symm.register_fake
def _(S, B):
    return B.new_empty(side(S), B.shape[1])


@torch.library.custom_op(f"{NS}::symm_right", mutates_args=())
def symm_right(B: Tensor, S: Tensor) -> Tensor:
    return symm_right_impl(B.contiguous(), S)


@symm_right.register_fake
def _(B, S):
    return B.new_empty(B.shape[0], side(S))


@torch.library.custom_op(f"{NS}::syrk_cublas", mutates_args=())
def syrk_cublas(A: Tensor, trans: bool) -> Tensor:
    """Name kept from kernels/ops.py:55-63 (there a cuBLAS call); the result holds both triangles."""
    return syrk_impl(A.contiguous(), trans)


@syrk_cublas.register_fake
def _(A, trans):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n, n)


@torch.library.custom_op(f"{NS}::syrk", mutates_args=())
def syrk(A: Tensor, trans: bool, mirror: bool) -> Tensor:
    """kernels/ops.py:66-75; the output is always mirrored (a valid answer for mirror = False as well: the
    contract there leaves the lower triangle unspecified)."""
    return syrk_impl(A.contiguous(), trans)


@syrk.register_fake
def _(A, trans, mirror):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n, n)


@torch.library.custom_op(f"{NS}::syrk2", mutates_args=())
def syrk2(A: Tensor, trans: bool, mirror: bool) -> Tensor:
    return syrk_impl(A.contiguous(), trans)


@syrk2.register_fake
def _(A, trans, mirror):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n, n)


@torch.library.custom_op(f"{NS}::syrk2p", mutates_args=())
def syrk2p(A: Tensor, trans: bool) -> Tensor:
    return syrk_packed_impl(A.contiguous(), trans)


@syrk2p.register_fake
def _(A, trans):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n * (n + 1) // 2)


@torch.library.custom_op(f"{NS}::unpack", mutates_args=())
def unpack(Pk: Tensor, n: int) -> Tensor:
    return unpack_impl(Pk, n)


@unpack.register_fake
def _(Pk, n):
    return Pk.new_empty(n, n)
