"""The reference's operator plug-in surface on B200 (psgd_pro_fast.py:106-126 EagerOps; kernels/ops.py:24-215).

B200Ops has the EagerOps method set (gram, gram_q, norm_lower_bound_spd / _skh, symm, symm_r, syrk, sym, flags),
so psgd_pro_fast.KronWhiten(ops=B200Ops) or make_ops(flags) callers keep working; the same contracts are also
registered as torch custom ops under the reference's names (psgd::tri_vmm, psgd::tri_rownorm2, psgd::symm,
psgd::symm_right, psgd::syrk_cublas, psgd::syrk, psgd::syrk2, psgd::syrk2p, psgd::unpack), each with a fake
implementation for tracing. When the reference's own kernels module has registered those names already, this
module registers under psgd_b200:: instead.

Every number is computed by libpsgd_b200.so on the current stream: the products in the tcgen05 GEMM with bf16 hi/lo
operands (three MMAs, fp32 accumulation; about 1e-6 relative to fp64 on random inputs), operands staged by the
staging kernels, symmetric inputs expanded from their storage form by psgd_sym_expand, which reads only the stored
triangle. Inputs are fp32 CUDA tensors as in the reference (kernels/k1.cu:275-278, kernels/blas.cpp:22); a
symmetric matrix may be given full, as an upper triangle in a square (the lower triangle is never read, NaN
allowed: kernels/ops.py:9) or packed (the row-major upper triangle, element (i, j), i <= j, at i n - i (i - 1) / 2 +
j - i: kernels/k2.py:78). This module only allocates outputs and staging buffers and fills launch descriptors.

Errors: argument problems raise RuntimeError at the call, as the reference's TORCH_CHECKs do. Device-side problems
(a bounded wait in a kernel that gave up) set bits in a per-device error word that every launch here shares; each
call copies the word to pinned host memory after its launches (no synchronisation), and the next call raises
RuntimeError once that copy has landed with a nonzero value. check_errors() synchronises and raises at once."""
import ctypes

import torch
from torch import Tensor

from . import _capi
from . import kernels as K
from ._capi import check

_KEEP = []  # item arrays and staging buffers of the last calls (released once later calls have been enqueued)
K_SUB = 32


def _keep(*objs):
    _KEEP.append(objs)
    del _KEEP[:-16]


# ---- the shared device error word ------------------------------------------------------------------------------
class _ErrorWords:
    def __init__(self):
        self.word, self.host, self.event = {}, {}, {}

    def get(self, dev):
        k = dev.index if dev.index is not None else torch.cuda.current_device()
        if k not in self.word:
            self.word[k] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", k))
            self.host[k] = torch.zeros(1, dtype=torch.int32).pin_memory()
        return self.word[k]

    def _raise_if_set(self, k):
        v = int(self.host[k][0])
        if v:
            raise RuntimeError(f"psgd_pro_b200.ops: a kernel reported device error flags {v:#x} "
                               "(a bounded wait gave up); the results of the calls since are not valid")

    def pending(self, dev):
        """Raises when an earlier call's copy of the word has landed and is nonzero (no waiting)."""
        k = dev.index if dev.index is not None else torch.cuda.current_device()
        ev = self.event.get(k)
        if ev is not None and ev.query():
            self._raise_if_set(k)

    def after(self, dev):
        if torch.cuda.is_current_stream_capturing():
            return
        k = dev.index if dev.index is not None else torch.cuda.current_device()
        self.host[k].copy_(self.word[k], non_blocking=True)
        ev = self.event.get(k) or torch.cuda.Event()
        ev.record()
        self.event[k] = ev

    def check(self):
        for k, ev in self.event.items():
            ev.synchronize()
            self._raise_if_set(k)

    def reset(self):
        for k, w in self.word.items():
            w.zero_()
            self.host[k].zero_()


_ERR = _ErrorWords()


def check_errors():
    """Waits for the plug-in's launches and raises RuntimeError if any kernel reported a device error."""
    _ERR.check()


def reset_errors():
    _ERR.reset()


class _call:
    """Brackets one public op: earlier device errors raise first; the error word is read back afterwards."""

    def __init__(self, t):
        self.dev = t.device

    def __enter__(self):
        _ERR.pending(self.dev)
        return _ERR.get(self.dev)

    def __exit__(self, exc_type, exc, tb):
        if exc_type is None:
            _ERR.after(self.dev)
        return False


def _check(t, name):
    if not (t.is_cuda and t.dtype == torch.float32):
        raise RuntimeError(f"psgd_pro_b200.ops: {name} must be an fp32 CUDA tensor")


def side(S):
    """n of a symmetric matrix in storage form (square, or packed with n(n+1)/2 values); kernels/ops.py:119-121."""
    return S.shape[0] if S.dim() == 2 else int(((8 * S.shape[0] + 1) ** 0.5 - 1) / 2)


def _upload(struct_obj):
    host = torch.empty(ctypes.sizeof(struct_obj), dtype=torch.uint8)
    ctypes.memmove(host.data_ptr(), ctypes.addressof(struct_obj), ctypes.sizeof(struct_obj))
    return host.to(torch.device("cuda", torch.cuda.current_device()))


_PAIRS = {}  # device work lists of the tile pairs (I <= J) by (n, device), built once per size


def _pairs64(n):
    dev = torch.device("cuda", torch.cuda.current_device())
    w = _PAIRS.get((n, dev))
    if w is None:
        T = -(-n // _capi.SYM_TILE)
        I, J = torch.triu_indices(T, T).to(torch.int32)
        code = (I << 16) | J
        w = (torch.stack([torch.zeros_like(code), code], 1).reshape(-1).to(dev), code.numel())
        if len(_PAIRS) > 256:
            _PAIRS.clear()
        _PAIRS[(n, dev)] = w
    return w


def _sym_item(S, sign):
    """SymItem reading S (square upper triangle or packed) and the storage-form checks of kernels/k1.cu:275-278."""
    _check(S, "S")
    n = side(S)
    it = _capi.SymItem()
    if S.dim() == 2:
        if S.shape[0] != S.shape[1] or S.stride(1) != 1:
            raise RuntimeError("psgd_pro_b200.ops: a square symmetric input must be n x n with unit column stride")
        it.a, it.lda, it.form = S.data_ptr(), S.stride(0), _capi.PSGD_SYM_SQUARE
    elif S.dim() == 1:
        if n * (n + 1) // 2 != S.shape[0] or not S.is_contiguous():
            raise RuntimeError("psgd_pro_b200.ops: a packed symmetric input must hold n(n+1)/2 contiguous values")
        it.a, it.lda, it.form = S.data_ptr(), n, _capi.PSGD_SYM_PACKED
    else:
        raise RuntimeError("psgd_pro_b200.ops: a symmetric input is a square matrix or a packed triangle")
    it.n, it.sign = n, int(sign)
    return it, n


def _sym_expand(it, n, err):
    items = _upload(it)
    work, nwork = _pairs64(n)
    check(_capi.lib().psgd_sym_expand(items.data_ptr(), work.data_ptr(), nwork, err.data_ptr(), K.stream_handle()),
          "psgd_sym_expand")
    _keep(items, work)
    return items


def _sym_operand(S, sign, err, extra=None):
    """Full (sign 1), skew (-1) or upper-triangular (0) matrix of S as a bf16 hi/lo operand, read from the stored
    triangle only; extra: further SymItem fields (reduction outputs)."""
    it, n = _sym_item(S, sign)
    hi, lo = K.operand(n, n, S.device, True)
    it.out_hi, it.out_lo, it.ld_out = hi.data_ptr(), lo.data_ptr(), hi.stride(0)
    for k, v in (extra or {}).items():
        setattr(it, k, v)
    _sym_expand(it, n, err)
    return (hi, lo), n


def _op(X, err, transpose=False):
    """bf16 hi/lo operand of X (or X^T), staged by the psgd_prep kernel."""
    op, keep = K.to_operand(X, transpose=transpose, split=True, err=err)
    _keep(keep)
    return op


def _gemm(a_op, b_op, M, N, Kd, err, alpha=1.0, mode=K.PSGD_GEMM_PLAIN, bn=None, **out):
    spec = K.make_spec(a_op, b_op, M, N, Kd, bn=bn or K_choose(N), alpha=alpha, mode=mode, **out)
    K.gemm(spec, 3, err)
    _keep(a_op, b_op)


def K_choose(N):
    best = None
    for b in (128, 64, 32, 16):
        waste = -(-N // b) * b - N
        if best is None or waste < best[0]:
            best = (waste, b)
    return best[1]


# ---- the products ---------------------------------------------------------------------------------------------------
def _syrk(X, trans, err, **out):
    A = _op(X, err, transpose=trans)
    n, Kd = (X.shape[1], X.shape[0]) if trans else (X.shape[0], X.shape[1])
    K.gemm(K.make_spec(A, A, n, n, Kd, bn=128, mode=K.PSGD_GEMM_SYRK, **out), 3, err)
    _keep(A)
    return n


def syrk_impl(X, trans):
    """Full symmetric X^T X (trans) or X X^T, computed on the upper tiles only and mirrored (exactly symmetric)."""
    _check(X, "X")
    X = X.contiguous()
    with _call(X) as err:
        n = X.shape[1] if trans else X.shape[0]
        C = torch.empty(n, n, device=X.device)
        _syrk(X, trans, err, out_f32=C)
    return C


def syrk_packed_impl(X, trans):
    """Row-major packed upper triangle of X^T X (trans) or X X^T, n(n+1)/2 values written by the SYRK epilogue
    itself (kernels/k2.py:78-80); no full square is formed."""
    _check(X, "X")
    X = X.contiguous()
    with _call(X) as err:
        n = X.shape[1] if trans else X.shape[0]
        P = torch.empty(n * (n + 1) // 2, device=X.device)
        _syrk(X, trans, err, out_packed=P)
    return P


def symm_impl(S, X):
    """S @ X with S symmetric in storage form (kernels/blas.cpp:35-49 cublasSsymm, side left)."""
    _check(X, "X")
    X = X.contiguous()
    with _call(X) as err:
        A, n = _sym_operand(S, 1, err)
        if X.shape[0] != n:
            raise RuntimeError("psgd_pro_b200.ops.symm: shape mismatch")
        p = X.shape[1]
        C = torch.empty(n, p, device=X.device)
        _gemm(A, _op(X, err, transpose=True), n, p, n, err, out_f32=C)
    return C


def symm_right_impl(X, S):
    """X @ S with S symmetric in storage form (kernels/blas.cpp:51-65, side right)."""
    _check(X, "X")
    X = X.contiguous()
    with _call(X) as err:
        B, n = _sym_operand(S, 1, err)
        if X.shape[1] != n:
            raise RuntimeError("psgd_pro_b200.ops.symm_right: shape mismatch")
        m = X.shape[0]
        C = torch.empty(m, n, device=X.device)
        _gemm(_op(X, err), B, m, n, n, err, out_f32=C)
    return C


def tri_vmm_impl(V, A, sign):
    """W = V @ A_sym for a symmetric (sign 1) or skew-symmetric (sign -1) A read from its upper triangle; the
    skew diagonal is taken as zero (kernels/k1.cu:1-3, :31-53)."""
    _check(V, "V")
    V = V.contiguous()
    with _call(V) as err:
        B, n = _sym_operand(A, 1 if sign > 0 else -1, err)
        m = V.shape[0]
        W = torch.empty(m, n, device=V.device)
        # W[v, c] = sum_k V[v, k] A[k, c] = sum_k V[v, k] (sign A[c, k]): B operand = A itself, alpha = sign
        _gemm(_op(V, err), B, m, n, n, err, alpha=float(sign), out_f32=W)
    return W


def trmm_impl(T, X):
    """triu(T) @ X for a square fp32 T whose upper triangle is read (the triangular-times-dense product of the
    benchmark plan; no reference op). The operand is staged with zeros below the diagonal and the product skips the
    zero blocks (PSGD_GEMM_TRMM)."""
    _check(X, "X")
    X = X.contiguous()
    with _call(X) as err:
        A, n = _sym_operand(T, 0, err)
        if X.shape[0] != n:
            raise RuntimeError("psgd_pro_b200.ops.trmm: shape mismatch")
        p = X.shape[1]
        C = torch.empty(n, p, device=X.device)
        _gemm(A, _op(X, err, transpose=True), n, p, n, err, mode=K.PSGD_GEMM_TRMM, out_f32=C)
    return C


def tri_rownorm2_impl(A):
    """(squared row norms, max |A_ij|) of the symmetric matrix held in the upper triangle (kernels/k1.cu:296-307):
    one pass over the stored triangle, then a fixed-order reduction of the per-tile partials."""
    with _call(A) as err:
        it, n = _sym_item(A, 1)
        T = -(-n // _capi.SYM_TILE)
        part_row = torch.empty(T, n, device=A.device)
        part_max = torch.zeros(T * T, device=A.device)
        r = torch.empty(n, device=A.device)
        m = torch.empty((), device=A.device)
        it.part_row, it.part_max, it.row_sq, it.absmax = part_row.data_ptr(), part_max.data_ptr(), r.data_ptr(), \
            m.data_ptr()
        items = _sym_expand(it, n, err)
        check(_capi.lib().psgd_sym_reduce(items.data_ptr(), 1, n, err.data_ptr(), K.stream_handle()), "sym_reduce")
        _keep(part_row, part_max)
    return r, m


def unpack_impl(Pk, n, sign=1):
    """Full symmetric n x n matrix from its row-major packed upper triangle (kernels/k2.py:88-103)."""
    _check(Pk, "Pk")
    with _call(Pk) as err:
        it, n2 = _sym_item(Pk.contiguous(), sign)
        if n2 != n:
            raise RuntimeError("psgd_pro_b200.ops.unpack: the packed length does not match n")
        C = torch.empty(n, n, device=Pk.device)
        it.out_f32, it.ld_f32 = C.data_ptr(), C.stride(0)
        _sym_expand(it, n, err)
    return C


def _norm_lower_bound(A, V, skew):
    """The subspace iteration of psgd_pro.py:19-65 with the random start V given (psgd_pro_fast.py:32-51), all on
    the device: A expanded from its stored triangle with its row sums of squares and diagonal (spd) or max |A|
    (skh); psgd_nlb_prep picks the row of largest norm, nf, and V0 = A_j / nf + sgn(<A_j / nf, V_r>) V_r; four
    products W^T = A^T V^T (N = 32) whose epilogues apply 1/nf and the row normalisation; psgd_nlb_finish takes
    nf * max_r |V_r|."""
    _check(V, "V")
    V = V.contiguous()
    with _call(V) as err:
        it, n = _sym_item(A, -1 if skew else 1)
        if V.shape != (K_SUB, n):
            raise RuntimeError("psgd_pro_b200.ops: V must be 32 x n")
        dev = V.device
        T = -(-n // _capi.SYM_TILE)
        part_row = torch.empty(T, n, device=dev)
        part_max = torch.zeros(T * T, device=dev)
        diag = torch.empty(n, device=dev)
        hi, lo = K.operand(n, n, dev, True)
        it.out_hi, it.out_lo, it.ld_out = hi.data_ptr(), lo.data_ptr(), hi.stride(0)
        it.part_row, it.part_max, it.diag = part_row.data_ptr(), part_max.data_ptr(), diag.data_ptr()
        _sym_expand(it, n, err)
        Aop = (hi, lo)
        V0, Wa, Wb = (K.operand(K_SUB, n, dev, True) for _ in range(3))
        nf = torch.empty(1, device=dev)
        nl = _capi.NlbPrepItem()
        nl.a_hi, nl.a_lo, nl.lda, nl.n, nl.skew = hi.data_ptr(), lo.data_ptr(), hi.stride(0), n, int(skew)
        nl.part_row, nl.row_slots = part_row.data_ptr(), T
        if skew:
            nl.part_max, nl.max_slots = part_max.data_ptr(), T * T
        else:
            nl.diag = diag.data_ptr()
        nl.v, nl.v0_hi, nl.v0_lo, nl.ldv, nl.nf_out = V.data_ptr(), V0[0].data_ptr(), V0[1].data_ptr(), \
            V0[0].stride(0), nf.data_ptr()
        nl_dev = _upload(nl)
        check(_capi.lib().psgd_nlb_prep(nl_dev.data_ptr(), 1, err.data_ptr(), K.stream_handle()), "psgd_nlb_prep")
        Tn = -(-n // 128)
        pc = torch.zeros(4, Tn, K_SUB, device=dev)
        for k in range(4):  # the same chain as the optimizer's norm-bound phases
            src, dst = (V0, Wa, Wb, Wa)[k], (Wa, Wb, Wa, None)[k]
            kw = dict(cs_nf=nf)
            if k in (0, 2):
                kw.update(cs_mode=1, part_col=pc[k])
            else:
                kw.update(cs_mode=2, cs_part=pc[k - 1], cs_T=Tn)
                if k == 3:
                    kw.update(part_col=pc[3])
            if dst is not None:
                kw.update(out_hi_t=dst[0], out_lo_t=dst[1])
            K.gemm(K.make_spec(Aop, src, n, K_SUB, n, bn=32, alpha=-1.0 if skew else 1.0, **kw), 3, err)
        out = torch.empty((), device=dev)
        fin = _capi.NlbFinishItem()
        fin.nf, fin.part, fin.slots, fin.ncols, fin.out = nf.data_ptr(), pc[3].data_ptr(), Tn, K_SUB, out.data_ptr()
        fin_dev = _upload(fin)
        check(_capi.lib().psgd_nlb_finish(fin_dev.data_ptr(), 1, err.data_ptr(), K.stream_handle()), "nlb_finish")
        _keep(part_row, part_max, diag, Aop, V0, Wa, Wb, nf, nl_dev, pc, fin_dev)
    return out


def norm_lower_bound_spd(A, V):
    """psgd_pro_fast.py:46-47 (A in storage form): nf = max diagonal + smallest normal."""
    return _norm_lower_bound(A, V, skew=False)


def norm_lower_bound_skh(A, V):
    """psgd_pro_fast.py:50-51 (A skew-symmetric, as R = Q^T - Q; read from its upper triangle): nf = max |A| +
    smallest normal."""
    return _norm_lower_bound(A, V, skew=True)


class B200Ops:
    """psgd_pro_fast.EagerOps (psgd_pro_fast.py:106-126) with the dense products on B200."""
    flags = frozenset({"b200"})

    @staticmethod
    def gram(Pg, i, expr):
        """term1 of factor i of a 2-D Pg (Pg Pg^T for i = 0, Pg^T Pg for i = 1); other orders use expr."""
        if Pg.dim() != 2:
            return expr(Pg, Pg)
        return syrk_impl(Pg, i == 1)

    @staticmethod
    def gram_q(q):
        return syrk_impl(q, True)

    norm_lower_bound_spd = staticmethod(norm_lower_bound_spd)
    norm_lower_bound_skh = staticmethod(norm_lower_bound_skh)

    @staticmethod
    def symm(A, q):
        return symm_impl(A, q)

    @staticmethod
    def syrk(X, trans):
        return syrk_impl(X, trans)

    sym = syrk

    @staticmethod
    def symm_r(X, S):
        return symm_right_impl(X, S)


def make_ops(flags=()):
    """kernels/ops.py:142-215 compatibility: every flag combination maps to the B200 kernels (there is no size
    crossover: the tensor-core products serve every shape). "packed" keeps term1 and P as packed triangles."""
    flags = frozenset(flags)

    class Ops(B200Ops):
        pass

    if "packed" in flags:
        Ops.sym = staticmethod(lambda X, trans: syrk_packed_impl(X, trans))
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
    return tri_vmm_impl(V, A, sign)


@tri_vmm.register_fake
def _(V, A, sign):
    return V.new_empty(V.shape)


@torch.library.custom_op(f"{NS}::tri_rownorm2", mutates_args=())
def tri_rownorm2(A: Tensor) -> tuple[Tensor, Tensor]:
    return tri_rownorm2_impl(A)


@tri_rownorm2.register_fake
def _(A):
    return A.new_empty(A.shape[0]), A.new_empty(())


@torch.library.custom_op(f"{NS}::symm", mutates_args=())
def symm(S: Tensor, B: Tensor) -> Tensor:
    return symm_impl(S, B)


@symm.register_fake
def _(S, B):
    return B.new_empty(side(S), B.shape[1])


@torch.library.custom_op(f"{NS}::symm_right", mutates_args=())
def symm_right(B: Tensor, S: Tensor) -> Tensor:
    return symm_right_impl(B, S)


@symm_right.register_fake
def _(B, S):
    return B.new_empty(B.shape[0], side(S))


@torch.library.custom_op(f"{NS}::syrk_cublas", mutates_args=())
def syrk_cublas(A: Tensor, trans: bool) -> Tensor:
    """Name kept from kernels/ops.py:55-63 (there a cuBLAS call); the result holds both triangles."""
    return syrk_impl(A, trans)


@syrk_cublas.register_fake
def _(A, trans):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n, n)


@torch.library.custom_op(f"{NS}::syrk", mutates_args=())
def syrk(A: Tensor, trans: bool, mirror: bool) -> Tensor:
    """kernels/ops.py:66-75; the output is always mirrored (a valid answer for mirror = False as well: the
    contract there leaves the lower triangle unspecified)."""
    return syrk_impl(A, trans)


@syrk.register_fake
def _(A, trans, mirror):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n, n)


@torch.library.custom_op(f"{NS}::syrk2", mutates_args=())
def syrk2(A: Tensor, trans: bool, mirror: bool) -> Tensor:
    return syrk_impl(A, trans)


@syrk2.register_fake
def _(A, trans, mirror):
    n = A.shape[1] if trans else A.shape[0]
    return A.new_empty(n, n)


@torch.library.custom_op(f"{NS}::syrk2p", mutates_args=())
def syrk2p(A: Tensor, trans: bool) -> Tensor:
    return syrk_packed_impl(A, trans)


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
