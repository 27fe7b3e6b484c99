"""KronWhiten for B200: the PSGD-Kron (dQ = Q0.5EQ1.5) gradient-whitening optimizer of psgd_pro.py:251-384 /
psgd_pro_fast.py:239-499, with the same constructor arguments, mutable hyper-parameter attributes, step(closure)
and step_math(grads), computed by the sm_100a kernels of libpsgd_b200.so.

Layout. Every parameter is handled as an n1 x n2 matrix after squeeze() (psgd_pro.py:327): a 2-D parameter as
itself, a 1-D parameter of size n as 1 x n with a fixed identity first factor, a 0-d parameter as 1 x 1 with one
diagonal factor of size 1. Each Kronecker factor is dense (n x n fp32 Q, the reference layout) or diagonal
(length-n fp32 q) by the rule of psgd_pro.py:189. The step runs as a fixed sequence of phases; each phase is one
grouped launch over every parameter (tensor-core GEMM groups for the contractions, memory-bound kernels for the
rest), so a step costs about two dozen launches regardless of the number of parameters, and the sequence is
captured in CUDA graphs after the first step.

Precision. precision="fp32" multiplies bf16 hi/lo operand pairs (three MMAs per product, about 16 significant
bits) and matches the reference's fp32 results within 1e-3; precision="bf16" uses one bf16 MMA per product with
fp32 accumulation and fp32 master Q, L (the reference run with bf16 matmuls, tolerance 2e-2). The default follows
the parameter dtype, as the reference's arithmetic does (Q inherits the parameter dtype, psgd_pro.py:210).

Deviations in rounding only (same mathematics): the Procrustes step is the rank-n form of psgd_pro_fast.py:141-153;
P_i = Q_i^T Q_i is kept as state between steps (the p2d path, psgd_pro_fast.py:164-192); for a 1-D parameter with
a dense factor, term1 = Pg Pg^T is rank one, so its norm bound is |Pg|^2 (the value the subspace iteration of
psgd_pro.py:19-41 converges to on a rank-one matrix) and term1 q = Pg (q^T Pg)^T.
"""
import ctypes
import math
import struct

import torch

from . import _capi
from . import kernels as K
from ._capi import (PSGD_FACTOR_DENSE, PSGD_FACTOR_DIAG, PSGD_FACTOR_RANK1, PSGD_FACTOR_SKEW, PSGD_PREP_DIRECT,
                    PSGD_PREP_NORMAL, PSGD_PREP_TRANS, HY_COUNT, HY_LR_PRECOND, HY_BETA_L, HY_DAMPING, HY_LR_PARAMS,
                    HY_MAX_AVG, HY_MAX_ELEM, HY_MOM_BETA, HY_MOM_ALPHA, HY_EMA_PHASE, HY_NOISE, HY_NOISE_KEY0,
                    HY_NOISE_KEY1, APPLY_CHUNK, check)

K_SUB = 32  # subspace dimension of the norm lower bounds (psgd_pro.py:19, psgd_pro_fast.py:29)
TT = 32     # tile edge of the element-wise kernels
BM = 128    # GEMM tile rows

# per-factor scalar slots
S_L, S_NF_SPD, S_AQ, S_BQ, S_NF_SKH, S_AM, S_BM, S_COUNT = range(8)


def is_dense(size, numel, max_size, max_skew):
    """psgd_pro.py:189."""
    return not (size <= 1 or size > max_size or size ** 2 > max_skew * numel)


def init_scale_from_grads(grads, damping):
    """psgd_pro.py:329-332: (max_i mean|g_i|^4 + damping^4)^(-1/8), accumulated in float64 (a one-time reduction;
    a sharded step takes it over every parameter's gradient on every rank, so all ranks agree bit for bit)."""
    m = max(float(torch.mean(g.detach().to(torch.float64).abs() ** 4)) for g in grads)
    return (m + damping ** 4) ** (-1 / 8)


def cdiv(a, b):
    return (a + b - 1) // b


def choose_bn(N, split):
    """GEMM tile width for an N-wide output: least padding, then the widest tile."""
    best = None
    for b in (256, 128, 64, 32, 16):
        if split == 3 and b > 128:
            continue
        waste = cdiv(N, b) * b - N
        if best is None or waste < best[0]:
            best = (waste, b)
    return best[1]


def _upload(cls, items, device):
    """A ctypes struct array copied into a device byte buffer."""
    arr = (cls * max(len(items), 1))(*items)
    host = torch.empty(ctypes.sizeof(arr), dtype=torch.uint8)
    ctypes.memmove(host.data_ptr(), ctypes.addressof(arr), ctypes.sizeof(arr))
    return host.to(device)


def _work(pairs, device):
    flat = [v for p in pairs for v in p]
    return torch.tensor(flat if flat else [0, 0], dtype=torch.int32).to(device), len(pairs)


def _tile_pairs(item, rows, cols):
    return [(item, (ti << 16) | tj) for ti in range(cdiv(rows, TT)) for tj in range(cdiv(cols, TT))]


class _Factor:
    """One Kronecker factor: 'dense' (n x n Q), 'diag' (length-n q) or 'none' (the fixed identity first factor of
    a 1-D parameter). Dense factors own their operand copies and per-step partial buffers."""

    def __init__(self, kind, n, scale, numel, fidx, plan, rank1=False):
        dev, split = plan.device, plan.split
        self.kind, self.n, self.fidx, self.rank1 = kind, n, fidx, rank1
        self.term2 = numel / n if kind != "none" else 0.0  # psgd_pro.py:127, :132
        if kind == "dense":
            self.q = torch.eye(n, device=dev) * scale
            sp = split == 3
            self.qta, self.qtb = K.operand(n, n, dev, sp), K.operand(n, n, dev, sp)
            self.P, self.T, self.R = K.operand(n, n, dev, sp), K.operand(n, n, dev, sp), K.operand(n, n, dev, sp)
            self.V0, self.Wa, self.Wb = (K.operand(K_SUB, n, dev, sp) for _ in range(3))
            self.Tn, self.T32 = cdiv(n, BM), cdiv(n, TT)
            # SYRK tiles are 128 x sbn; its row-sum partials use cdiv(n, sbn) direct + Tn mirrored slots
            self.sbn = 256 if split == 1 else 128
            self.Ts = cdiv(n, self.sbn) + self.Tn
            self.t_rows = torch.zeros(self.Ts, n, device=dev)
            self.t_diag = torch.zeros(n, device=dev)
            self.pc = torch.zeros(4, self.Tn, K_SUB, device=dev)
            self.pcs = torch.zeros(4, self.Tn, K_SUB, device=dev)
            self.r_rows = torch.zeros(self.T32, n, device=dev)
            self.r_max = torch.zeros(self.T32 * self.T32, device=dev)
            self.r_dot = torch.zeros(self.T32 * self.T32, device=dev)
            self.s_dot = torch.zeros(cdiv(n, _capi.TRACE_ROWS), device=dev)  # trace partials of S o Q
            self.refresh_operands()
        elif kind == "diag":
            self.q = torch.full((n,), float(scale), device=dev)
            self.p = self.q * self.q
        else:
            self.q, self.p = None, None

    def refresh_operands(self):
        """QT = Q^T and P = Q^T Q operand copies from the fp32 Q (initialisation and rebalancing)."""
        K.split_into(self.q.T.contiguous(), *self.qta)
        K.split_into(self.q.T @ self.q, *self.P)


class _Param:
    def __init__(self, param, shape, scale, plan, pidx):
        self.param, self.pidx = param, pidx
        self.shape = tuple(shape)
        numel = max(1, math.prod(self.shape))
        self.numel = numel
        order = len(shape)
        if order > _capi.PERMUTE_MAX_ORDER:
            raise NotImplementedError(f"psgd_pro_b200.KronWhiten handles parameters of order up to "
                                      f"{_capi.PERMUTE_MAX_ORDER}; got shape {tuple(shape)} (squeezed)")
        s = scale ** (1.0 / order) if order > 0 else scale  # psgd_pro.py:181 (0-d: Scale itself, :170)
        self.nd = order >= 3
        if self.nd:  # one factor per dim (psgd_pro.py:185-212); the products run through layout changes
            self.n1, self.n2 = numel // shape[-1], shape[-1]
            self.factors = [plan.new_factor("dense" if is_dense(n, numel, plan.max_size, plan.max_skew) else "diag",
                                            n, s, numel) for n in shape]
            self.f1 = self.f2 = None
            self.kind = ("nd",)
            self._nd_buffers(plan)
            return
        if order == 2:
            self.n1, self.n2 = shape
            k1 = "dense" if is_dense(self.n1, numel, plan.max_size, plan.max_skew) else "diag"
            k2 = "dense" if is_dense(self.n2, numel, plan.max_size, plan.max_skew) else "diag"
            self.f1 = plan.new_factor(k1, self.n1, s, numel)
            self.f2 = plan.new_factor(k2, self.n2, s, numel)
            self.factors = [self.f1, self.f2]
        elif order == 1:
            self.n1, self.n2 = 1, shape[0]
            k2 = "dense" if is_dense(self.n2, numel, plan.max_size, plan.max_skew) else "diag"
            self.f1 = _Factor("none", 1, 1.0, numel, -1, plan)
            self.f2 = plan.new_factor(k2, self.n2, s, numel, rank1=(k2 == "dense"))
            self.factors = [self.f2]
        else:
            self.n1 = self.n2 = 1
            self.f1 = _Factor("none", 1, 1.0, numel, -1, plan)
            self.f2 = plan.new_factor("diag", 1, s, numel)
            self.factors = [self.f2]
        self.kind = (self.f1.kind, self.f2.kind)
        dev, sp = plan.device, plan.split == 3
        n1, n2 = self.n1, self.n2
        k = self.kind
        self.gop = self.yT = self.pg_op = self.pgT = self.w = None
        self.gop_a = None  # the clean operand of the parameter update (PREP_NORMAL parameters)
        if k in (("dense", "dense"), ("diag", "dense"), ("none", "dense")):
            self.gop = K.operand(n1, n2, dev, sp)
            self.gop_a = K.operand(n1, n2, dev, sp)
        elif k == ("dense", "diag"):
            self.gop = K.operand(n2, n1, dev, sp)
        if k == ("dense", "dense"):
            self.yT = K.operand(n2, n1, dev, sp)
        if k in (("dense", "dense"), ("dense", "diag"), ("none", "dense")):
            self.pg_op = K.operand(n1, n2, dev, sp)
        if k in (("dense", "dense"), ("diag", "dense"), ("none", "dense")):
            self.pgT = K.operand(n2, n1, dev, sp)
        if k == ("none", "dense"):
            self.w = K.operand(n2, 1, dev, sp)
        self.pg32 = torch.empty(n1, n2, device=dev)

    def _nd_buffers(self, plan):
        """Order-r parameter: the staged gradient x (fp32, natural layout), two fp32 buffers the chain of mode
        products alternates between, and per dense mode k an operand for its product (the tensor with mode k last,
        N / d_k x d_k) and one for its term1 (mode k first, d_k x N / d_k); per diagonal mode the row sums of squares
        of the mode-first layout (its term1)."""
        dev, sp, N = plan.device, plan.split == 3, self.numel
        self.x32 = torch.empty(N, device=dev)
        self.ch = [torch.empty(N, device=dev), torch.empty(N, device=dev)]
        self.pg32 = torch.empty(self.n1, self.n2, device=dev)
        self.op_last, self.op_first, self.t1_diag = {}, {}, {}
        for k, (n, f) in enumerate(zip(self.shape, self.factors)):
            if f.kind == "dense":
                self.op_last[k] = K.operand(N // n, n, dev, sp)
                self.op_first[k] = K.operand(n, N // n, dev, sp)
            else:
                self.t1_diag[k] = torch.zeros(1, n, device=dev)
        self.apart = torch.zeros(cdiv(N, _capi.PERMUTE_CHUNK), device=dev)


def _permute_item(src, dims, src_last, dst_mode, dst_first, scales, op=None, out_f32=None, row_sq=None, part=None):
    """PermuteItem moving a tensor of natural dims `dims` from the layout with mode src_last moved to the end (None:
    natural) to the one with dst_mode moved to the end, or to the front when dst_first (None: natural)."""
    r, N = len(dims), math.prod(dims)
    src_order = [m for m in range(r) if m != src_last] + ([src_last] if src_last is not None else [])
    stride, st = {}, 1
    for m in reversed(src_order):
        stride[m] = st
        st *= dims[m]
    if dst_mode is None:
        out_order = list(range(r))
    elif dst_first:
        out_order = [dst_mode] + [m for m in range(r) if m != dst_mode]
    else:
        out_order = [m for m in range(r) if m != dst_mode] + [dst_mode]
    it = _capi.PermuteItem()
    it.src, it.order, it.numel = src.data_ptr(), r, N
    for pos, m in enumerate(out_order):
        it.omode[pos], it.odim[pos] = m, dims[m]
    for m in range(r):
        it.sstride[m] = stride[m]
        it.scale[m] = scales[m].data_ptr() if scales[m] is not None else None
    it.cols = (N // dims[dst_mode]) if (dst_mode is not None and dst_first) else \
        (dims[dst_mode] if dst_mode is not None else dims[-1])
    if op is not None:
        it.out_hi, it.out_lo, it.ld_out = K.ptr(op[0]), K.ptr(op[1]), op[0].stride(0)
    it.out_f32 = K.ptr(out_f32)
    it.row_sq, it.part = K.ptr(row_sq), K.ptr(part)
    units = (N // it.cols) if row_sq is not None else cdiv(N, _capi.PERMUTE_CHUNK)
    return it, units


class _Plan:
    """Buffers, item arrays and GEMM groups of one optimizer configuration (fixed device addresses)."""

    def __init__(self, params, shapes, scale, max_size, max_skew, split, device):
        self.device, self.split, self.max_size, self.max_skew = device, split, max_size, max_skew
        self.factors = []
        self.params = [_Param(p, s, scale, self, k) for k, (p, s) in enumerate(zip(params, shapes))]
        nf = max(1, len(self.factors))
        self.scal = torch.zeros(nf, S_COUNT, device=device)
        self.L = self.scal[:, S_L]
        self.hyper = torch.zeros(HY_COUNT, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.clip = torch.zeros(max(1, len(self.params)), device=device)
        # random draws: the damping noise of every parameter, then two 32 x n starts per dense factor
        # each parameter's slice starts on a 16-byte boundary (vector loads)
        self.xi = torch.zeros(sum(cdiv(p.numel, 4) * 4 for p in self.params), device=device)
        off = 0
        for p in self.params:
            p.xi = self.xi[off:off + p.numel].view(p.n1, p.n2)
            p.xi_off = off  # also the parameter's place in the generated noise sequence
            off += cdiv(p.numel, 4) * 4
        dense = [f for f in self.factors if f.kind == "dense"]
        self.vbuf = torch.zeros(sum(2 * K_SUB * f.n for f in dense), device=device)
        off = 0
        for f in dense:
            f.v_spd = self.vbuf[off:off + K_SUB * f.n].view(K_SUB, f.n)
            f.v_skh = self.vbuf[off + K_SUB * f.n:off + 2 * K_SUB * f.n].view(K_SUB, f.n)
            off += 2 * K_SUB * f.n
        self.grad_ptrs = None
        self.mom_key, self.ms_ptrs = None, None

    def new_factor(self, kind, n, scale, numel, rank1=False):
        f = _Factor(kind, n, scale, numel, len(self.factors), self, rank1)
        self.factors.append(f)
        return f

    # ---- phase construction ------------------------------------------------------------------------------------
    def spec(self, a, b, M, N, Kd, bn=None, **kw):
        return K.make_spec(a, b, M, N, Kd, bn=bn or choose_bn(N, self.split), **kw)

    def syrk(self, a, n, Kd, **kw):
        return K.make_spec(a, a, n, n, Kd, bn=256 if self.split == 1 else 128, mode=K.PSGD_GEMM_SYRK, **kw)

    def group(self, specs):
        if not specs:
            return None
        specs = sorted(specs, key=lambda s: -(s.K * cdiv(s.M, BM) * cdiv(s.N, s.bn)))
        return K.GemmGroup(specs, self.split, self.device)

    def s(self, f, slot):
        return self.scal[f.fidx, slot:slot + 1]

    def build(self, grads, ms, whiten_grad, grad_eps):
        """Encodes every phase. grads: the gradients in parameter order (their data pointers are baked into the
        staging items; update_grad_ptrs re-points them); ms: the momentum buffers or None. The staging passes
        take the momentum as their source where the reference does (psgd_pro.py:350-361: the update whitens g or m,
        the preconditioner is applied to m when there is momentum) and apply its EMA in the first pass of the step
        that reads it (hyper[HY_EMA_PHASE]: 1 when the update runs first on m, else 0)."""
        dev, split = self.device, self.split
        P = self.params
        self.grad_ptrs = tuple(t.data_ptr() for t in grads)
        self.mom_key = (ms is not None, bool(whiten_grad))
        self._ptr_items = {}
        # U0 / A0: gradient staging. When both passes stage the same source (no momentum, or the momentum in both),
        # the update's pass also writes the clean operand of PREP_NORMAL parameters (gop_a), and an apply that
        # follows an update in the same step stages only the other parameters (work list prep_a_rest).
        self.fuse_stage = ms is None or not whiten_grad
        self.prep_u, self.prep_a = [], []
        pu, pa, pa_rest = [], [], []
        self.t1 = {}
        for k, p in enumerate(P):
            kind = p.kind
            for phase, src, items, pairs in (("u", grads[k], self.prep_u, pu), ("a", grads[k], self.prep_a, pa)):
                it = _capi.PrepItem()
                it.g, it.g_bf16 = src.data_ptr(), int(src.dtype == torch.bfloat16)
                if ms is not None and (phase == "a" or not whiten_grad):
                    it.m, it.mom_phase = ms[k].data_ptr(), (1 if phase == "u" else 0)
                it.xi = p.xi.data_ptr() if phase == "u" else None
                it.noise_base = p.xi_off
                it.n1, it.n2, it.eps = p.n1, p.n2, grad_eps[k]
                if p.nd:  # order-r parameter: x (with noise and momentum) staged in fp32, natural layout
                    it.mode, it.out_f32 = PSGD_PREP_DIRECT, p.x32.data_ptr()
                    items.append(it)
                    pairs += _tile_pairs(len(items) - 1, p.n1, p.n2)
                    continue
                it.p1 = p.f1.p.data_ptr() if p.f1.kind == "diag" else None
                it.p2 = p.f2.p.data_ptr() if p.f2.kind == "diag" else None
                if kind == ("dense", "diag"):
                    it.mode = PSGD_PREP_TRANS
                    it.out_hi, it.out_lo, it.ld_out = K.ptr(p.gop[0]), K.ptr(p.gop[1]), p.gop[0].stride(0)
                elif p.gop is not None:
                    it.mode = PSGD_PREP_NORMAL
                    op = p.gop if phase == "u" else p.gop_a
                    it.out_hi, it.out_lo, it.ld_out = K.ptr(op[0]), K.ptr(op[1]), op[0].stride(0)
                    if phase == "u" and self.fuse_stage:
                        it.out2_hi, it.out2_lo = K.ptr(p.gop_a[0]), K.ptr(p.gop_a[1])
                else:
                    it.mode = PSGD_PREP_DIRECT
                    if phase == "u":
                        if p.f1.kind == "diag":
                            p.t1r = torch.zeros(cdiv(p.n2, TT), p.n1, device=dev)
                            it.part_row = p.t1r.data_ptr()
                            self.t1[p.f1.fidx] = (p.t1r, p.t1r.shape[0])
                        p.t1c = torch.zeros(cdiv(p.n1, TT), p.n2, device=dev)
                        it.part_col = p.t1c.data_ptr()
                        self.t1[p.f2.fidx] = (p.t1c, p.t1c.shape[0])
                    else:
                        p.apart = torch.zeros(cdiv(p.n1, TT) * cdiv(p.n2, TT), device=dev)
                        it.out_f32, it.part_tile = p.pg32.data_ptr(), p.apart.data_ptr()
                items.append(it)
                if it.mode == PSGD_PREP_NORMAL:
                    w = [(len(items) - 1, rb) for rb in range(cdiv(p.n1, _capi.PREP_ROWS))]
                else:
                    w = _tile_pairs(len(items) - 1, p.n1, p.n2)
                pairs += w
                if phase == "a" and not (it.mode == PSGD_PREP_NORMAL and self.fuse_stage):
                    pa_rest += w
        self.prep_u_dev = _upload(_capi.PrepItem, self.prep_u, dev)
        self.prep_a_dev = _upload(_capi.PrepItem, self.prep_a, dev)
        self.prep_u_work, self.prep_u_n = _work(pu, dev)
        self.prep_a_work, self.prep_a_n = _work(pa, dev)
        self.prep_a_rest_work, self.prep_a_rest_n = _work(pa_rest, dev)

        # U1, U2: Pg of the noisy gradient
        u1, u2, u3, u3r = [], [], [], []
        for p in P:
            if p.nd:
                continue
            n1, n2, f1, f2 = p.n1, p.n2, p.f1, p.f2
            if p.kind == ("dense", "dense"):
                u1.append(self.spec(p.gop, f2.P, n1, n2, n2, out_hi_t=p.yT[0], out_lo_t=p.yT[1]))
                u2.append(self.spec(f1.P, p.yT, n1, n2, n1, out_hi=p.pg_op[0], out_lo=p.pg_op[1],
                                    out_hi_t=p.pgT[0], out_lo_t=p.pgT[1]))
            elif p.kind == ("diag", "dense"):
                bn = choose_bn(n2, split)
                p.t1r = torch.zeros(cdiv(n2, bn), n1, device=dev)
                self.t1[f1.fidx] = (p.t1r, p.t1r.shape[0])
                u1.append(self.spec(p.gop, f2.P, n1, n2, n2, bn=bn, row_scale=f1.p, out_hi_t=p.pgT[0],
                                    out_lo_t=p.pgT[1], part_row=p.t1r))
            elif p.kind == ("none", "dense"):
                bn = choose_bn(n2, split)
                p.r1part = torch.zeros(cdiv(n2, bn), device=dev)
                u1.append(self.spec(p.gop, f2.P, 1, n2, n2, bn=bn, out_hi=p.pg_op[0], out_lo=p.pg_op[1],
                                    out_hi_t=p.pgT[0], out_lo_t=p.pgT[1], part_tile=p.r1part))
            elif p.kind == ("dense", "diag"):
                p.t1c = torch.zeros(cdiv(n1, BM), n2, device=dev)
                self.t1[f2.fidx] = (p.t1c, p.t1c.shape[0])
                u2.append(self.spec(f1.P, p.gop, n1, n2, n1, out_hi=p.pg_op[0], out_lo=p.pg_op[1], part_col=p.t1c))
            # U3: term1 of the dense factors (rank-one 1-D factors: w = q^T Pg instead)
            if f1.kind == "dense":
                u3.append(self.syrk(p.pg_op, n1, n2, out_hi=f1.T[0], out_lo=f1.T[1], part_row=f1.t_rows,
                                    diag_out=f1.t_diag))
            if f2.kind == "dense" and not f2.rank1:
                u3.append(self.syrk(p.pgT, n2, n1, out_hi=f2.T[0], out_lo=f2.T[1], part_row=f2.t_rows,
                                    diag_out=f2.t_diag))
            if f2.kind == "dense" and f2.rank1:
                u3r.append(self.spec(f2.qta, p.pg_op, n2, 1, n2, bn=16, out_hi=p.w[0], out_lo=p.w[1]))
        # order-r parameters: chains of mode products through layout changes; their term1 SYRKs join U3
        self.nd_u, nd_t1 = self._nd_chain(noisy=True, term1_specs=u3)
        self.nd_a = self._nd_chain(noisy=False)
        self.nd_t1 = nd_t1
        # the skinny rank-one products form groups of their own, so the big products' groups can run on CTA pairs
        # (and the 1 x n rows of 1-D parameters leave the Y products' groups for the same reason)
        self.g_u1, self.g_u1r = self.group([x for x in u1 if x.M >= BM]), self.group([x for x in u1 if x.M < BM])
        self.g_u2, self.g_u3, self.g_u3r = self.group(u2), self.group(u3), self.group(u3r)

        dense = [f for f in self.factors if f.kind == "dense"]
        nlb = [f for f in dense if not f.rank1]
        # U4..U8: norm lower bound of term1 (spd)
        self.nlb_spd_dev, self.nlb_spd_n = self._nlb_prep(nlb, skew=False)
        self.g_spd = self._nlb_chain(nlb, skew=False)
        # U9: L, q-update coefficients, diagonal factors
        fi = []
        for f in self.factors:
            it = _capi.FactorItem()
            it.n, it.term2, it.L = f.n, f.term2, self.s(f, S_L).data_ptr()
            if f.kind == "dense" and not f.rank1:
                it.kind, it.nf, it.part, it.slots, it.ncols = (PSGD_FACTOR_DENSE, self.s(f, S_NF_SPD).data_ptr(),
                                                             f.pc[3].data_ptr(), f.Tn, K_SUB)
            elif f.kind == "dense":
                p = next(p for p in P if p.f2 is f)
                it.kind, it.part, it.slots = PSGD_FACTOR_RANK1, p.r1part.data_ptr(), p.r1part.numel()
            else:
                part, slots = self.t1[f.fidx]
                it.kind, it.part, it.slots, it.q, it.p = PSGD_FACTOR_DIAG, part.data_ptr(), slots, f.q.data_ptr(), \
                    f.p.data_ptr()
                f.fac_scratch = torch.zeros(_capi.FAC_SCRATCH, device=dev)
                it.scratch = f.fac_scratch.data_ptr()
            it.alpha, it.beta = self.s(f, S_AQ).data_ptr(), self.s(f, S_BQ).data_ptr()
            fi.append(it)
        self.fac_dev, self.fac_n = _upload(_capi.FactorItem, fi, dev), len(fi)
        # U10: q <- q - lr/L (term1 q - term2 q)
        # (rank-one factors: the same update, q <- alpha Pg w^T + beta q, runs inside the skew kernel below)
        u10 = []
        for f in dense:
            if not f.rank1:
                u10.append(self.spec(f.T, f.qta, f.n, f.n, f.n, alpha_ptr=self.s(f, S_AQ), beta_ptr=self.s(f, S_BQ),
                                     alpha=1.0, beta=1.0, aux=f.q, out_f32=f.q, out_hi_t=f.qtb[0],
                                     out_lo_t=f.qtb[1]))
        self.g_u10 = self.group(u10)
        # U11: Rn = Q - Q^T
        sk, skw, skw1 = [], [], []
        for f in dense:
            it = _capi.SkewItem()
            it.q, it.n, it.r_hi, it.r_lo, it.ldr = f.q.data_ptr(), f.n, K.ptr(f.R[0]), K.ptr(f.R[1]), f.R[0].stride(0)
            it.part_row, it.part_max, it.part_dot = f.r_rows.data_ptr(), f.r_max.data_ptr(), f.r_dot.data_ptr()
            if f.rank1:  # U10 for this factor: q <- alpha Pg w^T + beta q, q^T to qtb
                p = next(p for p in P if p.f2 is f)
                it.u_hi, it.u_lo, it.ldu = K.ptr(p.pgT[0]), K.ptr(p.pgT[1]), p.pgT[0].stride(0)
                it.v_hi, it.v_lo, it.ldv = K.ptr(p.w[0]), K.ptr(p.w[1]), p.w[0].stride(0)
                it.alpha, it.beta = self.s(f, S_AQ).data_ptr(), self.s(f, S_BQ).data_ptr()
                it.qt_hi, it.qt_lo, it.ldqt = K.ptr(f.qtb[0]), K.ptr(f.qtb[1]), f.qtb[0].stride(0)
            sk.append(it)
            # pairs by diagonal (tj - ti, then ti): blocks running together read tiles at many row and column
            # offsets, not one column band of Q (whose rows sit a power-of-two stride apart)
            t64 = cdiv(f.n, _capi.SKEW_TILE)
            (skw1 if f.rank1 else skw).extend((len(sk) - 1, (ti << 16) | (ti + d)) for d in range(t64)
                                              for ti in range(t64 - d))
        self.skew_dev = _upload(_capi.SkewItem, sk, dev)
        self.skew_work, self.skew_n = _work(skw, dev)
        self.skew1_work, self.skew1_n = _work(skw1, dev)
        # U12..U16: norm lower bound of Rn (skew)
        self.nlb_skh_dev, self.nlb_skh_n = self._nlb_prep(dense, skew=True)
        self.g_skh = self._nlb_chain(dense, skew=True)
        # U17: S = Rn Rn^T with sum(S .* Q) partials
        self.g_u17 = self.group([self.syrk(f.R, f.n, f.n, out_hi=f.T[0], out_lo=f.T[1])
                                 for f in dense])
        # U18: Procrustes step size
        si = []
        for f in dense:
            it = _capi.FactorItem()
            it.kind, it.n, it.nf, it.part, it.slots, it.ncols = (PSGD_FACTOR_SKEW, f.n, self.s(f, S_NF_SKH).data_ptr(),
                                                                f.pcs[3].data_ptr(), f.Tn, K_SUB)
            it.part_dot_rq, it.n_rq = f.r_dot.data_ptr(), f.r_dot.numel()
            it.part_dot_sq, it.n_sq = f.s_dot.data_ptr(), f.s_dot.numel()
            it.alpha, it.beta = self.s(f, S_AM).data_ptr(), self.s(f, S_BM).data_ptr()
            si.append(it)
        self.skf_dev, self.skf_n = _upload(_capi.FactorItem, si, dev), len(si)
        # sum S o Q for the step size: one row-major pass over the stored S and Q
        ti, tw = [], []
        for f in dense:
            it = _capi.TraceItem()
            it.q, it.n, it.part = f.q.data_ptr(), f.n, f.s_dot.data_ptr()
            it.s_hi, it.s_lo, it.lds = K.ptr(f.T[0]), K.ptr(f.T[1]), f.T[0].stride(0)
            ti.append(it)
            tw += [(len(ti) - 1, r0) for r0 in range(0, f.n, _capi.TRACE_ROWS)]
        self.trace_dev = _upload(_capi.TraceItem, ti, dev)
        self.trace_work, self.trace_n = _work(tw, dev)
        # U19: M = a/s Rn + a^2/(2 s^2) S (in place of Rn)
        ri, rw = [], []
        for f in dense:
            it = _capi.RotItem()
            it.n, it.r_hi, it.r_lo, it.ldr = f.n, K.ptr(f.R[0]), K.ptr(f.R[1]), f.R[0].stride(0)
            it.s_hi, it.s_lo, it.lds = K.ptr(f.T[0]), K.ptr(f.T[1]), f.T[0].stride(0)
            it.alpha, it.beta = self.s(f, S_AM).data_ptr(), self.s(f, S_BM).data_ptr()
            ri.append(it)
            rw += [(len(ri) - 1, r0) for r0 in range(0, f.n, _capi.ROT_ROWS)]
        self.rot_dev = _upload(_capi.RotItem, ri, dev)
        self.rot_work, self.rot_n = _work(rw, dev)
        # U20: Q <- Q - M Q
        self.g_u20 = self.group([self.spec(f.R, f.qtb, f.n, f.n, f.n, alpha=-1.0, beta=1.0, aux=f.q, out_f32=f.q,
                                           out_hi_t=f.qta[0], out_lo_t=f.qta[1]) for f in dense])
        # U22: P = Q^T Q
        self.g_u22 = self.group([self.syrk(f.qta, f.n, f.n, out_hi=f.P[0], out_lo=f.P[1]) for f in dense])

        # A1, A2: preconditioned gradient of the clean gradient, with sum-of-squares partials
        a1, a2 = [], []
        for p in P:
            if p.nd:
                continue
            n1, n2, f1, f2 = p.n1, p.n2, p.f1, p.f2
            if p.kind == ("dense", "dense"):
                a1.append(self.spec(p.gop_a, f2.P, n1, n2, n2, out_hi_t=p.yT[0], out_lo_t=p.yT[1]))
                bn = choose_bn(n2, split)
                p.apart = torch.zeros(cdiv(n1, BM) * cdiv(n2, bn), device=dev)
                a2.append(self.spec(f1.P, p.yT, n1, n2, n1, bn=bn, out_f32=p.pg32, part_tile=p.apart))
            elif p.kind in (("diag", "dense"), ("none", "dense")):
                bn = choose_bn(n2, split)
                p.apart = torch.zeros(cdiv(n1, BM) * cdiv(n2, bn), device=dev)
                a1.append(self.spec(p.gop_a, f2.P, n1, n2, n2, bn=bn, row_scale=f1.p if f1.kind == "diag" else None,
                                    out_f32=p.pg32, part_tile=p.apart))
            elif p.kind == ("dense", "diag"):
                bn = choose_bn(n2, split)
                p.apart = torch.zeros(cdiv(n1, BM) * cdiv(n2, bn), device=dev)
                a2.append(self.spec(f1.P, p.gop, n1, n2, n1, bn=bn, out_f32=p.pg32, part_tile=p.apart))
        self.g_a1, self.g_a1r = self.group([x for x in a1 if x.M >= BM]), self.group([x for x in a1 if x.M < BM])
        self.g_a2 = self.group(a2)
        # A3: clip + apply
        ai, aw = [], []
        for k, p in enumerate(P):
            it = _capi.ApplyItem()  # (an order-r parameter's apart holds the final layout change's chunk sums)
            it.param, it.param_bf16, it.numel = p.param.data_ptr(), int(p.param.dtype == torch.bfloat16), p.numel
            it.pg, it.part, it.nparts, it.scale = p.pg32.data_ptr(), p.apart.data_ptr(), p.apart.numel(), \
                self.clip[k:k + 1].data_ptr()
            ai.append(it)
            aw += [(k, c) for c in range(cdiv(p.numel, APPLY_CHUNK))]
        self.apply_dev, self.apply_n = _upload(_capi.ApplyItem, ai, dev), len(ai)
        self.apply_work, self.apply_nw = _work(aw, dev)
        # factor balancing of one parameter (launched only when its coin fires)
        self.balance = {}
        for k, p in enumerate(P):
            if len(p.factors) < 2:
                continue
            fl, wm, wa = [], [], []
            for f in p.factors:
                numel = f.n * f.n if f.kind == "dense" else f.n
                nparts = cdiv(numel, APPLY_CHUNK)
                f.bal = torch.zeros(nparts + 1, device=dev)  # per-chunk max |q|, then the multiplier
                it = _capi.BalanceFactor()
                it.q, it.n, it.dense = f.q.data_ptr(), f.n, int(f.kind == "dense")
                it.part, it.nparts, it.scale = f.bal.data_ptr(), nparts, f.bal[nparts:].data_ptr()
                if f.kind == "dense":
                    it.qt_hi, it.qt_lo, it.ldqt = K.ptr(f.qta[0]), K.ptr(f.qta[1]), f.qta[0].stride(0)
                    it.p_hi, it.p_lo, it.ldp = K.ptr(f.P[0]), K.ptr(f.P[1]), f.P[0].stride(0)
                    wa += [(len(fl), (ti << 16) | tj) for ti in range(f.T32) for tj in range(f.T32)]
                else:
                    it.pdiag = f.p.data_ptr()
                    wa += [(len(fl), c) for c in range(nparts)]
                wm += [(len(fl), c) for c in range(nparts)]
                fl.append(it)
            wmd, nwm = _work(wm, dev)
            wad, nwa = _work(wa, dev)
            self.balance[k] = (_upload(_capi.BalanceFactor, fl, dev),
                               _upload(_capi.BalanceParam, [_capi.BalanceParam(0, len(fl))], dev), wmd, nwm, wad, nwa)

    def _nd_chain(self, noisy, term1_specs=None):
        """Stages of the order-r parameters' preconditioner application Pg = G x_1 P_1 ... x_r P_r (psgd_pro.py:
        107-112), all such parameters together: stage j changes every parameter's tensor to the layout with its
        j-th dense mode (from the last) at the end, as an operand (the diagonal factors' q^2 multiplied in at the
        first change), then one GEMM group multiplies each by its P (fp32 out, same layout). The last stage brings Pg
        to what follows: for the update (noisy) one operand per dense mode with that mode first (term1 = its SYRK,
        appended to term1_specs) and per diagonal mode the row sums of squares of that layout; for the apply the
        natural fp32 Pg with chunk sums of squares for the clip. Returns ([(permute launch, GEMM group)], final
        permute launch); a permute launch is (item array, work list, count) or None."""
        dev = self.device
        nd = [p for p in self.params if p.nd]
        if not nd:
            return [], None
        per_stage, final = [], []
        for p in nd:
            dims = p.shape
            dense = [k for k in range(len(dims)) if p.factors[k].kind == "dense"][::-1]
            scales = [f.p if f.kind == "diag" else None for f in p.factors]
            src, last, pending = p.x32, None, scales
            for j, k in enumerate(dense):
                f = p.factors[k]
                it, units = _permute_item(src, dims, last, k, False, pending, op=p.op_last[k])
                out = p.ch[j % 2][:p.numel].view(p.numel // dims[k], dims[k])
                spec = self.spec(p.op_last[k], f.P, p.numel // dims[k], dims[k], dims[k], out_f32=out)
                while len(per_stage) <= j:
                    per_stage.append(([], [], []))
                per_stage[j][0].append(it)
                per_stage[j][1].append(units)
                per_stage[j][2].append(spec)
                src, last, pending = p.ch[j % 2], k, [None] * len(dims)
            if noisy:
                for k, f in enumerate(p.factors):
                    if f.kind == "dense":
                        it, units = _permute_item(src, dims, last, k, True, pending, op=p.op_first[k])
                        n, R = dims[k], p.numel // dims[k]
                        term1_specs.append(self.syrk(p.op_first[k], n, R, out_hi=f.T[0], out_lo=f.T[1],
                                                     part_row=f.t_rows, diag_out=f.t_diag))
                    else:
                        it, units = _permute_item(src, dims, last, k, True, pending, row_sq=p.t1_diag[k][0])
                        self.t1[f.fidx] = (p.t1_diag[k], 1)
                    final.append((it, units))
            else:
                it, units = _permute_item(src, dims, last, None, False, pending, out_f32=p.pg32, part=p.apart)
                final.append((it, units))

        def launch_of(items_units):
            items = [iu[0] for iu in items_units]
            work = [(i, u) for i, (_, n) in enumerate(items_units) for u in range(n)]
            w, nw = _work(work, dev)
            return (_upload(_capi.PermuteItem, items, dev), w, nw)
        stages = [(launch_of(list(zip(its, us))), self.group(specs)) for its, us, specs in per_stage]
        return stages, launch_of(final)

    def _permute(self, launch, what):
        if launch is not None and launch[2] > 0:
            check(_capi.lib().psgd_permute(launch[0].data_ptr(), launch[1].data_ptr(), launch[2], self.err.data_ptr(),
                                           K.stream_handle()), what)

    def _prep_fn(self, L):
        """The staging entry point: with momentum buffers in the items, the one that honours them."""
        return L.psgd_prep_momentum if self.mom_key and self.mom_key[0] else L.psgd_prep

    def _run_nd(self, stages, final, tr, tag):
        if not stages and final is None:
            return
        for j, (perm, grp) in enumerate(stages):
            self._permute(perm, "permute")
            tr(f"{tag}_permute{j}")
            self._launch(grp)
            tr(f"{tag}_product{j}")
        self._permute(final, "permute")
        tr(f"{tag}_permute_out")

    def _nlb_prep(self, fs, skew):
        """One item (one CTA) per factor, the largest factors first: the items are independent, and starting the
        longest CTAs in the first wave shortens the launch's tail."""
        items = []
        for f in sorted(fs, key=lambda f: -f.n):
            it = _capi.NlbPrepItem()
            A = f.R if skew else f.T
            it.a_hi, it.a_lo, it.lda, it.n, it.skew = K.ptr(A[0]), K.ptr(A[1]), A[0].stride(0), f.n, int(skew)
            if skew:
                it.part_row, it.row_slots = f.r_rows.data_ptr(), f.T32
                it.part_max, it.max_slots = f.r_max.data_ptr(), f.r_max.numel()
                it.v = f.v_skh.data_ptr()
                it.nf_out = self.s(f, S_NF_SKH).data_ptr()
            else:
                it.part_row, it.row_slots, it.diag = f.t_rows.data_ptr(), f.Ts, f.t_diag.data_ptr()
                it.v = f.v_spd.data_ptr()
                it.nf_out = self.s(f, S_NF_SPD).data_ptr()
            it.v0_hi, it.v0_lo, it.ldv = K.ptr(f.V0[0]), K.ptr(f.V0[1]), f.V0[0].stride(0)
            items.append(it)
        return _upload(_capi.NlbPrepItem, items, self.device), len(items)

    def _nlb_chain(self, fs, skew):
        """The four subspace products W = V A of the norm lower bound (psgd_pro.py:37-40) as N = 32 GEMMs
        W^T = A^T V^T; the 1/nf and row normalisations are column scales of the epilogue."""
        groups = []
        for k in range(4):
            specs = []
            for f in fs:
                A = f.R if skew else f.T
                src = (f.V0, f.Wa, f.Wb, f.Wa)[k]
                dst = (f.Wa, f.Wb, f.Wa, None)[k]
                pc = f.pcs if skew else f.pc
                nf = self.s(f, S_NF_SKH if skew else S_NF_SPD)
                kw = dict(alpha=-1.0 if skew else 1.0, cs_nf=nf)
                if k in (0, 2):
                    kw.update(cs_mode=1, part_col=pc[k])
                else:
                    kw.update(cs_mode=2, cs_part=pc[k - 1], cs_T=f.Tn)
                    if k == 3:
                        kw.update(part_col=pc[3])
                if dst is not None:
                    kw.update(out_hi_t=dst[0], out_lo_t=dst[1])
                specs.append(self.spec(A, src, f.n, K_SUB, f.n, bn=32, **kw))
            groups.append(self.group(specs))
        return groups

    def update_grad_ptrs(self, grads):
        """Re-point the staging items at this step's gradient tensors (only when their addresses changed). The item
        arrays of each address set are built on the device once; switching sets is a device-to-device copy into
        the live arrays (stream-ordered, no host wait, captured graphs stay valid)."""
        ptrs = tuple(t.data_ptr() for t in grads)
        if ptrs == self.grad_ptrs:
            return
        cached = self._ptr_items.get(ptrs)
        if cached is None:
            cached = []
            for items in (self.prep_u, self.prep_a):
                for it, t in zip(items, grads):
                    it.g, it.g_bf16 = t.data_ptr(), int(t.dtype == torch.bfloat16)
                cached.append(_upload(_capi.PrepItem, items, self.device))
            if len(self._ptr_items) >= 8:  # a handful of gradient buffers in rotation at most
                self._ptr_items.clear()
            self._ptr_items[ptrs] = cached
        self.prep_u_dev.copy_(cached[0], non_blocking=True)
        self.prep_a_dev.copy_(cached[1], non_blocking=True)
        self.grad_ptrs = ptrs

    # ---- launches ------------------------------------------------------------------------------------------------
    def _launch(self, g):
        if g is not None:
            g.launch(self.err)

    def run_update(self, trace=None):
        """The update phases in order; trace(name) (debugging) is called after each launch."""
        L, st, err, hy = _capi.lib(), K.stream_handle(), self.err.data_ptr(), self.hyper.data_ptr()
        tr = trace or (lambda name: None)
        check(self._prep_fn(L)(self.prep_u_dev.data_ptr(), self.prep_u_work.data_ptr(), self.prep_u_n, hy, err, st), "prep")
        tr("prep")
        self._run_nd(self.nd_u, self.nd_t1, tr, "nd")
        self._launch(self.g_u1)
        tr("u1")
        self._launch(self.g_u1r)
        tr("u1_r1")
        self._launch(self.g_u2)
        tr("u2")
        self._launch(self.g_u3)
        tr("term1")
        self._launch(self.g_u3r)
        tr("term1_r1")
        check(L.psgd_nlb_prep(self.nlb_spd_dev.data_ptr(), self.nlb_spd_n, err, st), "nlb_prep spd")
        tr("nlb_prep_spd")
        for k, g in enumerate(self.g_spd):
            self._launch(g)
            tr(f"nlb_spd{k}")
        check(L.psgd_factor_update(self.fac_dev.data_ptr(), self.fac_n, hy, err, st), "factor_update")
        tr("factor")
        self._launch(self.g_u10)
        tr("qupdate")
        check(L.psgd_skew(self.skew_dev.data_ptr(), self.skew_work.data_ptr(), self.skew_n, err, st), "skew")
        tr("skew")
        check(L.psgd_skew_rank1(self.skew_dev.data_ptr(), self.skew1_work.data_ptr(), self.skew1_n, err, st), "skew r1")
        tr("skew_r1")
        check(L.psgd_nlb_prep(self.nlb_skh_dev.data_ptr(), self.nlb_skh_n, err, st), "nlb_prep skh")
        tr("nlb_prep_skh")
        for k, g in enumerate(self.g_skh):
            self._launch(g)
            tr(f"nlb_skh{k}")
        self._launch(self.g_u17)
        tr("S")
        check(L.psgd_trace(self.trace_dev.data_ptr(), self.trace_work.data_ptr(), self.trace_n, int(self.split == 3),
                           err, st), "trace")
        tr("trace")
        check(L.psgd_factor_update(self.skf_dev.data_ptr(), self.skf_n, hy, err, st), "procrustes scalars")
        tr("procrustes_scalars")
        check(L.psgd_rot(self.rot_dev.data_ptr(), self.rot_work.data_ptr(), self.rot_n, int(self.split == 3), err, st),
              "rot")
        tr("rot")
        self._launch(self.g_u20)
        tr("procrustes")
        self._launch(self.g_u22)
        tr("gram")

    def run_apply(self, trace=None, after_update=False):
        """The parameter update. after_update: the update phases ran earlier in this step, so their staging pass
        already wrote the clean operands it could (fuse_stage) and only the other parameters are staged here."""
        L, st, err, hy = _capi.lib(), K.stream_handle(), self.err.data_ptr(), self.hyper.data_ptr()
        tr = trace or (lambda name: None)
        work, nwork = (self.prep_a_rest_work, self.prep_a_rest_n) if after_update and self.fuse_stage else \
            (self.prep_a_work, self.prep_a_n)
        if nwork:
            check(self._prep_fn(L)(self.prep_a_dev.data_ptr(), work.data_ptr(), nwork, hy, err, st), "prep")
        tr("a_prep")
        self._run_nd(self.nd_a[0], self.nd_a[1], tr, "a_nd")
        self._launch(self.g_a1)
        tr("a1")
        self._launch(self.g_a1r)
        tr("a1_r1")
        self._launch(self.g_a2)
        tr("a2")
        check(L.psgd_apply(self.apply_dev.data_ptr(), self.apply_n, self.apply_work.data_ptr(), self.apply_nw, hy,
                           err, st), "apply")
        tr("apply")

    def phase_groups(self):
        """(name, GemmGroup) of every tensor-core phase, in the names run_update / run_apply trace."""
        out = [("u1", self.g_u1), ("u1_r1", self.g_u1r), ("u2", self.g_u2), ("term1", self.g_u3),
               ("term1_r1", self.g_u3r)]
        out += [(f"nlb_spd{k}", g) for k, g in enumerate(self.g_spd)]
        out += [("qupdate", self.g_u10)]
        out += [(f"nlb_skh{k}", g) for k, g in enumerate(self.g_skh)]
        out += [("S", self.g_u17), ("procrustes", self.g_u20), ("gram", self.g_u22), ("a1", self.g_a1),
                ("a1_r1", self.g_a1r),
                ("a2", self.g_a2)]
        out += [(f"nd_product{j}", g) for j, (_, g) in enumerate(self.nd_u)]
        out += [(f"a_nd_product{j}", g) for j, (_, g) in enumerate(self.nd_a[0])]
        return [(n, g) for n, g in out if g is not None]

    def launches_per_step(self, update=True, update_first=True):
        """Kernels of libpsgd_b200.so launched by one step (the RNG fill of the update uses torch's kernels)."""
        a_prep = self.prep_a_rest_n if (update and update_first and self.fuse_stage) else self.prep_a_n
        n = 2 + int(a_prep > 0)  # clip scale, apply, the apply's staging
        groups = [self.g_a1, self.g_a1r, self.g_a2]
        nd_perm = lambda stages, final: sum(int(p is not None and p[2] > 0) for p, _ in stages) + \
            int(final is not None and final[2] > 0)
        n += nd_perm(*self.nd_a)
        groups += [g for _, g in self.nd_a[0]]
        if update:
            n += nd_perm(self.nd_u, self.nd_t1)
            groups += [g for _, g in self.nd_u]
            n += 1  # prep
            n += int(self.nlb_spd_n > 0) + int(self.nlb_skh_n > 0)  # norm-bound starts
            n += 2 * int(self.fac_n > 0) + 2 * int(self.skf_n > 0)  # factor scalars: two launches each
            n += int(self.skew_n > 0) + int(self.skew1_n > 0) + int(self.rot_n > 0)  # skew (two kinds), rot
            n += int(self.trace_n > 0)  # trace of S o Q
            groups += [self.g_u1, self.g_u1r, self.g_u2, self.g_u3, self.g_u3r, self.g_u10, self.g_u17, self.g_u20,
                       self.g_u22]
            groups += self.g_spd + self.g_skh
        return n + sum(g is not None for g in groups)


class KronWhiten:
    """psgd_pro.KronWhiten (psgd_pro.py:251-384) on B200. Same constructor arguments and mutable attributes
    (lr_params, lr_preconditioner, betaL, damping, momentum, grad_clip_max_amps,
    preconditioner_update_probability, update_preconditioner_first), step(closure) and step_math(grads) of
    psgd_pro_fast.py:440-499. Extra keyword arguments: precision ("fp32", "bf16" or None = from the parameter
    dtype) and cuda_graphs (capture the step after the first call).

    The keyword arguments psgd_pro_fast.KronWhiten adds (psgd_pro_fast.py:245-264) are accepted, so its callers
    drop in; the B200 step subsumes what they select, and the two argument checks of the reference are kept:
      compile    (None, a torch.compile mode or options): the step is captured in CUDA graphs whatever the value;
      ops        (EagerOps or a kernel class): the dense-factor arithmetic always runs in this package's kernels;
      batch      same-shape parameters always share one grouped launch per phase (no vmap stacking);
      cache_p, p2d   P_i = Q_i^T Q_i is always kept as state between steps (psgd_pro_fast.py:164-192);
      graph_rng  the damping noise is always generated on the device (in the staging kernel);
      r2         the Procrustes step always takes the one-product form of psgd_pro_fast.py:141-153 (r2=False selects
                 the two-product form of :129-138 there; the two differ in rounding only)."""

    def __init__(self, params_with_grad, preconditioner_max_size=float("inf"), preconditioner_max_skew=1.0,
                 preconditioner_init_scale=None, lr_params=0.001, lr_preconditioner=0.1, betaL=0.9, damping=1e-9,
                 momentum=0.0, grad_clip_max_amps=(2.0, 10.0), preconditioner_update_probability=1.0,
                 update_preconditioner_first=True, whiten_grad=True, compile=None, ops=None, batch=False,
                 cache_p=False, graph_rng=False, p2d=False, r2=False, precision=None, cuda_graphs=True):
        # psgd_pro_fast.py:289, :294: the reference's own argument checks
        assert not (cache_p and compile is not None), "cache_p relies on tensor version counters: eager only"
        assert not (p2d and batch), "p2d keeps per-parameter P state; batch stacks parameters"
        self.ops = ops  # kept for callers that read it back; the arithmetic does not go through it
        self.lr_params = lr_params
        self.lr_preconditioner = lr_preconditioner
        self.betaL = betaL
        self.damping = damping
        self.momentum = momentum if (0 < momentum < 1) else 0.0
        self.grad_clip_max_amps = grad_clip_max_amps
        self.preconditioner_update_probability = preconditioner_update_probability
        self.update_preconditioner_first = update_preconditioner_first
        self._preconditioner_max_size = preconditioner_max_size
        self._preconditioner_max_skew = preconditioner_max_skew
        params_with_grad = [params_with_grad] if isinstance(params_with_grad, torch.Tensor) else params_with_grad
        self._params_with_grad = [p for p in params_with_grad if p.requires_grad]
        if not self._params_with_grad:
            raise ValueError("no parameter requires grad")
        dev = self._params_with_grad[0].device
        if dev.type != "cuda":
            raise RuntimeError("psgd_pro_b200.KronWhiten runs on CUDA devices only (there is no CPU fallback)")
        for p in self._params_with_grad:
            if p.dtype not in (torch.float32, torch.bfloat16) or not p.is_contiguous() or p.device != dev:
                raise ValueError("parameters must be contiguous fp32 or bf16 tensors on one CUDA device")
        self._device = dev
        if precision is None:
            precision = "bf16" if self._params_with_grad[0].dtype == torch.bfloat16 else "fp32"
        if precision not in ("fp32", "bf16"):
            raise ValueError("precision must be 'fp32' or 'bf16'")
        self.precision = precision
        self._split = 3 if precision == "fp32" else 1
        self._whiten_grad = whiten_grad
        if not whiten_grad:
            assert self.momentum > 0, "Cannot whiten momentum if the momentum setting is invalid."
        self._init_scale = preconditioner_init_scale
        self._plan = None
        self._ms, self._counter_m = None, 0
        self._use_graphs = cuda_graphs
        self._graphs = {}
        self._hyper_host = None
        self._steps = 0
        self._noise_key = None  # key word of the in-kernel noise generator, drawn from torch's RNG at the first step
        self.trace = None  # optional callable(name) run after every launch (profiling; disables graphs)
        _capi.lib()  # fail loudly now if the kernels are missing
        if preconditioner_init_scale is not None:
            self._build(preconditioner_init_scale)

    # ---- state ---------------------------------------------------------------------------------------------
    @property
    def param_groups(self):
        """A read-only view of the hyper-parameters in torch.optim's shape (the attributes stay the source)."""
        return [dict(params=self._params_with_grad, lr=self.lr_params, lr_preconditioner=self.lr_preconditioner,
                     betaL=self.betaL, damping=self.damping, momentum=self.momentum,
                     grad_clip_max_amps=self.grad_clip_max_amps,
                     preconditioner_update_probability=self.preconditioner_update_probability)]

    def set_init_scale(self, scale):
        """Initialises the preconditioner with Q factors scale^(1/order) I (psgd_pro.py:181, :210) before the first
        step, as preconditioner_init_scale would; used when the scale comes from gradients this optimizer does
        not see (a rank of a sharded step takes it over every parameter's gradient, psgd_pro.py:329-332)."""
        if self._plan is not None:
            raise RuntimeError("the preconditioner is already initialised")
        self._build(float(scale))

    def _build(self, scale):
        shapes = [tuple(p.squeeze().shape) for p in self._params_with_grad]
        self._plan = _Plan(self._params_with_grad, shapes, float(scale), self._preconditioner_max_size,
                           self._preconditioner_max_skew, self._split, self._device)
        self._graphs = {}

    def state_dict(self):
        """Per parameter {"Q": [q_0, ...], "L": [l_0, ...], "m": momentum or None} in parameter order (the
        reference's Q and L of self._QLs_exprs[i][0], psgd_pro.py:306), plus counter_m."""
        out = []
        if self._plan is None:
            return {"state": None, "counter_m": self._counter_m}
        for k, p in enumerate(self._plan.params):
            Q = [f.q.view(()) if (len(p.shape) == 0) else f.q for f in p.factors]
            L = [self._plan.L[f.fidx] for f in p.factors]
            m = self._ms[k] if self._ms is not None else None
            out.append({"Q": Q, "L": L, "m": m})
        return {"state": out, "counter_m": self._counter_m}

    def load_state_dict(self, sd):
        """Restores Q, L (and momentum) saved by state_dict (or taken from a reference KronWhiten's
        _QLs_exprs), rebuilding the operand copies (Q^T, P = Q^T Q) from the loaded Q."""
        if sd["state"] is None:
            self._plan = None
            return
        if self._plan is None:
            self._build(1.0)
        for k, (p, st) in enumerate(zip(self._plan.params, sd["state"])):
            for f, q, l in zip(p.factors, st["Q"], st["L"]):
                f.q.copy_(torch.as_tensor(q).reshape(f.q.shape).to(f.q))
                self._plan.L[f.fidx].copy_(torch.as_tensor(l).to(self._plan.L))
                if f.kind == "dense":
                    f.refresh_operands()
                else:
                    f.p.copy_(f.q * f.q)
            if st.get("m") is not None:
                m = torch.as_tensor(st["m"]).to(self._device)
                if self._ms is None:
                    self._ms = [torch.zeros(q.squeeze().shape, dtype=m.dtype, device=self._device)
                                for q in self._params_with_grad]
                if self._ms[k].dtype != m.dtype or self._ms[k].shape != m.shape:
                    self._ms[k] = torch.zeros(m.shape, dtype=m.dtype, device=self._device)
                self._ms[k].copy_(m)
        self._counter_m = sd.get("counter_m", 0)
        self._graphs = {}

    # ---- the step ------------------------------------------------------------------------------------------
    def _set_hyper(self, beta_m=0.0, noise=None, ema_phase=0):
        """Device hyper-parameter vector. noise: None (the damping noise is read from the draws buffer) or the
        (key0, key1) of the in-kernel generator; ema_phase: the staging pass that applies the momentum EMA."""
        h = [0.0] * HY_COUNT
        h[HY_LR_PRECOND], h[HY_BETA_L], h[HY_DAMPING] = self.lr_preconditioner, self.betaL, self.damping
        h[HY_LR_PARAMS] = self.lr_params
        h[HY_MAX_AVG], h[HY_MAX_ELEM] = self.grad_clip_max_amps
        h[HY_MOM_BETA], h[HY_MOM_ALPHA] = beta_m, 1 - beta_m  # psgd_pro.py:341: mul_(beta).add_(g, alpha=1 - beta)
        h[HY_EMA_PHASE] = float(ema_phase)
        bits = [struct.unpack("<i", struct.pack("<f", float(x)))[0] for x in h]
        if noise is not None:
            bits[HY_NOISE] = struct.unpack("<i", struct.pack("<f", 1.0))[0]
            bits[HY_NOISE_KEY0], bits[HY_NOISE_KEY1] = (struct.unpack("<i", struct.pack("<I", k & 0xFFFFFFFF))[0]
                                                        for k in noise)
        bits = tuple(bits)
        if bits != self._hyper_host:
            self._plan.hyper.view(torch.int32).copy_(torch.tensor(bits, dtype=torch.int32))
            self._hyper_host = bits

    def _balance(self, ks):
        """psgd_pro.py:96-105 for the parameters ks whose coin fired (probability 0.01 each per step): one
        psgd_balance call per parameter rescales its factors and their Q^T / P operand copies on the device, from
        item arrays and work lists encoded when the plan was built."""
        plan = self._plan
        for k in ks:
            b = plan.balance.get(k)
            if b is None:  # order-1 preconditioners are left alone (psgd_pro.py:101)
                continue
            fdev, pdev, wmd, nwm, wad, nwa = b
            check(_capi.lib().psgd_balance(fdev.data_ptr(), pdev.data_ptr(), 1, wmd.data_ptr(), nwm,
                                           wad.data_ptr(), nwa, plan.err.data_ptr(), K.stream_handle()), "balance")

    def _phase(self, name, fn):
        if not self._use_graphs:
            return fn()
        g = self._graphs.get(name)
        if g is None:
            if self._steps < 1:  # first call runs eagerly (sets kernel attributes, validates the plan)
                return fn()
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(self._device)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                with torch.cuda.graph(g, stream=side):
                    fn()
            torch.cuda.current_stream().wait_stream(side)
            self._graphs[name] = g
        g.replay()

    @torch.no_grad()
    def step_math(self, grads, draws=None):
        """The step after the gradients exist (psgd_pro_fast.py:440-490). draws (tests): {"update": u,
        "coins": [c per param], "normals": [[xi, V_spd, V_skh per dense factor ...] per param]} replaces the
        random draws (the update runs when u < preconditioner_update_probability, balancing when c < 0.01)."""
        grads = [g.squeeze() for g in grads]
        if len(grads) != len(self._params_with_grad):
            raise ValueError("one gradient per parameter is required")
        for g, p in zip(grads, self._params_with_grad):
            if g.device != self._device or g.dtype not in (torch.float32, torch.bfloat16):
                raise ValueError("gradients must be fp32 or bf16 tensors on the parameters' device")
        grads = [g if g.is_contiguous() else g.contiguous() for g in grads]
        if self._plan is None:
            self._build(init_scale_from_grads(grads, self.damping))
        plan = self._plan
        beta = 0.0
        if self.momentum > 0:  # psgd_pro.py:334-343; the EMA itself runs in the staging kernel
            beta = min(self._counter_m / (1 + self._counter_m), self.momentum)
            if self._ms is None or any(m.dtype != g.dtype or m.shape != g.shape for m, g in zip(self._ms, grads)):
                self._ms = [torch.zeros_like(g) for g in grads]
            elif self._counter_m == 0:  # momentum (re)started: the reference starts from zeros
                for m in self._ms:
                    m.zero_()
            self._counter_m += 1
        else:
            self._ms, self._counter_m = None, 0
        ms = self._ms if self.momentum > 0 else None
        key = (ms is not None, bool(self._whiten_grad))
        stale = ms is not None and plan.ms_ptrs != [m.data_ptr() for m in ms]
        if plan.grad_ptrs is None or plan.mom_key != key or stale:
            eps = [torch.finfo(g.dtype).eps for g in grads]  # psgd_pro.py:122
            plan.build(grads, ms, self._whiten_grad, eps)
            plan.ms_ptrs = [m.data_ptr() for m in ms] if ms is not None else None
            self._graphs = {}
        elif tuple(t.data_ptr() for t in grads) != plan.grad_ptrs:
            plan.update_grad_ptrs(grads)
        if draws is None and self._noise_key is None:
            self._noise_key = int(torch.randint(0, 2 ** 31, (1,)).item())
        if draws is None:
            update = bool(torch.rand([]) < self.preconditioner_update_probability)
            coins = (torch.rand(len(plan.params)) < 0.01).tolist() if update else []
            use_graph = True
        else:
            update = draws["update"] < self.preconditioner_update_probability
            coins = [c < 0.01 for c in draws["coins"]] if update else []
            use_graph = False
            if update:
                self._load_draws(draws["normals"])
        # the momentum EMA runs in the first staging pass of this step that reads the momentum
        ema_phase = 1 if (ms is not None and not self._whiten_grad and update and self.update_preconditioner_first) \
            else 0
        self._set_hyper(beta, noise=(self._noise_key, self._steps) if draws is None else None, ema_phase=ema_phase)

        trace = self.trace
        if trace is not None:
            use_graph = False  # launch-level CUDA events need eager launches
            trace("start")

        def upd():
            if draws is None:  # the damping noise comes from the prep kernel's generator
                plan.vbuf.normal_()
                if trace is not None:
                    trace("rng")
            plan.run_update(trace)

        after = update and self.update_preconditioner_first

        def app():
            plan.run_apply(trace, after_update=after)

        run = (lambda name, fn: self._phase(name, fn)) if use_graph else (lambda name, fn: fn())
        fired = [k for k, c in enumerate(coins) if c]
        def bal():
            self._balance(fired)
            if trace is not None:
                trace("balance")

        if after:
            run("update", upd)
            bal()
        run("apply_after_update" if after else "apply", app)
        if update and not self.update_preconditioner_first:
            run("update", upd)
            bal()
        self._steps += 1

    def _load_draws(self, normals):
        plan = self._plan
        for p, nd in zip(plan.params, normals):
            it = iter(nd)
            p.xi.copy_(torch.as_tensor(next(it)).reshape(p.n1, p.n2))
            for f in p.factors:
                if f.kind == "dense":
                    f.v_spd.copy_(torch.as_tensor(next(it)))
                    f.v_skh.copy_(torch.as_tensor(next(it)))

    @torch.no_grad()
    def step(self, closure):
        """psgd_pro.py:319-384: evaluates the closure, takes the gradients, runs step_math; returns the closure's
        return value."""
        with torch.enable_grad():
            closure_returns = closure()
            loss = closure_returns if isinstance(closure_returns, torch.Tensor) else closure_returns[0]
            grads = torch.autograd.grad(loss, self._params_with_grad)
        self.step_math(grads)
        return closure_returns

    def check_errors(self):
        """Raises if a kernel recorded a device-side error: a bounded wait that gave up, or a factor whose L or
        Procrustes step came out NaN or infinite (a diverging run; the reference would carry the NaN on)."""
        if self._plan is not None:
            e = int(self._plan.err.item())
            if e:
                raise RuntimeError(f"psgd_pro_b200: device error flags {e:#x}: {_capi.describe_err(e)}")

    def clear_errors(self):
        if self._plan is not None:
            self._plan.err.zero_()
