"""Thin torch-facing wrappers around the C ABI (include/psgd_b200.h): tensors in, device pointers and sizes out.
Every call runs on the current CUDA stream and checks the return code; nothing here computes on the host."""
import ctypes

import torch

from . import _capi
from ._capi import GemmSpec, PSGD_GEMM_PLAIN, PSGD_GEMM_SYRK, PSGD_GEMM_TRMM, check

BF16 = torch.bfloat16


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_handle():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def pad8(n):
    return (n + 7) // 8 * 8


def operand(rows, cols, device, split=True):
    """(hi, lo) bf16 buffers for a rows x cols operand with a 16-byte aligned leading dimension (lo None when
    split is False). The padding columns are zero and stay zero (TMA reads only `cols` columns)."""
    ld = pad8(max(cols, 1))
    hi = torch.zeros(rows, ld, dtype=BF16, device=device)
    lo = torch.zeros(rows, ld, dtype=BF16, device=device) if split else None
    return hi, lo


def split_into(x, hi, lo):
    """hi[:, :c] = bf16(x), lo[:, :c] = bf16(x - hi) (torch ops; test and plug-in helper)."""
    r, c = x.shape
    h = x.to(BF16)
    hi[:r, :c].copy_(h)
    if lo is not None:
        lo[:r, :c].copy_((x - h.float()).to(BF16))


def make_spec(a, b, M, N, K, bn=128, mode=PSGD_GEMM_PLAIN, alpha=1.0, beta=0.0, alpha_ptr=None, beta_ptr=None,
              aux=None, row_scale=None, col_scale=None, out_f32=None, out_hi=None, out_lo=None, out_hi_t=None,
              out_lo_t=None, part_tile=None, part_col=None, part_row=None, diag_out=None, dot_aux=None,
              part_dot=None, cs_part=None, cs_T=0, cs_mode=0, cs_nf=None, out_packed=None):
    """GemmSpec for D = A B^T with a = (a_hi, a_lo), b = (b_hi, b_lo) bf16 operands (lo may be None)."""
    a_hi, a_lo = a
    b_hi, b_lo = b
    s = GemmSpec()
    s.a_hi, s.a_lo, s.lda = ptr(a_hi), ptr(a_lo), a_hi.stride(0)
    s.b_hi, s.b_lo, s.ldb = ptr(b_hi), ptr(b_lo), b_hi.stride(0)
    s.M, s.N, s.K, s.bn, s.mode = M, N, K, bn, mode
    s.alpha, s.beta = alpha, beta
    s.alpha_ptr, s.beta_ptr = ptr(alpha_ptr), ptr(beta_ptr)
    s.aux, s.ld_aux = ptr(aux), (aux.stride(0) if aux is not None else 0)
    s.row_scale, s.col_scale = ptr(row_scale), ptr(col_scale)
    s.out_f32, s.ld_f32 = ptr(out_f32), (out_f32.stride(0) if out_f32 is not None else 0)
    s.out_hi, s.out_lo = ptr(out_hi), ptr(out_lo)
    s.ld_b = out_hi.stride(0) if out_hi is not None else 0
    s.out_hi_t, s.out_lo_t = ptr(out_hi_t), ptr(out_lo_t)
    s.ld_bt = out_hi_t.stride(0) if out_hi_t is not None else 0
    s.part_tile, s.part_col, s.part_row, s.diag_out = ptr(part_tile), ptr(part_col), ptr(part_row), ptr(diag_out)
    s.dot_aux, s.ld_dot, s.part_dot = ptr(dot_aux), (dot_aux.stride(0) if dot_aux is not None else 0), ptr(part_dot)
    s.cs_part, s.cs_T, s.cs_mode, s.cs_nf = ptr(cs_part), cs_T, cs_mode, ptr(cs_nf)
    s.out_packed = ptr(out_packed)
    return s


def gemm(spec, split, err):
    """One problem, launched on the current stream. err: int32 CUDA tensor (device error word)."""
    check(_capi.lib().psgd_gemm(ctypes.byref(spec), split, ptr(err), stream_handle()), "psgd_gemm")


class GemmGroup:
    """Many problems encoded once (descriptor table and tile list copied to device buffers owned here) and
    launched as one persistent grid, any number of times (CUDA-graph capturable)."""

    def __init__(self, specs, split, device, keep=()):
        L = _capi.lib()
        self.keep = list(keep)  # tensors the specs point into (raw pointers do not keep them alive)
        self.split, self.n = split, len(specs)
        self.specs = (GemmSpec * len(specs))(*specs)
        nbytes = L.psgd_gemm_table_bytes(len(specs))
        ntiles_max = L.psgd_gemm_count_tiles(self.specs, len(specs))
        check(min(ntiles_max, 0), "psgd_gemm_count_tiles")
        host_table = torch.empty(nbytes + 64, dtype=torch.uint8)
        off = (-host_table.data_ptr()) % 64
        host_table = host_table[off:off + nbytes]
        host_tiles = torch.empty(2 * max(ntiles_max, 1), dtype=torch.int32)
        nt, kind = ctypes.c_int(0), ctypes.c_int(0)
        check(L.psgd_gemm_encode(self.specs, len(specs), host_table.data_ptr(), nbytes, host_tiles.data_ptr(),
                                 ntiles_max, ctypes.byref(nt), ctypes.byref(kind)), "psgd_gemm_encode")
        self.ntiles, self.kind = nt.value, kind.value
        self.flops = sum((s.M * s.M * s.K) if s.mode == PSGD_GEMM_SYRK else (2 * s.M * s.N * s.K) for s in specs)
        self.table = host_table.to(device)
        self.tiles = host_tiles[:2 * max(self.ntiles, 1)].to(device)
        assert self.table.data_ptr() % 64 == 0

    def launch(self, err):
        check(_capi.lib().psgd_gemm_launch(self.table.data_ptr(), self.tiles.data_ptr(), self.ntiles, self.split,
                                           self.kind, ptr(err), stream_handle()), "psgd_gemm_launch")


_WORK = {}  # device work lists by (rows, cols, row path, device): built once per shape (read-only afterwards)


def _prep_work(rows, cols, normal, dev):
    key = (rows, cols, normal, dev)
    w = _WORK.get(key)
    if w is None:
        if normal:  # (0, row block)
            nb = (rows + _capi.PREP_ROWS - 1) // _capi.PREP_ROWS
            w = torch.stack([torch.zeros(nb, dtype=torch.int32), torch.arange(nb, dtype=torch.int32)], 1)
        else:  # (0, (ti << 16) | tj) over the 32 x 32 tiles
            ti = torch.arange((rows + 31) // 32, dtype=torch.int32)
            tj = torch.arange((cols + 31) // 32, dtype=torch.int32)
            code = ((ti[:, None] << 16) | tj[None, :]).reshape(-1)
            w = torch.stack([torch.zeros_like(code), code], 1)
        w = (w.reshape(-1).to(dev), w.shape[0])
        if len(_WORK) > 256:
            _WORK.clear()
        _WORK[key] = w
    return w


def _prep_one(item_fields, rows, cols, normal, err=None):
    """One psgd_prep launch for a single item (plug-in helpers; item and work list uploaded per call). err: the
    device error word to report into (a fresh one when None)."""
    it = _capi.PrepItem()
    for k, v in item_fields.items():
        setattr(it, k, v)
    dev = torch.device("cuda", torch.cuda.current_device())
    host = torch.empty(ctypes.sizeof(it), dtype=torch.uint8)
    ctypes.memmove(host.data_ptr(), ctypes.addressof(it), ctypes.sizeof(it))
    items = host.to(dev)
    work, nwork = _prep_work(rows, cols, normal, dev)
    hyper = torch.zeros(_capi.HY_COUNT, device=dev)
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
    check(_capi.lib().psgd_prep(items.data_ptr(), work.data_ptr(), nwork, hyper.data_ptr(), err.data_ptr(),
                                stream_handle()), "psgd_prep")
    return (items, work, hyper, err)  # kept alive by the caller until the launch has run


def to_operand(X, transpose=False, split=True, err=None):
    """(hi, lo) bf16 operand of the fp32 / bf16 matrix X (or of X^T), staged by the psgd_prep kernel."""
    X = X.contiguous()
    r, c = X.shape
    hi, lo = operand(c, r, X.device, split) if transpose else operand(r, c, X.device, split)
    keep = _prep_one(dict(g=X.data_ptr(), g_bf16=int(X.dtype == BF16), mode=_capi.PSGD_PREP_TRANS if transpose
                          else _capi.PSGD_PREP_NORMAL, xi=None, n1=r, n2=c, p1=None, p2=None, out_hi=ptr(hi),
                          out_lo=ptr(lo), ld_out=hi.stride(0), eps=0.0), r, c, not transpose, err)
    return (hi, lo), keep
