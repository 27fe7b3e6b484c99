"""ctypes binding of libpsgd_b200.so (the C ABI declared in include/psgd_b200.h).

The library is built in-tree (psgd_pro_b200/_lib/libpsgd_b200.so). There is no fallback: when the library is
missing or a call fails, a RuntimeError says so."""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("PSGD_B200_LIB") or os.path.join(_HERE, "_lib", "libpsgd_b200.so")  # env: another build

c_vp, c_ll, c_int, c_float = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_float
c_fp = ctypes.POINTER(ctypes.c_float)

ERRORS = {-1: "invalid argument (shape, stride, alignment or mode)", -2: "CUDA launch failed",
          -3: "TMA descriptor encoding failed", -4: "caller table or workspace too small",
          -5: "size beyond the fixed scratch of the no-allocation entry point"}

PSGD_GEMM_PLAIN, PSGD_GEMM_SYRK, PSGD_GEMM_TRMM = 0, 1, 2


class GemmSpec(ctypes.Structure):
    """Mirror of PsgdGemmSpec (include/psgd_b200.h); field order and types must match exactly."""
    _fields_ = [
        ("a_hi", c_vp), ("a_lo", c_vp), ("lda", c_ll),
        ("b_hi", c_vp), ("b_lo", c_vp), ("ldb", c_ll),
        ("M", c_int), ("N", c_int), ("K", c_int),
        ("bn", c_int), ("mode", c_int),
        ("alpha", c_float), ("beta", c_float),
        ("alpha_ptr", c_vp), ("beta_ptr", c_vp),
        ("aux", c_vp), ("ld_aux", c_ll),
        ("row_scale", c_vp), ("col_scale", c_vp),
        ("out_f32", c_vp), ("ld_f32", c_ll),
        ("out_hi", c_vp), ("out_lo", c_vp), ("ld_b", c_ll),
        ("out_hi_t", c_vp), ("out_lo_t", c_vp), ("ld_bt", c_ll),
        ("part_tile", c_vp), ("part_col", c_vp), ("part_row", c_vp), ("diag_out", c_vp),
        ("dot_aux", c_vp), ("ld_dot", c_ll), ("part_dot", c_vp),
        ("cs_part", c_vp), ("cs_T", c_int), ("cs_mode", c_int), ("cs_nf", c_vp),
        ("out_packed", c_vp),
    ]


class PrepItem(ctypes.Structure):
    _fields_ = [("g", c_vp), ("g_bf16", c_int), ("mode", c_int), ("xi", c_vp), ("n1", c_int), ("n2", c_int),
                ("p1", c_vp), ("p2", c_vp), ("out_hi", c_vp), ("out_lo", c_vp), ("ld_out", c_ll),
                ("out_f32", c_vp), ("part_row", c_vp), ("part_col", c_vp), ("part_tile", c_vp), ("eps", c_float),
                ("noise_base", c_ll), ("m", c_vp), ("mom_phase", c_int), ("out2_hi", c_vp), ("out2_lo", c_vp)]


class NlbPrepItem(ctypes.Structure):
    _fields_ = [("a_hi", c_vp), ("a_lo", c_vp), ("lda", c_ll), ("n", c_int), ("skew", c_int),
                ("part_row", c_vp), ("row_slots", c_int), ("diag", c_vp), ("part_max", c_vp), ("max_slots", c_int),
                ("v", c_vp), ("v0_hi", c_vp), ("v0_lo", c_vp), ("ldv", c_ll), ("nf_out", c_vp)]


class FactorItem(ctypes.Structure):
    _fields_ = [("kind", c_int), ("n", c_int), ("term2", c_float), ("L", c_vp), ("nf", c_vp), ("part", c_vp),
                ("slots", c_int), ("ncols", c_int), ("alpha", c_vp), ("beta", c_vp), ("q", c_vp), ("p", c_vp),
                ("part_dot_rq", c_vp), ("n_rq", c_int), ("part_dot_sq", c_vp), ("n_sq", c_int), ("scratch", c_vp)]


class SkewItem(ctypes.Structure):
    _fields_ = [("q", c_vp), ("n", c_int), ("r_hi", c_vp), ("r_lo", c_vp), ("ldr", c_ll), ("part_row", c_vp),
                ("part_max", c_vp), ("part_dot", c_vp), ("u_hi", c_vp), ("u_lo", c_vp), ("ldu", c_ll),
                ("v_hi", c_vp), ("v_lo", c_vp), ("ldv", c_ll), ("alpha", c_vp), ("beta", c_vp),
                ("qt_hi", c_vp), ("qt_lo", c_vp), ("ldqt", c_ll)]


class RotItem(ctypes.Structure):
    _fields_ = [("n", c_int), ("r_hi", c_vp), ("r_lo", c_vp), ("ldr", c_ll), ("s_hi", c_vp), ("s_lo", c_vp),
                ("lds", c_ll), ("alpha", c_vp), ("beta", c_vp)]


class TraceItem(ctypes.Structure):
    _fields_ = [("q", c_vp), ("n", c_int), ("s_hi", c_vp), ("s_lo", c_vp), ("lds", c_ll), ("part", c_vp)]


class ApplyItem(ctypes.Structure):
    _fields_ = [("param", c_vp), ("param_bf16", c_int), ("numel", c_ll), ("pg", c_vp), ("part", c_vp),
                ("nparts", c_int), ("scale", c_vp)]


class BalanceFactor(ctypes.Structure):
    _fields_ = [("q", c_vp), ("n", c_int), ("dense", c_int), ("qt_hi", c_vp), ("qt_lo", c_vp), ("ldqt", c_ll),
                ("p_hi", c_vp), ("p_lo", c_vp), ("ldp", c_ll), ("pdiag", c_vp), ("part", c_vp), ("nparts", c_int),
                ("scale", c_vp)]


class BalanceParam(ctypes.Structure):
    _fields_ = [("f0", c_int), ("nf", c_int)]


class SymItem(ctypes.Structure):
    _fields_ = [("a", c_vp), ("lda", c_ll), ("form", c_int), ("n", c_int), ("sign", c_int),
                ("out_hi", c_vp), ("out_lo", c_vp), ("ld_out", c_ll), ("out_f32", c_vp), ("ld_f32", c_ll),
                ("part_row", c_vp), ("part_max", c_vp), ("diag", c_vp), ("row_sq", c_vp), ("absmax", c_vp)]


class NlbFinishItem(ctypes.Structure):
    _fields_ = [("nf", c_vp), ("part", c_vp), ("slots", c_int), ("ncols", c_int), ("out", c_vp)]


PERMUTE_MAX_ORDER = 8
PERMUTE_CHUNK = 4096


class PermuteItem(ctypes.Structure):
    _fields_ = [("src", c_vp), ("order", c_int), ("omode", c_int * PERMUTE_MAX_ORDER),
                ("odim", c_ll * PERMUTE_MAX_ORDER), ("sstride", c_ll * PERMUTE_MAX_ORDER),
                ("scale", c_vp * PERMUTE_MAX_ORDER), ("numel", c_ll), ("cols", c_ll), ("out_hi", c_vp),
                ("out_lo", c_vp), ("ld_out", c_ll), ("out_f32", c_vp), ("row_sq", c_vp), ("part", c_vp)]


PSGD_PREP_NORMAL, PSGD_PREP_TRANS, PSGD_PREP_DIRECT = 0, 1, 2
PREP_ROWS = 8
ROT_ROWS = 8
TRACE_ROWS = 8
SKEW_TILE = 64
FAC_SCRATCH = 32   # floats of scratch per diagonal factor item
PSGD_FACTOR_DENSE, PSGD_FACTOR_RANK1, PSGD_FACTOR_DIAG, PSGD_FACTOR_SKEW = 0, 1, 2, 3
HY_LR_PRECOND, HY_BETA_L, HY_DAMPING, HY_LR_PARAMS, HY_MAX_AVG, HY_MAX_ELEM, HY_MOM_BETA = range(7)
HY_NOISE, HY_NOISE_KEY0, HY_NOISE_KEY1, HY_EMA_PHASE, HY_MOM_ALPHA, HY_COUNT = 7, 8, 9, 10, 11, 12
APPLY_CHUNK = 8192
SYM_TILE = 64
PSGD_SYM_SQUARE, PSGD_SYM_PACKED = 0, 1

# (name, restype, argtypes) of every exported entry point; tests check that each symbol is present.
SIGNATURES = [
    ("psgd_num_sms", c_int, []),
    ("psgd_gemm", c_int, [ctypes.POINTER(GemmSpec), c_int, c_vp, c_vp]),
    ("psgd_gemm_table_bytes", ctypes.c_size_t, [c_int]),
    ("psgd_gemm_count_tiles", c_int, [ctypes.POINTER(GemmSpec), c_int]),
    ("psgd_gemm_encode", c_int, [ctypes.POINTER(GemmSpec), c_int, c_vp, ctypes.c_size_t, c_vp, c_int,
                                 ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    ("psgd_gemm_launch", c_int, [c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    ("psgd_prep", c_int, [c_vp, c_vp, c_int, c_vp, c_vp, c_vp]),
    ("psgd_prep_momentum", c_int, [c_vp, c_vp, c_int, c_vp, c_vp, c_vp]),
    ("psgd_nlb_prep", c_int, [c_vp, c_int, c_vp, c_vp]),
    ("psgd_factor_update", c_int, [c_vp, c_int, c_vp, c_vp, c_vp]),
    ("psgd_skew", c_int, [c_vp, c_vp, c_int, c_vp, c_vp]),
    ("psgd_skew_rank1", c_int, [c_vp, c_vp, c_int, c_vp, c_vp]),
    ("psgd_rot", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    ("psgd_trace", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    ("psgd_apply", c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_vp]),
    ("psgd_balance", c_int, [c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_vp]),
    ("psgd_apply_noalloc", c_int, [c_vp, c_int, c_vp, c_ll, c_float, c_float, c_float, c_vp]),
    ("psgd_sym_expand", c_int, [c_vp, c_vp, c_int, c_vp, c_vp]),
    ("psgd_sym_reduce", c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    ("psgd_nlb_finish", c_int, [c_vp, c_int, c_vp, c_vp]),
    ("psgd_struct_sizes", c_int, [c_vp, c_int]),
    ("psgd_set_wait_limit_ns", ctypes.c_ulonglong, [ctypes.c_ulonglong]),
    ("psgd_wait_probe", c_int, [c_vp, ctypes.c_ulonglong, c_vp]),
    ("psgd_permute", c_int, [c_vp, c_vp, c_int, c_vp, c_vp]),
]

# device error word bits (include/psgd_b200.h PSGD_ERR_*)
ERR_BITS = {1: "a wait for a TMA stage gave up", 2: "a wait for a free stage gave up",
            4: "a wait on an accumulator handoff gave up", 8: "a descriptor failed a device-side check",
            16: "a factor's L or the Procrustes step came out NaN or infinite"}


def describe_err(v):
    return "; ".join(t for b, t in ERR_BITS.items() if v & b) or f"flags {v:#x}"

# the structs in the order psgd_struct_sizes reports them
STRUCTS = [GemmSpec, PrepItem, NlbPrepItem, FactorItem, SkewItem, RotItem, TraceItem, ApplyItem, BalanceFactor,
           BalanceParam, SymItem, NlbFinishItem, PermuteItem]


def _check_layout(L):
    """Refuses a library whose structs differ from these bindings (a stale build): a kernel would otherwise read
    item arrays at the wrong stride."""
    n = L.psgd_struct_sizes(None, 0)
    sizes = (ctypes.c_longlong * n)()
    L.psgd_struct_sizes(sizes, n)
    mine = [ctypes.sizeof(c) for c in STRUCTS]
    if n != len(mine) or list(sizes) != mine:
        raise RuntimeError(f"psgd_pro_b200: {LIB_PATH} was built from another version of include/psgd_b200.h "
                           f"(struct sizes {list(sizes)} against the bindings' {mine}); rebuild it with "
                           "`python -m psgd_pro_b200.build`")

_lib = None


def lib():
    """The loaded library, with argument types declared. Raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"psgd_pro_b200: {LIB_PATH} is missing; build it with `python -m psgd_pro_b200.build`"
                               " (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _check_layout(L)
        _lib = L
    return _lib


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"psgd_pro_b200: {what} failed: {ERRORS.get(rc, rc)}")
    return rc
