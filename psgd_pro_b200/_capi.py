"""ctypes binding of libpsgd_b200.so (the C ABI declared in include/psgd_b200.h).

The library is built in-tree (psgd_pro_b200/_lib/libpsgd_b200.so). There is no fallback: when the library is
missing or a call fails, a RuntimeError says so."""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libpsgd_b200.so")

c_vp, c_ll, c_int, c_float = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_float
c_fp = ctypes.POINTER(ctypes.c_float)

ERRORS = {-1: "invalid argument (shape, stride, alignment or mode)", -2: "CUDA launch failed",
          -3: "TMA descriptor encoding failed", -4: "caller table or workspace too small"}

PSGD_GEMM_PLAIN, PSGD_GEMM_SYRK = 0, 1


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
    ]


# (name, restype, argtypes) of every exported entry point; tests check that each symbol is present.
SIGNATURES = [
    ("psgd_num_sms", c_int, []),
    ("psgd_gemm", c_int, [ctypes.POINTER(GemmSpec), c_int, c_vp, c_vp]),
    ("psgd_gemm_table_bytes", ctypes.c_size_t, [c_int]),
    ("psgd_gemm_count_tiles", c_int, [ctypes.POINTER(GemmSpec), c_int]),
    ("psgd_gemm_encode", c_int, [ctypes.POINTER(GemmSpec), c_int, c_vp, ctypes.c_size_t, c_vp, c_int,
                                 ctypes.POINTER(c_int)]),
    ("psgd_gemm_launch", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
]

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
        _lib = L
    return _lib


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"psgd_pro_b200: {what} failed: {ERRORS.get(rc, rc)}")
    return rc
