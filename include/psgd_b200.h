/* psgd_b200.h: the C ABI of libpsgd_b200.so, the sm_100a kernels behind the PSGD-Kron optimizer step.
 *
 * Conventions shared by every entry point:
 *   - Plain pointers and sizes only. The caller owns and allocates every buffer (inputs, outputs, workspace,
 *     the device error word); no entry point allocates device memory or synchronises the device.
 *   - Work is enqueued on `stream`, in stream order. Matrices are row-major with an explicit leading dimension
 *     in elements. bf16 operand buffers need a leading dimension that is a multiple of 8 and a 16-byte aligned
 *     base (the TMA rule); fp32 buffers need 4-byte alignment.
 *   - Return value: 0 on success, a negative PSGD_E* code when the arguments are rejected (nothing is launched)
 *     or the launch fails. Device-side problems (a wait that gave up) set bits in *dev_err instead of trapping.
 *   - "hi/lo" operands: an fp32 matrix X is carried as two bf16 matrices, hi = bf16(X) and lo = bf16(X - hi).
 *     split = 3 multiplies hi*hi + hi*lo + lo*hi (about 16 significant bits, for fp32-parity results);
 *     split = 1 uses the hi copies only (bf16 tensor-core arithmetic with fp32 accumulation).
 */
#ifndef PSGD_B200_H
#define PSGD_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PSGD_OK 0
#define PSGD_EINVAL -1     /* bad shape, stride, alignment or mode */
#define PSGD_ELAUNCH -2    /* the CUDA launch itself failed */
#define PSGD_ETMAP -3      /* the TMA descriptor could not be encoded */
#define PSGD_ESPACE -4     /* a caller-provided table or workspace is too small */
#define PSGD_ELIMIT -5     /* a size beyond the fixed scratch of psgd_apply_noalloc */

/* ---------------------------------------------------------------------------------------------------------
 * Tensor-core GEMM: D = A * B^T (both operands K-major bf16 hi/lo, fp32 accumulation in TMEM), followed by a
 * fused epilogue. One spec describes one problem; a group launch runs many problems as one persistent grid.
 *   value(r, c)  = alpha' * D[r, c] + beta' * aux[r, c]       (aux term only when aux != NULL)
 *                  then * row_scale[r] * colscale[c]           (when given)
 *   alpha' = alpha * (*alpha_ptr if alpha_ptr), beta' likewise (device scalars, read at run time).
 *   colscale[c] = col_scale[c], or from cs_mode (the subspace products of the norm lower bounds):
 *                 1 -> value / *cs_nf;  2 -> (value / (sqrt(sum_t cs_part[t * N + c]) + FLT_MIN)) / *cs_nf
 *                 (t < cs_T), the two divisions applied in this order
 * Outputs (each optional): out_f32 (r, c) fp32; out_hi/out_lo (r, c) bf16; out_hi_t/out_lo_t (c, r) bf16.
 * Reductions (each optional, deterministic, one slot per tile, no atomics):
 *   part_tile[tm * tiles_n + tn] = sum value^2 over the tile
 *   part_col[tm * N + c]         = sum over the tile's rows of value^2
 *   part_row[tn * M + r]         = sum over the tile's columns of value^2
 * mode PSGD_GEMM_SYRK: A == B, M == N, bn 128 or 256; only the tiles that reach the upper triangle run (tile
 *   (tm, tn) with tn >= tm * 128 / bn) and each element (r, c) with c >= r is written together with its mirror
 *   (c, r), so the output is exactly symmetric. Reductions in this mode:
 *   part_row[slot * M + r]: row sums of squares of the full symmetric matrix split over tiles_n + tiles_m slots
 *     (slot tn: the direct elements of tile (tm, tn); slot tiles_n + tm: the mirrored ones); slots no tile writes
 *     are never touched, so the buffer must start at zero once and the sum over all slots is the row sum;
 *   diag_out[r] = value(r, r); part_dot[tm * tiles_n + tn] = the tile's share of sum(S .* dot_aux) over both
 *     triangles (again zero-initialised once; the total is the sum of all entries).
 *   out_packed (SYRK only): the upper triangle as n(n+1)/2 fp32 values, row-major packed, (r, c >= r) at
 *     r n - r (r - 1) / 2 + c - r (the PACKED store of kernels/k2.py:78-80); may be the only output.
 * mode PSGD_GEMM_TRMM: A is upper triangular (A[r, k] = 0 for k < r; the caller stages it with zeros there) and
 *   M == K: tile (tm, tn) reduces over k >= its first row only, so the zero blocks left of the diagonal are neither
 *   loaded nor multiplied (n^2 (n + 1) useful FLOPs for a square T X instead of 2 n^3). No counterpart in the
 *   reference (the triangular-times-dense product of its benchmark plan).
 */
#define PSGD_GEMM_PLAIN 0
#define PSGD_GEMM_SYRK 1
#define PSGD_GEMM_TRMM 2

typedef struct PsgdGemmSpec {
  const void* a_hi; const void* a_lo; long long lda;   /* A: M x K bf16 */
  const void* b_hi; const void* b_lo; long long ldb;   /* B: N x K bf16 */
  int M, N, K;
  int bn;       /* tile width: 16, 32, 64, 128 or 256 (<= 128 with split = 3) */
  int mode;     /* PSGD_GEMM_PLAIN, PSGD_GEMM_SYRK or PSGD_GEMM_TRMM */
  float alpha, beta;
  const float* alpha_ptr; const float* beta_ptr;
  const float* aux; long long ld_aux;
  const float* row_scale; const float* col_scale;
  float* out_f32; long long ld_f32;
  void* out_hi; void* out_lo; long long ld_b;
  void* out_hi_t; void* out_lo_t; long long ld_bt;
  float* part_tile; float* part_col; float* part_row; float* diag_out;
  const float* dot_aux; long long ld_dot; float* part_dot;
  const float* cs_part; int cs_T; int cs_mode; const float* cs_nf;
  float* out_packed;
} PsgdGemmSpec;

/* One problem, launched directly (its descriptor travels as a kernel parameter). Replaces the per-call cuBLAS
 * and Triton products of the reference (kernels/blas.cpp:20-65 syrk/symm/symm_right, kernels/k2.py:17-85
 * _syrk_kernel/_syrk2_kernel). */
int psgd_gemm(const PsgdGemmSpec* spec, int split, int* dev_err, cudaStream_t stream);

/* Grouped form: encode once on the host into caller buffers, copy the table and tile list to the device, then
 * launch any number of times on the same device (the launch reads only device memory, so it can be captured in
 * a CUDA graph). The tile list (uint32 pairs; psgd_gemm_count_tiles gives its length, *ntiles the entries used)
 * starts with a header that splits the tiles into one segment per SM: tiles are taken in the order the specs are
 * given (callers put the costliest problems first) and each goes to the SM with the least estimated work so far.
 * Encoding also reports the group's kernel (*kind: the epilogue kind 0..5, plus 8 for CTA pairs or 16 for the
 * narrow ring), which the launch takes back: interior tiles of the problems of that epilogue kind run a specialised
 * epilogue, all other tiles the general one. */
size_t psgd_gemm_table_bytes(int nspecs);
int psgd_gemm_count_tiles(const PsgdGemmSpec* specs, int nspecs);
int psgd_gemm_encode(const PsgdGemmSpec* specs, int nspecs, void* host_table, size_t table_bytes,
                     uint32_t* host_tiles, int max_tiles, int* ntiles, int* kind);
int psgd_gemm_launch(const void* dev_table, const uint32_t* dev_tiles, int ntiles, int split, int kind,
                     int* dev_err, cudaStream_t stream);

/* Number of SMs the grouped launches use on the current device (grid size of the persistent kernels). */
int psgd_num_sms(void);

/* Device error word bits (*dev_err of every entry point; bits accumulate until the caller clears the word). */
#define PSGD_ERR_TIMEOUT_FULL 1    /* a wait for a TMA stage (or the wait probe's barrier) gave up */
#define PSGD_ERR_TIMEOUT_EMPTY 2   /* a wait for a free stage gave up */
#define PSGD_ERR_TIMEOUT_ACC 4     /* a wait on an accumulator handoff gave up */
#define PSGD_ERR_BAD_DESC 8        /* a descriptor failed a device-side check */
#define PSGD_ERR_NONFINITE 16      /* psgd_factor_update: a factor's L or the Procrustes step came out NaN / Inf */

/* Sets how long the GEMM kernels' waits for work (a TMA stage, a free stage, an accumulator) may take before the
 * launch gives up and sets PSGD_ERR_TIMEOUT_* (default 2 s; 0 restores it) for launches made after the call;
 * returns the previous limit. An aborting CTA still waits for its own copies and MMAs in flight with the default
 * limit before it releases shared memory and TMEM. No counterpart in the reference (it has no device waits). */
unsigned long long psgd_set_wait_limit_ns(unsigned long long ns);

/* One thread waits, with the library's bounded wait, on a barrier that nothing ever arrives at, for limit_ns
 * (at most 2 s), then sets PSGD_ERR_TIMEOUT_FULL in *dev_err and returns: the bounded-wait path made to run out,
 * for tests of the error reporting (the context stays usable). No counterpart in the reference. */
int psgd_wait_probe(int* dev_err, unsigned long long limit_ns, cudaStream_t stream);

/* Layout check: writes sizeof of PsgdGemmSpec, PsgdPrepItem, PsgdNlbPrepItem, PsgdFactorItem, PsgdSkewItem,
 * PsgdRotItem, PsgdTraceItem, PsgdApplyItem, PsgdBalanceFactor, PsgdBalanceParam, PsgdSymItem, PsgdNlbFinishItem,
 * PsgdPermuteItem (in this order, at most n of them) and returns how many structs there are (sizes may be NULL to ask). A binding
 * compares them with its own struct definitions once, before its first launch. */
int psgd_struct_sizes(long long* sizes, int n);

/* ---------------------------------------------------------------------------------------------------------
 * Memory-bound step kernels. Each takes a device array of items (one per parameter or factor, encoded by the
 * caller), an optional device work list of (item, tile) pairs (uint32 pairs: item index, (ti << 16) | tj),
 * the device hyper-parameter vector and the device error word. Sums are deterministic: fixed-order partials,
 * no atomics. Hyper-parameter slots (float hyper[PSGD_HY_COUNT]): */
#define PSGD_HY_LR_PRECOND 0   /* lr_preconditioner */
#define PSGD_HY_BETA_L 1       /* betaL */
#define PSGD_HY_DAMPING 2      /* damping */
#define PSGD_HY_LR_PARAMS 3    /* lr_params */
#define PSGD_HY_MAX_AVG 4      /* grad_clip_max_amps[0] */
#define PSGD_HY_MAX_ELEM 5     /* grad_clip_max_amps[1] */
#define PSGD_HY_MOM_BETA 6     /* momentum factor of this step */
#define PSGD_HY_NOISE 7        /* nonzero: psgd_prep generates the damping noise itself (below) */
#define PSGD_HY_NOISE_KEY0 8   /* the generator's key, two uint32 stored bit for bit in float slots */
#define PSGD_HY_NOISE_KEY1 9
#define PSGD_HY_EMA_PHASE 10   /* which staging pass of this step applies the momentum EMA (see PsgdPrepItem.m) */
#define PSGD_HY_MOM_ALPHA 11   /* 1 - momentum factor of this step, as the caller rounds it to float */
#define PSGD_HY_COUNT 12

/* Gradient staging on 32 x 32 tiles of an n1 x n2 gradient G (fp32 or bf16, contiguous):
 * x = G + (damping + eps |G|) * xi when xi != NULL (the damping noise of psgd_pro.py:122-123), else x = G.
 *   PREP_NORMAL: out (n1 x n2, bf16 hi/lo)           = x
 *   PREP_TRANS:  out (n2 x n1, bf16 hi/lo)           = (x * p2[j])^T
 *   PREP_DIRECT: out_f32 (n1 x n2) = p1[i] x p2[j]   (both factors diagonal: the whole preconditioned gradient)
 *               with optional part_row[tj][i], part_col[ti][j], part_tile[ti * tiles_j + tj] sums of squares.
 * p1/p2 NULL mean ones. Work entries: (item, row block of PSGD_PREP_ROWS rows) for PREP_NORMAL, (item,
 * (ti << 16) | tj) 32 x 32 tiles otherwise. Replaces the exprP prologue of psgd_pro.py:123 and
 * psgd_pro_fast.py:176. */
#define PSGD_PREP_ROWS 8   /* PREP_NORMAL work entries cover PSGD_PREP_ROWS rows: (item, row block) */
/* Damping noise (items with xi != NULL): read from xi, or, when hyper[PSGD_HY_NOISE] != 0, generated in the kernel:
 * element e (index i * n2 + j of the item) gets the standard normal number s = noise_base + e of the sequence
 * Philox4x32-10 (Salmon et al., SC'11) with key (KEY0, KEY1) and counter (s / 4, 0, 0, 0), its four words w
 * taken as uniforms u = ((w >> 9) + 1/2) / 2^23 and two Box-Muller pairs: sqrt(-2 ln u0) (cos, sin)(2 pi u1 - pi)
 * give numbers 4c, 4c + 1, and words 2, 3 the same way give 4c + 2, 4c + 3. The values depend on the key and
 * position only, not on the launch geometry. */
#define PSGD_PREP_NORMAL 0
#define PSGD_PREP_TRANS 1
#define PSGD_PREP_DIRECT 2
typedef struct PsgdPrepItem {
  const void* g; int g_bf16; int mode;
  const float* xi;
  int n1, n2;
  const float* p1; const float* p2;
  void* out_hi; void* out_lo; long long ld_out;
  float* out_f32;
  float* part_row; float* part_col; float* part_tile;
  float eps;
  long long noise_base;  /* position of element 0 in the generated noise sequence (a multiple of 4) */
  /* Momentum (psgd_pro.py:334-343; psgd_prep_momentum only), NULL for none: the buffer m (n1 x n2, g's dtype).
   * When m is set, the staged
   * source is the momentum instead of g: if mom_phase == hyper[PSGD_HY_EMA_PHASE] this pass first applies the EMA,
   * m = rn(rn(beta m) + alpha g) with beta = hyper[PSGD_HY_MOM_BETA], alpha = hyper[PSGD_HY_MOM_ALPHA] (rn:
   * rounding to g's dtype, as torch's in-place mul_ and add_ on that dtype), writes m back and stages it; otherwise it
   * stages m as stored. */
  void* m; int mom_phase;
  /* PREP_NORMAL only, NULL for none: x before the damping noise is also stored here (bf16 hi / lo halves, the
   * layout and ld_out of out_hi), so one read of G stages both the noisy operand of the preconditioner update and
   * the clean operand of the parameter update. */
  void* out2_hi; void* out2_lo;
} PsgdPrepItem;
int psgd_prep(const PsgdPrepItem* items, const uint32_t* work, int nwork, const float* hyper, int* dev_err,
              cudaStream_t stream);
/* The same honouring the items' momentum fields (m, mom_phase below); psgd_prep ignores them (its kernel is built
 * without the momentum path, which keeps its register count and occupancy). */
int psgd_prep_momentum(const PsgdPrepItem* items, const uint32_t* work, int nwork, const float* hyper, int* dev_err,
                       cudaStream_t stream);

/* Start of the norm lower bound (psgd_pro.py:31-36 spd, :55-60 skh; psgd_pro_fast.py:32-38), one CTA per item:
 * nf = max diag + tiny (spd) or max |A| + tiny (skh), j = argmax row norm (from part_row[row_slots][n]),
 * V0 = A_j / nf + sgn(<A_j / nf, V_r>) V_r for the 32 rows of v, written as bf16 hi/lo (32 x n); *nf_out = nf. */
typedef struct PsgdNlbPrepItem {
  const void* a_hi; const void* a_lo; long long lda;
  int n; int skew;
  const float* part_row; int row_slots;
  const float* diag;
  const float* part_max; int max_slots;
  const float* v;
  void* v0_hi; void* v0_lo; long long ldv;
  float* nf_out;
} PsgdNlbPrepItem;
int psgd_nlb_prep(const PsgdNlbPrepItem* items, int nitems, int* dev_err, cudaStream_t stream);

/* Per-factor scalar work after the subspace iteration (psgd_pro.py:126-135, psgd_pro_fast.py:178-189); one CTA
 * per item, except FACTOR_DIAG items, whose n entries are split into PSGD_FAC_SPLIT ranges (two launches):
 *   FACTOR_DENSE: ell = nf * max_c sqrt(sum_t part[t * ncols + c]) + term2  (the bound of the 4th product)
 *   FACTOR_RANK1: ell = sum_t part[t] + term2                  (1-D gradient: term1 = Pg Pg^T, bound = |Pg|^2)
 *   both: L = max(betaL L + (1 - betaL) ell, ell); *alpha = -lr/L; *beta = 1 + lr/L * term2
 *         (the q update q - lr/L (term1 q - term2 q) as beta q + alpha term1 q)
 *   FACTOR_DIAG: term1_i = sum_s part[s * n + i]; ell = max term1 + term2; L as above;
 *         q_i *= 1 - lr/L (term1_i - term2); p_i = q_i^2.
 *   FACTOR_SKEW: s = nf * max_c ||W4_c|| + tiny (the skew bound of R = Q - Q^T); tr(RQ) = sum(part_dot_rq) / s,
 *         tr(RRQ) = -sum(part_dot_sq[0 .. n_sq)) / s^2; a = min(-tr(RQ)/tr(RRQ), 1/8) if tr(RRQ) < 0 else 1/8;
 *         *alpha = a, *beta = 1 / s   (the Procrustes step of psgd_pro_fast.py:141-153). */
/* Any item whose ell, L, q-update coefficients or Procrustes step come out NaN or infinite sets PSGD_ERR_NONFINITE
 * (the values are still written, as the reference would carry the NaN on). */
#define PSGD_FACTOR_DENSE 0
#define PSGD_FACTOR_RANK1 1
#define PSGD_FACTOR_DIAG 2
#define PSGD_FACTOR_SKEW 3
typedef struct PsgdFactorItem {
  int kind; int n; float term2;
  float* L;
  const float* nf; const float* part; int slots; int ncols;
  float* alpha; float* beta;
  float* q; float* p;
  const float* part_dot_rq; int n_rq;
  const float* part_dot_sq; int n_sq;
  float* scratch;  /* FACTOR_DIAG: PSGD_FAC_SCRATCH floats (the item's n is split into PSGD_FAC_SPLIT ranges) */
} PsgdFactorItem;
#define PSGD_FAC_SPLIT 16
#define PSGD_FAC_SCRATCH 32
int psgd_factor_update(const PsgdFactorItem* items, int nitems, const float* hyper, int* dev_err,
                       cudaStream_t stream);

/* Rn = Q - Q^T (psgd_pro_fast.py:147; psgd_pro.py:87 up to sign), written as bf16 hi/lo. Work entries are
 * pairs of PSGD_SKEW_TILE-square tiles (TI <= TJ): one block reads Q[TI, TJ] and Q[TJ, TI] once and writes both
 * Rn tiles. Reductions use 32-wide slots (tiles32 = ceil(n / 32)): part_row[slot][i] (row sums of squares over the
 * block's columns, slot 2 TJ or 2 TI), and per pair part_max (max |Rn|) and part_dot (sum Rn * Q) in entry
 * (2 TI) * tiles32 + 2 TJ. Every other slot stays as the caller left it (zero: consumers sum or max over all).
 * The pair's share of sum Rn * Q is taken as (1/2) sum Rn^2 over its two tiles (the identity
 * sum_ij (Q_ij - Q_ji) Q_ij = (1/2) sum_ij (Q_ij - Q_ji)^2), which has no cancellation. */
#define PSGD_SKEW_TILE 64
typedef struct PsgdSkewItem {
  float* q; int n;
  void* r_hi; void* r_lo; long long ldr;
  float* part_row; float* part_max; float* part_dot;
  /* Rank-one factors (1-D parameters, psgd_pro.py:132-135 with term1 = Pg Pg^T): when u_hi != NULL the q update
   * runs here first, q <- (*alpha) (u v^T) + (*beta) q with u = u_hi (+ u_lo) and v = v_hi (+ v_lo) the n-vectors
   * stored one per row (leading dimensions ldu, ldv; the K = 1 operands of that product), summed hi * hi, + hi * lo,
   * + lo * hi; the updated q is written back (fp32) and as q^T (bf16 hi/lo, qt_hi/qt_lo, leading dimension ldqt),
   * and Rn is taken from the updated q. */
  const void* u_hi; const void* u_lo; long long ldu;
  const void* v_hi; const void* v_lo; long long ldv;
  const float* alpha; const float* beta;
  void* qt_hi; void* qt_lo; long long ldqt;
} PsgdSkewItem;
int psgd_skew(const PsgdSkewItem* items, const uint32_t* work, int nwork, int* dev_err, cudaStream_t stream);
/* The same for work entries whose items carry the rank-one q update (u_hi != NULL); psgd_skew ignores those
 * fields. No counterpart entry point in the reference: there the update is a separate product (psgd_pro.py:135). */
int psgd_skew_rank1(const PsgdSkewItem* items, const uint32_t* work, int nwork, int* dev_err, cudaStream_t stream);

/* M = a (Rn / s) + a^2 / 2 ((S / s) / s) (bf16 hi/lo in, bf16 hi/lo out in place of Rn), with a = *alpha and
 * 1/s = *beta from PSGD_FACTOR_SKEW: the Procrustes multiplier of psgd_pro_fast.py:153. Work entries: (item,
 * first row of a block of PSGD_ROT_ROWS rows); whole padded rows are processed (padding columns are zero and stay
 * zero). */
#define PSGD_ROT_ROWS 8
typedef struct PsgdRotItem {
  int n;
  void* r_hi; void* r_lo; long long ldr;
  const void* s_hi; const void* s_lo; long long lds;
  const float* alpha; const float* beta;
} PsgdRotItem;
/* has_lo: the items' r_lo / s_lo are set (fp32 mode; with 0 they are ignored). */
int psgd_rot(const PsgdRotItem* items, const uint32_t* work, int nwork, int has_lo, int* dev_err,
             cudaStream_t stream);

/* Trace of the Procrustes line search, sum_ij S_ij Q_ij with S = Rn Rn^T (psgd_pro_fast.py:149-151): S as stored
 * (bf16 hi, plus lo when s_lo != NULL; leading dimension lds) against the fp32 n x n Q, both read row-major once.
 * Work entries: (item, first row of a block of PSGD_TRACE_ROWS rows); entry (item, r0) writes the block's sum to
 * part[r0 / PSGD_TRACE_ROWS] (a fixed-order block reduction), so sum(part[0 .. ceil(n / PSGD_TRACE_ROWS))) is the
 * trace. A separate pass because the alternative, the S product's epilogue reading Q at each tile and at its mirror,
 * cost more than this pass's 6 bytes per element. */
#define PSGD_TRACE_ROWS 8
typedef struct PsgdTraceItem {
  const float* q; int n;
  const void* s_hi; const void* s_lo; long long lds;
  float* part;
} PsgdTraceItem;
/* has_lo: the items' s_lo are set (fp32 mode; with 0 they are ignored). */
int psgd_trace(const PsgdTraceItem* items, const uint32_t* work, int nwork, int has_lo, int* dev_err,
               cudaStream_t stream);

/* Clip and apply (psgd_pro.py:371-381, branch-free as psgd_pro_fast.py:426-438): per parameter
 * avg = sqrt(sum(part) / numel), g = clamp(pg * min(1, max_avg / avg), +-max_elem), param -= lr_params * g.
 * Work items are (item, chunk) pairs over chunks of PSGD_APPLY_CHUNK elements. */
#define PSGD_APPLY_CHUNK 8192
typedef struct PsgdApplyItem {
  void* param; int param_bf16; long long numel;
  const float* pg;
  const float* part; int nparts;
  float* scale;   /* scratch: the clip scale of this parameter (written by the first pass) */
} PsgdApplyItem;
int psgd_apply(const PsgdApplyItem* items, int nitems, const uint32_t* work, int nwork, const float* hyper,
               int* dev_err, cudaStream_t stream);

/* Factor balancing of the listed parameters (psgd_pro.py:96-105, drawn with probability 0.01 per parameter):
 * max |q| of each factor (absmax over work_max entries (factor, chunk of PSGD_APPLY_CHUNK values) into part),
 * c_k = (prod_k max_k)^(1/order) / max_k per parameter (into *scale), then work_apply entries rescale: dense
 * factors per 32 x 32 tile (factor, (ti << 16) | tj): Q *= c, Q^T rewritten from the new Q, P *= c^2; diagonal
 * factors per chunk (factor, chunk): q *= c, p = q^2. part and scale are caller scratch. */
typedef struct PsgdBalanceFactor {
  float* q; int n; int dense;
  void* qt_hi; void* qt_lo; long long ldqt;
  void* p_hi; void* p_lo; long long ldp;
  float* pdiag;
  float* part; int nparts;
  float* scale;
} PsgdBalanceFactor;
typedef struct PsgdBalanceParam { int f0; int nf; } PsgdBalanceParam;
int psgd_balance(const PsgdBalanceFactor* factors, const PsgdBalanceParam* params, int nparams,
                 const uint32_t* work_max, int nwork_max, const uint32_t* work_apply, int nwork_apply, int* dev_err,
                 cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------------------
 * Symmetric matrices in storage form (kernels/ops.py:7-11): PSGD_SYM_SQUARE, an n x n fp32 square (leading
 * dimension lda) whose upper triangle (j >= i) holds the matrix, the lower triangle never read (it may hold
 * anything, NaN included, kernels/ops.py:9); PSGD_SYM_PACKED, the row-major packed upper triangle, n(n+1)/2 fp32
 * values with (i, j >= i) at i n - i (i - 1) / 2 + j - i (kernels/k2.py:78-80). The full matrix is
 * A(i, j) = U(i, j) for j >= i and sign * U(j, i) below: sign 1 symmetric, -1 skew-symmetric (diagonal taken as
 * zero, as kernels/k1.cu:41-50 does), 0 upper triangular (zeros below; the staging of a TRMM operand).
 * psgd_sym_expand reads only the stored triangle, once, in pairs of PSGD_SYM_TILE-square tiles (work entries
 * (item, (I << 16) | J), I <= J), and writes each optional output:
 *   out_hi / out_lo (bf16 hi/lo, leading dimension ld_out): the full matrix as a tensor-core operand;
 *   out_f32 (ld_f32): the full matrix in fp32 (kernels/k2.py:88-103 unpack);
 *   part_row[slot * n + i]: sums of squares of row i over the columns of 64-column block slot (every slot written);
 *   part_max[I * T + J] (T = ceil(n / 64)): max |A| over the pair's tiles;  diag[i] = A(i, i).
 * psgd_sym_reduce finishes tri_rownorm2 (kernels/k1.cu:296-307): row_sq[i] = sum of part_row over the slots,
 * *absmax = max of part_max (max_n: the largest n of the items). */
#define PSGD_SYM_TILE 64
#define PSGD_SYM_SQUARE 0
#define PSGD_SYM_PACKED 1
typedef struct PsgdSymItem {
  const float* a; long long lda; int form; int n; int sign;
  void* out_hi; void* out_lo; long long ld_out;
  float* out_f32; long long ld_f32;
  float* part_row; float* part_max; float* diag;
  float* row_sq; float* absmax;
} PsgdSymItem;
int psgd_sym_expand(const PsgdSymItem* items, const uint32_t* work, int nwork, int* dev_err, cudaStream_t stream);
int psgd_sym_reduce(const PsgdSymItem* items, int nitems, int max_n, int* dev_err, cudaStream_t stream);

/* End of a norm lower bound (psgd_pro.py:40-41, psgd_pro_fast.py:43): *out = *nf * max_c sqrt(sum_t part[t * ncols
 * + c]) over the column sums of squares of the last subspace product, one block per item. */
typedef struct PsgdNlbFinishItem {
  const float* nf; const float* part; int slots; int ncols; float* out;
} PsgdNlbFinishItem;
int psgd_nlb_finish(const PsgdNlbFinishItem* items, int nitems, int* dev_err, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------------------
 * Layout changes of order-r parameters (r >= 3; psgd_pro.py:107-112 exprP, :222-228 exprGs): a tensor with natural
 * dims d[0..r-1] moves from a source layout to an output layout, both the natural order with at most one mode moved
 * (to the end, or for the output also to the front), so that the mode a product contracts is the last (mode
 * products with P) or the first (term1 = the contraction over every other mode) dimension of a row-major matrix.
 * The caller describes the output layout position by position (omode: the natural mode at each position, outermost
 * first; odim: its size) and the source by the stride of each natural mode (sstride); scale[m] (a diagonal factor's
 * q^2, or NULL) multiplies every element by scale[m][i_m] on the way. Outputs (each optional): the operand out_hi /
 * out_lo (the output as a rows x cols matrix, cols given, row pitch ld_out), out_f32 (unpadded, output layout),
 * row_sq (sum of squares of each output row; work units are then rows) and part (sum of squares per work unit).
 * Work entries (item, unit): an output row when row_sq is set, else a chunk of PSGD_PERMUTE_CHUNK output elements. */
#define PSGD_PERMUTE_MAX_ORDER 8
#define PSGD_PERMUTE_CHUNK 4096
typedef struct PsgdPermuteItem {
  const float* src;
  int order; int omode[PSGD_PERMUTE_MAX_ORDER];
  long long odim[PSGD_PERMUTE_MAX_ORDER];
  long long sstride[PSGD_PERMUTE_MAX_ORDER];
  const float* scale[PSGD_PERMUTE_MAX_ORDER];
  long long numel, cols;
  void* out_hi; void* out_lo; long long ld_out;
  float* out_f32; float* row_sq; float* part;
} PsgdPermuteItem;
int psgd_permute(const PsgdPermuteItem* items, const uint32_t* work, int nwork, int* dev_err, cudaStream_t stream);

/* Clip and apply for one parameter without any device memory from the caller. It has no counterpart in the
 * reference, which always works through torch and so always allocates. It exists for callers that cannot
 * allocate device memory: a plugin whose host application owns every device allocation, code that runs inside
 * another framework's memory pool where a raw cudaMalloc is not allowed, or a latency-critical loop that cannot
 * afford the device-wide synchronisation of cudaMalloc / cudaFree. The caller passes the parameter (fp32, or bf16
 * when param_bf16 != 0; updated in place), its preconditioned gradient pg (fp32, numel values) and the three
 * hyper-parameters by value; the result is that of psgd_apply: param -= lr_params * clamp(pg * min(1,
 * max_avg_amp / rms(pg)), +-max_elem_amp).
 * Scratch: one sum of squares per PSGD_APPLY_CHUNK elements, kept in a fixed 16 KB array inside the library that
 * every GPU loading the library holds until the process exits. Limit: numel <= PSGD_APPLY_NOALLOC_MAX_NUMEL
 * (33,554,432); larger parameters are rejected with PSGD_ELIMIT (use psgd_apply for them).
 * The first call on a device looks up the array's device address with that device current; make that first call
 * before any stream capture. All calls on a device share the array and leave their sums in it; each call writes
 * every slot it reads before reading it, so nothing carries over, but calls whose kernels overlap on the GPU (on
 * different streams) race on the array and produce wrong results. When a CUDA error from earlier work is already
 * pending on the calling thread, the call launches nothing and returns PSGD_ELAUNCH, leaving that error in place.
 * Non-finite values propagate as in the reference: a NaN in pg reaches the parameter. */
#define PSGD_APPLY_NOALLOC_SLOTS 4096
#define PSGD_APPLY_NOALLOC_MAX_NUMEL (4096LL * PSGD_APPLY_CHUNK)
int psgd_apply_noalloc(void* param, int param_bf16, const float* pg, long long numel, float lr_params,
                       float max_avg_amp, float max_elem_amp, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* PSGD_B200_H */
