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

/* ---------------------------------------------------------------------------------------------------------
 * Tensor-core GEMM: D = A * B^T (both operands K-major bf16 hi/lo, fp32 accumulation in TMEM), followed by a
 * fused epilogue. One spec describes one problem; a group launch runs many problems as one persistent grid.
 *   value(r, c)  = alpha' * D[r, c] + beta' * aux[r, c]       (aux term only when aux != NULL)
 *                  then * row_scale[r] * colscale[c]           (when given)
 *   alpha' = alpha * (*alpha_ptr if alpha_ptr), beta' likewise (device scalars, read at run time).
 *   colscale[c] = col_scale[c], or from cs_mode: 1 -> 1 / *cs_nf;
 *                 2 -> 1 / (*cs_nf * (sqrt(sum_t cs_part[t * N + c]) + FLT_MIN))   (t < cs_T)
 * Outputs (each optional): out_f32 (r, c) fp32; out_hi/out_lo (r, c) bf16; out_hi_t/out_lo_t (c, r) bf16.
 * Reductions (each optional, deterministic, one slot per tile, no atomics):
 *   part_tile[tm * tiles_n + tn] = sum value^2 over the tile
 *   part_col[tm * N + c]         = sum over the tile's rows of value^2
 *   part_row[tn * M + r]         = sum over the tile's columns of value^2
 * mode PSGD_GEMM_SYRK: A == B, M == N, bn == 128; only tiles with tm <= tn run and the symmetric result is
 *   written to both triangles (element (r, c) with c >= r and its mirror), so the output is exactly symmetric.
 *   part_row then holds the row sums of squares of the full symmetric matrix, split over T = tiles_n slots
 *   (part_row[slot * M + r]); diag_out[r] = value(r, r); part_dot[tm * tiles_n + tn] = sum over the tile's share
 *   of the symmetric matrix of value * dot_aux (both triangles), i.e. sum_t part_dot = sum(S .* dot_aux).
 */
#define PSGD_GEMM_PLAIN 0
#define PSGD_GEMM_SYRK 1

typedef struct PsgdGemmSpec {
  const void* a_hi; const void* a_lo; long long lda;   /* A: M x K bf16 */
  const void* b_hi; const void* b_lo; long long ldb;   /* B: N x K bf16 */
  int M, N, K;
  int bn;       /* tile width: 16, 32, 64, 128 or 256 (<= 128 with split = 3) */
  int mode;     /* PSGD_GEMM_PLAIN or PSGD_GEMM_SYRK */
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
} PsgdGemmSpec;

/* One problem, launched directly (its descriptor travels as a kernel parameter). Replaces the per-call cuBLAS
 * and Triton products of the reference (kernels/blas.cpp:20-65 syrk/symm/symm_right, kernels/k2.py:17-85
 * _syrk_kernel/_syrk2_kernel). */
int psgd_gemm(const PsgdGemmSpec* spec, int split, int* dev_err, cudaStream_t stream);

/* Grouped form: encode once on the host into caller buffers, copy the table and tile list to the device, then
 * launch any number of times (the launch reads only device memory, so it can be captured in a CUDA graph).
 * Tiles run in the order the specs are given (callers put the costliest problems first). */
size_t psgd_gemm_table_bytes(int nspecs);
int psgd_gemm_count_tiles(const PsgdGemmSpec* specs, int nspecs);
int psgd_gemm_encode(const PsgdGemmSpec* specs, int nspecs, void* host_table, size_t table_bytes,
                     uint32_t* host_tiles, int max_tiles, int* ntiles);
int psgd_gemm_launch(const void* dev_table, const uint32_t* dev_tiles, int ntiles, int split, int* dev_err,
                     cudaStream_t stream);

/* Number of SMs the grouped launches use on the current device (grid size of the persistent kernels). */
int psgd_num_sms(void);

#ifdef __cplusplus
}
#endif
#endif /* PSGD_B200_H */
