// Symmetric matrices in storage form (the triangle-in-square and packed forms of the reference's plug-in surface,
// kernels/ops.py:7-11, kernels/k2.py:78-80, kernels/k1.cu:56-57): one pass that reads only the stored upper
// triangle and writes the full matrix as a tensor-core operand (bf16 hi/lo) and/or fp32, with the row sums of
// squares, max |A| and the diagonal; the reductions that finish tri_rownorm2 (kernels/k1.cu:296-307) and the norm
// lower bound (psgd_pro.py:19-41: nf * max row norm of the last subspace product).
//
// Work: pairs of 64 x 64 tiles (I <= J). One block reads the stored tile U(I, J) once into shared memory and writes
// the output tiles (I, J) and, for I < J, its mirror (J, I) = sign * U(I, J)^T; on the diagonal tile the lower half
// is the mirror of the upper half (or zero). All reductions are fixed-order partials (no atomics).
#include "common.cuh"
#include "psgd_b200.h"

#include <float.h>

namespace psgd {
namespace {

constexpr int ST = PSGD_SYM_TILE;  // 64
constexpr int SP = ST + 1;         // shared-memory pitch (conflict-free row and column walks)
constexpr int SYM_THREADS = 256;

__device__ __forceinline__ float sym_load(const PsgdSymItem& it, long long i, long long j) {
  // (i, j) with j >= i: square form at i * lda + j, packed form at i n - i (i - 1) / 2 + j - i
  if (it.form == PSGD_SYM_PACKED) return it.a[i * it.n - (i * (i - 1)) / 2 + (j - i)];
  return it.a[i * it.lda + j];
}

__device__ __forceinline__ void put(const PsgdSymItem& it, long long r, long long c, float v) {
  if (it.out_hi) {
    __nv_bfloat16 h, l;
    split_bf16(v, h, l);
    reinterpret_cast<__nv_bfloat16*>(it.out_hi)[r * it.ld_out + c] = h;
    if (it.out_lo) reinterpret_cast<__nv_bfloat16*>(it.out_lo)[r * it.ld_out + c] = l;
  }
  if (it.out_f32) it.out_f32[r * it.ld_f32 + c] = v;
}

__global__ void __launch_bounds__(SYM_THREADS) sym_expand_kernel(const PsgdSymItem* __restrict__ items,
                                                                 const uint32_t* __restrict__ work, int nwork) {
  __shared__ float s[ST][SP];
  __shared__ float red[SYM_THREADS / 32];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdSymItem& it = items[work[2 * w]];
    const int I = (int)(work[2 * w + 1] >> 16), J = (int)(work[2 * w + 1] & 0xFFFF);
    const long long n = it.n, r0 = (long long)I * ST, c0 = (long long)J * ST;
    const float sign = (float)it.sign;
    const bool diag = I == J;
    // 1. the stored upper tile (rows of I, columns of J); nothing below the diagonal is read
    for (int e = t; e < ST * ST; e += SYM_THREADS) {
      const int r = e / ST, c = e % ST;
      const long long gr = r0 + r, gc = c0 + c;
      s[r][c] = (gr < n && gc < n && gc >= gr) ? sym_load(it, gr, gc) : 0.f;
    }
    __syncthreads();
    if (diag) {  // lower half of the diagonal tile: the mirror (sign 0: zero); a skew matrix has a zero diagonal
      for (int e = t; e < ST * ST; e += SYM_THREADS) {
        const int r = e / ST, c = e % ST;
        if (r > c) s[r][c] = sign * s[c][r];
        if (r == c && it.sign < 0) s[r][c] = 0.f;
      }
      __syncthreads();
    }
    // 2. outputs: tile (I, J) row-major, then the mirror tile (J, I) = sign * s^T
    if (it.out_hi || it.out_f32) {
      for (int e = t; e < ST * ST; e += SYM_THREADS) {
        const int r = e / ST, c = e % ST;
        const long long gr = r0 + r, gc = c0 + c;
        if (gr < n && gc < n) put(it, gr, gc, s[r][c]);
      }
      if (!diag) {
        for (int e = t; e < ST * ST; e += SYM_THREADS) {
          const int r = e / ST, c = e % ST;  // output row c0 + r, column r0 + c
          const long long gr = c0 + r, gc = r0 + c;
          if (gr < n && gc < n) put(it, gr, gc, sign * s[c][r]);
        }
      }
    }
    if (it.diag && diag) {
      for (int r = t; r < ST; r += SYM_THREADS)
        if (r0 + r < n) it.diag[r0 + r] = s[r][r];
    }
    // 3. row sums of squares: rows of I over the columns of J (slot J); rows of J over the columns of I (slot I)
    const int T = (int)((n + ST - 1) / ST);
    if (it.part_row) {
      if (t < ST) {
        float acc = 0.f;
        for (int c = 0; c < ST; ++c) acc += s[t][c] * s[t][c];
        if (r0 + t < n) it.part_row[(long long)J * n + r0 + t] = acc;
      } else if (t < 2 * ST && !diag) {
        const int c = t - ST;
        float acc = 0.f;
        for (int r = 0; r < ST; ++r) acc += (sign * s[r][c]) * (sign * s[r][c]);
        if (c0 + c < n) it.part_row[(long long)I * n + c0 + c] = acc;
      }
    }
    // 4. max |A| over both tiles (the mirror has the same magnitudes unless it is zero)
    if (it.part_max) {
      float m = 0.f;
      for (int e = t; e < ST * ST; e += SYM_THREADS) m = fmaxf(m, fabsf(s[e / ST][e % ST]));
      m = warp_max(m);
      if (lane == 0) red[wid] = m;
      __syncthreads();
      if (t == 0) {
        float mm = red[0];
        for (int k = 1; k < SYM_THREADS / 32; ++k) mm = fmaxf(mm, red[k]);
        it.part_max[(long long)I * T + J] = mm;
      }
    }
    __syncthreads();  // s is reused by the next pair
  }
}

// row_sq[i] = sum over the slots of part_row[slot][i]; *absmax = max over the pairs' part_max. Blocks walk (item,
// 256-row chunk) entries; the chunk-0 block of an item also reduces the maxima.
__global__ void __launch_bounds__(SYM_THREADS) sym_reduce_kernel(const PsgdSymItem* __restrict__ items, int nitems,
                                                                 int chunks_per_item) {
  __shared__ float red[SYM_THREADS / 32];
  for (int w = blockIdx.x; w < nitems * chunks_per_item; w += gridDim.x) {
    const PsgdSymItem& it = items[w / chunks_per_item];
    const int chunk = w % chunks_per_item;
    const long long n = it.n;
    const int T = (int)((n + ST - 1) / ST);
    const long long i = (long long)chunk * SYM_THREADS + threadIdx.x;
    if (it.row_sq && it.part_row && i < n) {
      float acc = 0.f;
      for (int sl = 0; sl < T; ++sl) acc += it.part_row[(long long)sl * n + i];
      it.row_sq[i] = acc;
    }
    if (chunk == 0 && it.absmax && it.part_max) {
      float m = 0.f;
      for (int I = 0; I < T; ++I)
        for (int J = I + (int)threadIdx.x; J < T; J += SYM_THREADS) m = fmaxf(m, it.part_max[(long long)I * T + J]);
      m = warp_max(m);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
      __syncthreads();
      if (threadIdx.x == 0) {
        float mm = red[0];
        for (int k = 1; k < SYM_THREADS / 32; ++k) mm = fmaxf(mm, red[k]);
        *it.absmax = mm;
      }
      __syncthreads();
    }
  }
}

// out[k] = (*nf) * max_c sqrt(sum_t part[t * ncols + c]): the norm lower bound from the column sums of squares of
// the last subspace product (psgd_pro.py:40-41, psgd_pro_fast.py:43), one block per item.
__global__ void __launch_bounds__(SYM_THREADS) nlb_finish_kernel(const PsgdNlbFinishItem* __restrict__ items) {
  __shared__ float red[SYM_THREADS / 32];
  const PsgdNlbFinishItem& it = items[blockIdx.x];
  float m = 0.f;
  for (int c = threadIdx.x; c < it.ncols; c += SYM_THREADS) {
    float acc = 0.f;
    for (int t = 0; t < it.slots; ++t) acc += it.part[(long long)t * it.ncols + c];
    m = fmaxf(m, sqrtf(acc));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int k = 1; k < SYM_THREADS / 32; ++k) mm = fmaxf(mm, red[k]);
    *it.out = *it.nf * mm;
  }
}

template <typename Kernel>
int occupancy_grid(Kernel kernel, int nwork) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, SYM_THREADS, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int cap = sms * per_sm;
  return nwork < cap ? nwork : cap;
}

}  // namespace
}  // namespace psgd

using namespace psgd;

extern "C" int psgd_sym_expand(const PsgdSymItem* items, const uint32_t* work, int nwork, int* dev_err,
                               cudaStream_t stream) {
  if (!items || (nwork > 0 && !work) || nwork < 0 || !dev_err) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  sym_expand_kernel<<<occupancy_grid(sym_expand_kernel, nwork), SYM_THREADS, 0, stream>>>(items, work, nwork);
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}

extern "C" int psgd_sym_reduce(const PsgdSymItem* items, int nitems, int max_n, int* dev_err, cudaStream_t stream) {
  if (!items || nitems < 0 || max_n < 0 || !dev_err) return PSGD_EINVAL;
  if (nitems == 0 || max_n == 0) return PSGD_OK;
  const int chunks = (max_n + SYM_THREADS - 1) / SYM_THREADS;
  const long long nwork = (long long)nitems * chunks;
  if (nwork > 0x7fffffff) return PSGD_EINVAL;
  sym_reduce_kernel<<<occupancy_grid(sym_reduce_kernel, (int)nwork), SYM_THREADS, 0, stream>>>(items, nitems, chunks);
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}

extern "C" int psgd_nlb_finish(const PsgdNlbFinishItem* items, int nitems, int* dev_err, cudaStream_t stream) {
  if (!items || nitems < 0 || !dev_err) return PSGD_EINVAL;
  if (nitems == 0) return PSGD_OK;
  nlb_finish_kernel<<<nitems, SYM_THREADS, 0, stream>>>(items);
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}
