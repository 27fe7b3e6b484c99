// Layout changes of order-r parameters (r >= 3): the mode products of the preconditioner application
// (psgd_pro.py:107-112, exprP of :237-238) and the contractions over every mode but one (exprGs, :222-228) reduce to
// matrix products once the contracted mode is the last (or the first) dimension of a row-major layout; this kernel
// moves a tensor between such layouts, multiplying in the diagonal factors' scales on the way, and writes the result
// as a tensor-core operand (bf16 hi/lo, padded rows), in fp32, and / or as per-row sums of squares.
//
// Layouts: the natural order of the dims with at most one mode moved to the end (PsgdPermuteItem.src_mode, dst_mode)
// or, for the output, to the front (dst_first). Each output element is read once from its source position (the
// source index is rebuilt from the output index by one division per dim).
#include "common.cuh"
#include "psgd_b200.h"

namespace psgd {
namespace {

constexpr int PM_THREADS = 256;

__device__ __forceinline__ float pm_value(const PsgdPermuteItem& it, long long f, long long& src) {
  // f: flat output index in the output layout; walk its digits from the fastest dim outwards
  long long rest = f, s = 0;
  float v = 1.f;
#pragma unroll 1
  for (int p = it.order - 1; p >= 0; --p) {
    const long long d = it.odim[p];
    const long long i = rest % d;
    rest /= d;
    const int m = it.omode[p];
    s += i * it.sstride[m];
    if (it.scale[m]) v *= it.scale[m][i];
  }
  src = s;
  return v;
}

__device__ __forceinline__ void pm_store(const PsgdPermuteItem& it, long long f, float v) {
  if (it.out_hi) {
    const long long row = f / it.cols, col = f - row * it.cols;
    __nv_bfloat16 h, l;
    split_bf16(v, h, l);
    reinterpret_cast<__nv_bfloat16*>(it.out_hi)[row * it.ld_out + col] = h;
    if (it.out_lo) reinterpret_cast<__nv_bfloat16*>(it.out_lo)[row * it.ld_out + col] = l;
  }
  if (it.out_f32) it.out_f32[f] = v;
}

__global__ void __launch_bounds__(PM_THREADS) permute_kernel(const PsgdPermuteItem* __restrict__ items,
                                                             const uint32_t* __restrict__ work, int nwork) {
  __shared__ float red[PM_THREADS / 32];
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdPermuteItem& it = items[work[2 * w]];
    const long long unit = work[2 * w + 1];
    // a unit is one output row (row_sq wanted) or a chunk of PSGD_PERMUTE_CHUNK output elements
    const long long f0 = it.row_sq ? unit * it.cols : unit * PSGD_PERMUTE_CHUNK;
    const long long f1 = it.row_sq ? f0 + it.cols : min(f0 + (long long)PSGD_PERMUTE_CHUNK, it.numel);
    float acc = 0.f;
    for (long long f = f0 + threadIdx.x; f < f1; f += PM_THREADS) {
      long long src;
      const float sc = pm_value(it, f, src);
      const float v = it.src[src] * sc;
      pm_store(it, f, v);
      acc += v * v;
    }
    if (it.row_sq || it.part) {  // fixed-order block sum
      acc = warp_sum(acc);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
        for (int k = 0; k < PM_THREADS / 32; ++k) t += red[k];
        if (it.row_sq) it.row_sq[unit] = t;
        if (it.part) it.part[unit] = t;
      }
      __syncthreads();
    }
  }
}

}  // namespace
}  // namespace psgd

extern "C" int psgd_permute(const PsgdPermuteItem* items, const uint32_t* work, int nwork, int* dev_err,
                            cudaStream_t stream) {
  using namespace psgd;
  if (!items || nwork < 0 || (nwork > 0 && !work) || !dev_err) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, permute_kernel, PM_THREADS, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int grid = nwork < sms * per_sm ? nwork : sms * per_sm;
  permute_kernel<<<grid, PM_THREADS, 0, stream>>>(items, work, nwork);
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}
