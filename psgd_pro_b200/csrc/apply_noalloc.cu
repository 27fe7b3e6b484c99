// Clip + apply for one parameter using a fixed scratch array inside the library instead of caller memory
// (psgd_apply_noalloc in include/psgd_b200.h). For callers that cannot allocate device memory; the arithmetic is
// that of psgd_apply: avg = sqrt(sum(pg^2) / numel), g = clamp(pg * min(1, max_avg / avg), +-max_elem),
// param -= lr * g.
#include "common.cuh"
#include "psgd_b200.h"

#include <float.h>

#include <atomic>

namespace psgd {
namespace {

constexpr int NA_CHUNK = PSGD_APPLY_CHUNK;
constexpr int NA_SLOTS = PSGD_APPLY_NOALLOC_SLOTS;
constexpr int NA_THREADS = 256;

// One partial sum of squares per chunk of the gradient. Every GPU that loads the library holds these 16 KB until
// the process exits; all calls on a device share them.
static __device__ __align__(256) float g_apply_scratch[NA_SLOTS];

// Fixed-order block sum (identical result in every block that sums the same values).
__device__ __forceinline__ float na_block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < NA_THREADS / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

// Pass 1: slot b = sum of squares of chunk b. Every slot the second pass reads is written here first, so nothing
// left in the array by an earlier call is ever used.
__global__ void __launch_bounds__(NA_THREADS) na_sumsq_kernel(const float* __restrict__ pg, long long numel,
                                                              float* __restrict__ scratch) {
  __shared__ float red[NA_THREADS / 32];
  const long long base = (long long)blockIdx.x * NA_CHUNK;
  const long long end = min(base + (long long)NA_CHUNK, numel);
  float s = 0.f;
  for (long long k = base + threadIdx.x; k < end; k += NA_THREADS) {
    const float v = pg[k];
    s += v * v;
  }
  const float t = na_block_sum(s, red);
  if (threadIdx.x == 0) scratch[blockIdx.x] = t;
}

// Pass 2: every block sums the nslots partials in the same order (so all blocks use the same clip scale) and
// updates its chunk of the parameter.
__global__ void __launch_bounds__(NA_THREADS) na_apply_kernel(void* param, int param_bf16,
                                                              const float* __restrict__ pg, long long numel,
                                                              int nslots, float lr, float max_avg, float max_elem,
                                                              const float* __restrict__ scratch) {
  __shared__ float red[NA_THREADS / 32];
  float s = 0.f;
  for (int t = threadIdx.x; t < nslots; t += NA_THREADS) s += scratch[t];
  const float total = na_block_sum(s, red);
  const float avg = sqrtf(total / (float)numel);
  // as psgd_pro.py:374-376: scale only when avg > max_avg (a NaN avg leaves the scale 1)
  const float sc = avg > max_avg ? max_avg / avg : 1.f;
  const long long base = (long long)blockIdx.x * NA_CHUNK;
  const long long end = min(base + (long long)NA_CHUNK, numel);
  for (long long k = base + threadIdx.x; k < end; k += NA_THREADS) {
    const float x = pg[k] * sc;
    const float g = isnan(x) ? x : fminf(fmaxf(x, -max_elem), max_elem);  // torch.clamp keeps NaN
    if (param_bf16) {
      __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(param);
      p[k] = __float2bfloat16_rn(__bfloat162float(p[k]) - lr * g);
    } else {
      float* p = reinterpret_cast<float*>(param);
      p[k] = p[k] - lr * g;
    }
  }
}

// Device address of g_apply_scratch on the current device, looked up once per device with that device current.
// In host code the name g_apply_scratch is only a host-side stand-in, never a device address.
// The cache is shared by host threads: each entry is atomic (threads that race on the first call of a device
// look the address up twice and store the same value).
float* scratch_on_current_device() {
  static std::atomic<float*> addr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  float* a = addr[dev].load(std::memory_order_acquire);
  if (a == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_apply_scratch) != cudaSuccess || p == nullptr) return nullptr;
    a = static_cast<float*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}

}  // namespace
}  // namespace psgd

extern "C" int psgd_apply_noalloc(void* param, int param_bf16, const float* pg, long long numel, float lr_params,
                                  float max_avg_amp, float max_elem_amp, cudaStream_t stream) {
  using namespace psgd;
  if (param == nullptr || pg == nullptr || numel < 0) return PSGD_EINVAL;
  if (numel > PSGD_APPLY_NOALLOC_MAX_NUMEL) return PSGD_ELIMIT;
  if (numel == 0) return PSGD_OK;
  // An error left pending by earlier, unrelated work is not this call's: launch nothing and leave it in place
  // for its owner to read (the launch checks below would otherwise report and clear it).
  if (cudaPeekAtLastError() != cudaSuccess) return PSGD_ELAUNCH;
  float* scratch = scratch_on_current_device();
  if (scratch == nullptr) return PSGD_ELAUNCH;
  const int nslots = (int)((numel + NA_CHUNK - 1) / NA_CHUNK);
  na_sumsq_kernel<<<nslots, NA_THREADS, 0, stream>>>(pg, numel, scratch);
  if (cudaGetLastError() != cudaSuccess) return PSGD_ELAUNCH;
  na_apply_kernel<<<nslots, NA_THREADS, 0, stream>>>(param, param_bf16, pg, numel, nslots, lr_params, max_avg_amp,
                                                     max_elem_amp, scratch);
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}
