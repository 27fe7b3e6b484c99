// Memory-bound kernels of the PSGD-Kron step (everything that is not a tensor-core contraction): gradient
// staging with the damping noise, the start of the norm lower bounds, per-factor scalar updates (L, the diagonal
// factors, the Procrustes step size), Rn = Q - Q^T, the Procrustes multiplier, and clip + apply.
// Grouped: one launch covers every parameter / factor of a phase through a device item array (and a tile work
// list for the tiled kernels). Reductions are deterministic (fixed-order partials, no atomics).
#include <atomic>

#include "common.cuh"
#include "psgd_b200.h"

#include <float.h>

namespace psgd {

constexpr int TT = 32;        // tile edge of the tiled element-wise kernels
constexpr int TROWS = 8;      // threads per tile column (256 threads, 4 rows each)
constexpr int PREP_ROWS = PSGD_PREP_ROWS;  // rows per work entry of the row-vector staging path

PSGD_DEVI float load_g(const void* g, int bf16, long long idx) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g)[idx])
              : reinterpret_cast<const float*>(g)[idx];
}

PSGD_DEVI void store_g(void* g, int bf16, long long idx, float v) {
  if (bf16) reinterpret_cast<__nv_bfloat16*>(g)[idx] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(g)[idx] = v;
}

// The momentum EMA of psgd_pro.py:340-341, m.mul_(beta).add_(g, alpha=1 - beta) on a tensor of g's dtype: each
// in-place op rounds to that dtype (bf16: the product, then the sum).
PSGD_DEVI float round_dt(float v, bool bf16) { return bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : v; }
PSGD_DEVI float ema_value(float m, float g, float beta, float alpha, bool bf16) {
  return round_dt(fmaf(alpha, g, round_dt(m * beta, bf16)), bf16);
}

// The staged source value of element idx: g, or the momentum (after this pass's EMA when it applies it).
PSGD_DEVI float load_src(const PsgdPrepItem& it, const void* src, bool ema, long long idx, float beta, float alpha) {
  if (!ema) return load_g(src, it.g_bf16, idx);
  const float v = ema_value(load_g(it.m, it.g_bf16, idx), load_g(it.g, it.g_bf16, idx), beta, alpha, it.g_bf16);
  store_g(it.m, it.g_bf16, idx, v);
  return v;
}

PSGD_DEVI void store_split(void* hi, void* lo, long long idx, float v) {
  __nv_bfloat16 h, l;
  split_bf16(v, h, l);
  reinterpret_cast<__nv_bfloat16*>(hi)[idx] = h;
  if (lo) reinterpret_cast<__nv_bfloat16*>(lo)[idx] = l;
}

PSGD_DEVI float load_split(const void* hi, const void* lo, long long idx) {
  float v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(hi)[idx]);
  if (lo) v += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(lo)[idx]);
  return v;
}

// ---- counter-based normal numbers ----------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11): ten rounds of
// two 32 x 32 -> 64-bit multiplications on a 4-word counter, the 2-word key bumped by Weyl constants between
// rounds. The four output words become four standard normal numbers by two Box-Muller transforms.
PSGD_DEVI uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// The ten round keys of a key (k0, k1), formed once per thread: the generator's rounds then take them as operands
// instead of bumping the key between rounds.
struct PhiloxKeys {
  uint32_t k0[10], k1[10];
};
PSGD_DEVI PhiloxKeys philox_keys(uint32_t k0, uint32_t k1) {
  PhiloxKeys ks;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    ks.k0[r] = k0 + (uint32_t)r * 0x9E3779B9u;
    ks.k1[r] = k1 + (uint32_t)r * 0xBB67AE85u;
  }
  return ks;
}
PSGD_DEVI uint4 philox4x32_10(uint4 c, const PhiloxKeys& ks) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ ks.k0[r], lo1, hi0 ^ c.w ^ ks.k1[r], lo0);
  }
  return c;
}

// Numbers 4 blk .. 4 blk + 3 of the sequence with key (k0, k1).
PSGD_DEVI float unit_open(uint32_t w) {  // ((w >> 9) + 1/2) / 2^23, exactly: [1, 2) by its bits, minus 1 - 2^-24
  return __uint_as_float(0x3f800000u | (w >> 9)) - 0.99999994039535522f;
}
PSGD_DEVI float4 normal4_words(const uint4 w);
PSGD_DEVI float4 normal4(unsigned long long blk, uint32_t k0, uint32_t k1) {
  return normal4_words(philox4x32_10(make_uint4((uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u), k0, k1));
}
PSGD_DEVI float4 normal4(unsigned long long blk, const PhiloxKeys& ks) {
  return normal4_words(philox4x32_10(make_uint4((uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u), ks));
}
// The four numbers of one generator output.
PSGD_DEVI float4 normal4_words(const uint4 w) {
  const float u0 = unit_open(w.x), u1 = unit_open(w.y), u2 = unit_open(w.z), u3 = unit_open(w.w);
  // hardware approximations of log, reciprocal square root, sin and cos (errors near 1e-6, far below what damping
  // noise needs); -2 ln u > 0 for every u above; the angle 2 pi u - pi lies in (-pi, pi), where __sincosf is most
  // accurate
  const float t0 = -2.f * __logf(u0), t2 = -2.f * __logf(u2);
  const float r0 = t0 * rsqrtf(t0), r1 = t2 * rsqrtf(t2);
  constexpr float TWO_PI = 6.2831853071795865f, PI = 3.1415926535897932f;
  float s0, c0, s1, c1;
  __sincosf(TWO_PI * u1 - PI, &s0, &c0);
  __sincosf(TWO_PI * u3 - PI, &s1, &c1);
  return make_float4(r0 * c0, r0 * s0, r1 * c1, r1 * s1);
}

// Number s of the sequence.
PSGD_DEVI float normal1(unsigned long long s, uint32_t k0, uint32_t k1) {
  const float4 v = normal4(s >> 2, k0, k1);
  const int i = (int)(s & 3);
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// ---- gradient staging ------------------------------------------------------------------------------------------
// floor(k / d) for 0 <= k < 8 d: for d <= 2^16 by one float multiply ((k + 1/2) / d lies at least 1 / (2 d) from
// every integer, far more than the rounding error of (k + 1/2) * (1/d), below 2^-20 for quotients under 8; checked
// exhaustively for every such d), else by integer division.
PSGD_DEVI int div_small(int k, int d, float inv_d) { return d <= 65536 ? (int)(((float)k + 0.5f) * inv_d) : k / d; }

// PREP_NORMAL rows r0 .. r0 + rows - 1 in 8-element vectors (16-byte bf16 G chunks, two for fp32 G; 16-byte
// operand stores). Each thread first requests PREP_VEC vectors' G chunks into its own shared-memory slots
// (cp.async: the loads are in flight together without holding registers), then converts them one at a time.
constexpr int PREP_VEC = 8;                                     // bf16 G vectors per thread per batch (fp32: half)
constexpr int PREP_SMEM = PREP_VEC * 256 * (int)sizeof(uint4);  // 32 KB: a thread's slots at stage[s * 256 + t]

PSGD_DEVI void cp_async16_raw(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}

// Eight consecutive values as bf16 operand halves at element o: hi = bf16(x) two at a time (packed conversions),
// lo = bf16(x - hi) only when a lo half is staged (16-byte stores).
PSGD_DEVI void st8_split(void* out_hi, void* out_lo, long long o, const float* x) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out_hi) + o) = *reinterpret_cast<const uint4*>(h);
  if (out_lo) {
    __align__(16) __nv_bfloat162 l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 hf = __bfloat1622float2(h[i]);
      l[i] = __floats2bfloat162_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out_lo) + o) = *reinterpret_cast<const uint4*>(l);
  }
}

// EMA: the item's momentum EMA runs in this pass (g is staged through shared memory, m is read into registers for
// the whole batch before the conversions, and the new m is written back); otherwise `src` (g or m) is staged.
template <bool BF16, bool EMA>
PSGD_DEVI void prep_rows_vec8(const PsgdPrepItem& it, const void* gsrc, long long r0, int rows, float damping,
                              bool gen, const PhiloxKeys& ks, float mbeta, float malpha, uint4* stage) {
  constexpr int PV = BF16 ? PREP_VEC : PREP_VEC / 2, CH = BF16 ? 1 : 2;  // vectors per batch, chunks per vector
  const int nvr = it.n2 >> 3, nvec = rows * nvr, t = threadIdx.x;
  const float inv_nvr = 1.f / (float)nvr;
  for (int base = t; base < nvec; base += blockDim.x * PV) {
    uint4 mv[EMA ? PV * CH : 1];
#pragma unroll
    for (int s = 0; s < PV; ++s) {
      const int j = base + s * blockDim.x;
      if (j < nvec) {
        const int r = div_small(j, nvr, inv_nvr);
        const long long idx = (r0 + r) * it.n2 + (long long)(j - r * nvr) * 8;
        const char* src = reinterpret_cast<const char*>(gsrc) + idx * (BF16 ? 2 : 4);
#pragma unroll
        for (int c = 0; c < CH; ++c) cp_async16_raw(stage + (s * CH + c) * 256 + t, src + 16 * c);
        if (EMA) {
          const uint4* mp = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(it.m) + idx * (BF16 ? 2 : 4));
#pragma unroll
          for (int c = 0; c < CH; ++c) mv[(s * CH + c) % (EMA ? PV * CH : 1)] = mp[c];
        }
      }
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
#pragma unroll(EMA ? PV : 1)
    for (int s = 0; s < PV; ++s) {
      const int j = base + s * blockDim.x;
      if (j >= nvec) break;
      const int r = div_small(j, nvr, inv_nvr);
      const long long row = r0 + r, col = (long long)(j - r * nvr) * 8, idx = row * it.n2 + col;
      float x[8];
      if (BF16) {
        const uint4 v = stage[s * 256 + t];
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __bfloat162float(h[i]);
      } else {
        const float4 a = reinterpret_cast<const float4*>(stage)[(2 * s) * 256 + t];
        const float4 b = reinterpret_cast<const float4*>(stage)[(2 * s + 1) * 256 + t];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      }
      if (EMA) {  // x holds g: m = rn(rn(beta m) + alpha g), written back, then staged
        uint4 mo[CH];
        if (BF16) {
          const uint4 v = mv[(s * CH) % (EMA ? PV * CH : 1)];
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
          __align__(16) __nv_bfloat16 o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            o[i] = __float2bfloat16_rn(fmaf(malpha, x[i], round_dt(__bfloat162float(h[i]) * mbeta, true)));
            x[i] = __bfloat162float(o[i]);
          }
          mo[0] = *reinterpret_cast<const uint4*>(o);
        } else {
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const uint4 v = mv[(s * CH + c) % (EMA ? PV * CH : 1)];
            const float mm[4] = {__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w)};
#pragma unroll
            for (int i = 0; i < 4; ++i) x[4 * c + i] = fmaf(malpha, x[4 * c + i], mm[i] * mbeta);
            mo[c] = make_uint4(__float_as_uint(x[4 * c]), __float_as_uint(x[4 * c + 1]), __float_as_uint(x[4 * c + 2]),
                               __float_as_uint(x[4 * c + 3]));
          }
        }
        uint4* mp = reinterpret_cast<uint4*>(reinterpret_cast<char*>(it.m) + idx * (BF16 ? 2 : 4));
#pragma unroll
        for (int c = 0; c < CH; ++c) mp[c] = mo[c];
      }
      const long long o = row * it.ld_out + col;
      if (it.out2_hi) st8_split(it.out2_hi, it.out2_lo, o, x);  // the clean operand, before the damping noise
      if (it.xi) {
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {
          const float4 z = gen ? normal4((unsigned long long)(it.noise_base + idx) / 4 + hv, ks)
                               : *reinterpret_cast<const float4*>(it.xi + idx + 4 * hv);
          const float zz[4] = {z.x, z.y, z.z, z.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) x[4 * hv + i] += (damping + it.eps * fabsf(x[4 * hv + i])) * zz[i];
        }
      }
      st8_split(it.out_hi, it.out_lo, o, x);
    }
  }
}

// MOM: the momentum fields of the items are honoured (a separate instantiation, so the staging without momentum
// keeps its register count and occupancy; psgd_prep launches MOM = false, psgd_prep_momentum MOM = true).
template <bool MOM>
__global__ void __launch_bounds__(256) prep_kernel(const PsgdPrepItem* __restrict__ items,
                                                  const uint32_t* __restrict__ work, int nwork,
                                                  const float* __restrict__ hyper) {
  extern __shared__ uint4 prep_stage[];  // PREP_SMEM bytes: the row-vector path's G slots
  __shared__ float tile[TT][TT + 1];
  __shared__ float colred[TROWS][TT];
  __shared__ float tred[TROWS];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float damping = hyper[PSGD_HY_DAMPING];
  const bool gen = hyper[PSGD_HY_NOISE] != 0.f;  // noise from the counter-based generator instead of xi
  const uint32_t k0 = __float_as_uint(hyper[PSGD_HY_NOISE_KEY0]), k1 = __float_as_uint(hyper[PSGD_HY_NOISE_KEY1]);
  const PhiloxKeys ks = philox_keys(k0, k1);
  const float mbeta = hyper[PSGD_HY_MOM_BETA], malpha = hyper[PSGD_HY_MOM_ALPHA];
  const int ema_phase = (int)hyper[PSGD_HY_EMA_PHASE];
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdPrepItem& it = items[work[2 * w]];
    // the staged source: g, or the momentum (this pass applies its EMA when the item's phase is this step's)
    const bool ema = MOM && it.m != nullptr && it.mom_phase == ema_phase;
    const void* src = (MOM && it.m != nullptr && !ema) ? it.m : it.g;
    if (it.mode == PSGD_PREP_NORMAL) {  // rows PREP_ROWS * wv .. : 4-element vectors along each row
      const long long r0 = (long long)work[2 * w + 1] * PREP_ROWS;
      const int rows = (int)min((long long)PREP_ROWS, it.n1 - r0);
      const bool vec = (it.n2 % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                       (!ema || (reinterpret_cast<uintptr_t>(it.m) & 15) == 0) &&
                       (it.xi == nullptr || (reinterpret_cast<uintptr_t>(it.xi) & 15) == 0) &&
                       (it.noise_base & 3) == 0 && (it.ld_out % 8) == 0 &&
                       (reinterpret_cast<uintptr_t>(it.out_hi) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(it.out_lo) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(it.out2_hi) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(it.out2_lo) & 15) == 0;
      if (vec) {
        if (MOM && ema) {
          if (it.g_bf16)
            prep_rows_vec8<true, true>(it, src, r0, rows, damping, gen, ks, mbeta, malpha, prep_stage);
          else
            prep_rows_vec8<false, true>(it, src, r0, rows, damping, gen, ks, mbeta, malpha, prep_stage);
        } else {
          if (it.g_bf16)
            prep_rows_vec8<true, false>(it, src, r0, rows, damping, gen, ks, mbeta, malpha, prep_stage);
          else
            prep_rows_vec8<false, false>(it, src, r0, rows, damping, gen, ks, mbeta, malpha, prep_stage);
        }
      } else {
        for (int k = threadIdx.x; k < rows * it.n2; k += blockDim.x) {
          const long long row = r0 + k / it.n2, col = k % it.n2;
          const long long idx = row * it.n2 + col;
          float x = load_src(it, src, ema, idx, mbeta, malpha);
          if (it.out2_hi) store_split(it.out2_hi, it.out2_lo, row * it.ld_out + col, x);
          if (it.xi) x += (damping + it.eps * fabsf(x)) * (gen ? normal1(it.noise_base + idx, k0, k1) : it.xi[idx]);
          store_split(it.out_hi, it.out_lo, row * it.ld_out + col, x);
        }
      }
      continue;
    }
    const int ti = work[2 * w + 1] >> 16, tj = work[2 * w + 1] & 0xFFFF;
    const int i0 = ti * TT, j0 = tj * TT;
    const int j = j0 + tx;
    float vals[TT / TROWS];
#pragma unroll
    for (int u = 0; u < TT / TROWS; ++u) {
      const int i = i0 + ty + u * TROWS;
      float x = 0.f;
      if (i < it.n1 && j < it.n2) {
        const long long idx = (long long)i * it.n2 + j;
        x = load_src(it, src, ema, idx, mbeta, malpha);
        if (it.xi) x += (damping + it.eps * fabsf(x)) * (gen ? normal1(it.noise_base + idx, k0, k1) : it.xi[idx]);
      }
      vals[u] = x;
    }
    if (it.mode == PSGD_PREP_TRANS) {
      const float s2 = (it.p2 && j < it.n2) ? it.p2[j] : 1.f;
#pragma unroll
      for (int u = 0; u < TT / TROWS; ++u) tile[ty + u * TROWS][tx] = vals[u] * s2;
      __syncthreads();
#pragma unroll
      for (int u = 0; u < TT / TROWS; ++u) {
        const int jj = j0 + ty + u * TROWS, ii = i0 + tx;  // output row jj, column ii
        if (jj < it.n2 && ii < it.n1) store_split(it.out_hi, it.out_lo, (long long)jj * it.ld_out + ii, tile[tx][ty + u * TROWS]);
      }
      __syncthreads();
    } else {  // PSGD_PREP_DIRECT
      const float s2 = (it.p2 && j < it.n2) ? it.p2[j] : 1.f;
      float csum = 0.f, tsum = 0.f;
#pragma unroll
      for (int u = 0; u < TT / TROWS; ++u) {
        const int i = i0 + ty + u * TROWS;
        const bool ok = i < it.n1 && j < it.n2;
        const float s1 = (it.p1 && i < it.n1) ? it.p1[i] : 1.f;
        const float v = ok ? s1 * vals[u] * s2 : 0.f;
        if (ok && it.out_f32) it.out_f32[(long long)i * it.n2 + j] = v;
        const float v2 = v * v;
        csum += v2;
        const float rs = warp_sum(v2);  // this warp holds one row of the tile
        if (tx == 0 && it.part_row && i < it.n1) it.part_row[(long long)tj * it.n1 + i] = rs;
        tsum += rs;
      }
      colred[ty][tx] = csum;
      if (tx == 0) tred[ty] = tsum;
      __syncthreads();
      if (ty == 0) {
        float c = 0.f;
#pragma unroll
        for (int r = 0; r < TROWS; ++r) c += colred[r][tx];
        if (it.part_col && j < it.n2) it.part_col[(long long)ti * it.n2 + j] = c;
        if (tx == 0 && it.part_tile) {
          float t = 0.f;
#pragma unroll
          for (int r = 0; r < TROWS; ++r) t += tred[r];
          const int tiles_j = (it.n2 + TT - 1) / TT;
          it.part_tile[(long long)ti * tiles_j + tj] = t;
        }
      }
      __syncthreads();
    }
  }
}

// ---- norm lower bound start --------------------------------------------------------------------------------------
constexpr int NLB_THREADS = 512;

__global__ void __launch_bounds__(NLB_THREADS) nlb_prep_kernel(const PsgdNlbPrepItem* __restrict__ items) {
  const PsgdNlbPrepItem& it = items[blockIdx.x];
  const int n = it.n, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  __shared__ float s_val[NLB_THREADS / 32];
  __shared__ int s_idx[NLB_THREADS / 32];
  __shared__ float s_dot[32][NLB_THREADS / 32];
  __shared__ float s_nf;
  __shared__ int s_j;
  // argmax of row norms (first maximum) and the normalising factor
  float best = -1.f, mx = 0.f;
  int bj = 0x7fffffff;
  for (int i = tid; i < n; i += NLB_THREADS) {
    float r = 0.f;
    for (int s = 0; s < it.row_slots; ++s) r += it.part_row[(long long)s * n + i];
    if (r > best) { best = r; bj = i; }
    if (!it.skew) mx = fmaxf(mx, it.diag[i]);
  }
  if (it.skew)
    for (int t = tid; t < it.max_slots; t += NLB_THREADS) mx = fmaxf(mx, it.part_max[t]);
  if (!it.skew && tid >= n) mx = -FLT_MAX;
  // reduce (value desc, index asc) and max
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
    if (ob > best || (ob == best && oj < bj)) { best = ob; bj = oj; }
  }
  const float wmx = warp_max(mx);
  if (lane == 0) { s_val[wid] = best; s_idx[wid] = bj; s_dot[0][wid] = wmx; }
  __syncthreads();
  if (tid == 0) {
    float b = s_val[0], m = s_dot[0][0];
    int jj = s_idx[0];
    for (int w = 1; w < NLB_THREADS / 32; ++w) {
      if (s_val[w] > b || (s_val[w] == b && s_idx[w] < jj)) { b = s_val[w]; jj = s_idx[w]; }
      m = fmaxf(m, s_dot[0][w]);
    }
    s_nf = m + FLT_MIN;  // + smallest normal (psgd_pro.py:32, :56)
    s_j = (jj >= n || jj < 0) ? 0 : jj;
    *it.nf_out = s_nf;
  }
  __syncthreads();
  const float nf = s_nf;
  const long long rowj = (long long)s_j * it.lda;
  // dots <A_j / nf, V_r> for the 32 rows
  float dot[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) dot[r] = 0.f;
  for (int k = tid; k < n; k += NLB_THREADS) {
    const float a = load_split(it.a_hi, it.a_lo, rowj + k) / nf;
#pragma unroll
    for (int r = 0; r < 32; ++r) dot[r] += a * it.v[(long long)r * n + k];
  }
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    const float d = warp_sum(dot[r]);
    if (lane == 0) s_dot[r][wid] = d;
  }
  __syncthreads();
  if (tid < 32) {
    float d = 0.f;
    for (int w = 0; w < NLB_THREADS / 32; ++w) d += s_dot[tid][w];
    s_dot[tid][0] = d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);  // torch.sgn
  }
  __syncthreads();
  for (int k = tid; k < n; k += NLB_THREADS) {
    const float a = load_split(it.a_hi, it.a_lo, rowj + k) / nf;
#pragma unroll
    for (int r = 0; r < 32; ++r)
      store_split(it.v0_hi, it.v0_lo, (long long)r * it.ldv + k, a + s_dot[r][0] * it.v[(long long)r * n + k]);
  }
}

// Range c of nsplit ranges of 0 .. n (multiples of 32 long; empty past the end).
PSGD_DEVI void split_range(int n, int nsplit, int c, int& lo, int& hi) {
  const int ch = ((n + nsplit - 1) / nsplit + 31) & ~31;
  lo = min(n, c * ch);
  hi = min(n, lo + ch);
}

// ---- per-factor scalars ------------------------------------------------------------------------------------------
constexpr int FAC_THREADS = 256;

PSGD_DEVI float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

PSGD_DEVI float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = -FLT_MAX;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
  return t;
}

// max over columns c < ncols of sqrt(sum_t part[t * ncols + c])
PSGD_DEVI float max_col_norm(const float* part, int slots, int ncols, float* red) {
  float m = 0.f;
  for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
    float s = 0.f;
    for (int t = 0; t < slots; ++t) s += part[(long long)t * ncols + c];
    m = fmaxf(m, sqrtf(s));
  }
  return block_max(m, red);
}

// Blocks item * FAC_SPLIT + c: FACTOR_DIAG items use every c (ranges of their n entries), the others c = 0 only.
constexpr int FAC_SPLIT = PSGD_FAC_SPLIT;
static_assert(FAC_SPLIT + 1 <= PSGD_FAC_SCRATCH, "factor scratch too small");

__global__ void __launch_bounds__(FAC_THREADS) factor_kernel(const PsgdFactorItem* __restrict__ items,
                                                            const float* __restrict__ hyper, int* __restrict__ err) {
  const PsgdFactorItem& it = items[blockIdx.x / FAC_SPLIT];
  const int c = blockIdx.x % FAC_SPLIT;
  if (c != 0 && it.kind != PSGD_FACTOR_DIAG) return;
  __shared__ float red[FAC_THREADS / 32];
  const float lr = hyper[PSGD_HY_LR_PRECOND], betaL = hyper[PSGD_HY_BETA_L];
  if (it.kind == PSGD_FACTOR_DENSE || it.kind == PSGD_FACTOR_RANK1) {
    float ell;
    if (it.kind == PSGD_FACTOR_DENSE) {
      ell = *it.nf * max_col_norm(it.part, it.slots, it.ncols, red) + it.term2;
    } else {
      float s = 0.f;
      for (int t = threadIdx.x; t < it.slots; t += blockDim.x) s += it.part[t];
      ell = block_sum(s, red) + it.term2;
    }
    if (threadIdx.x == 0) {
      const float Lold = *it.L;
      const float L = fmaxf(betaL * Lold + (1.f - betaL) * ell, ell);
      *it.L = L;
      const float coef = lr / L;
      *it.alpha = -coef;
      *it.beta = 1.f + coef * it.term2;
      if (!isfinite(ell) || !isfinite(L) || !isfinite(coef)) atomicOr(err, ERR_NONFINITE);
    }
  } else if (it.kind == PSGD_FACTOR_DIAG) {  // this range's term1 (kept in p until factor_diag_kernel) and max
    int lo, hi;
    split_range(it.n, FAC_SPLIT, c, lo, hi);
    float m = -FLT_MAX;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      float t1 = 0.f;
      for (int s = 0; s < it.slots; ++s) t1 += it.part[(long long)s * it.n + i];
      it.p[i] = t1;
      m = fmaxf(m, t1);
    }
    m = block_max(m, red);
    if (threadIdx.x == 0) {
      it.scratch[c] = m;
      if (c == 0) it.scratch[FAC_SPLIT] = *it.L;
    }
  } else {  // PSGD_FACTOR_SKEW
    const float s = *it.nf * max_col_norm(it.part, it.slots, it.ncols, red) + FLT_MIN;
    float a1 = 0.f;
    for (int t = threadIdx.x; t < it.n_rq; t += blockDim.x) a1 += it.part_dot_rq[t];
    const float sum_rq = block_sum(a1, red);
    float a2 = 0.f;
    for (int t = threadIdx.x; t < it.n_sq; t += blockDim.x) a2 += it.part_dot_sq[t];
    const float sum_sq = block_sum(a2, red);
    if (threadIdx.x == 0) {
      // divide step by step, as the reference normalises R before its products: with R = 0 (Q exactly
      // symmetric) s is the smallest normal and every quotient stays finite
      const float tr_rq = sum_rq / s;
      const float tr_rrq = -((sum_sq / s) / s);
      const float amax = 0.125f;
      const float a = tr_rrq < 0.f ? fminf(-tr_rq / tr_rrq, amax) : amax;
      *it.alpha = a;
      *it.beta = 1.f / s;
      // fminf drops a NaN quotient: a non-finite trace or bound is flagged here
      if (!isfinite(s) || !isfinite(tr_rq) || !isfinite(tr_rrq)) atomicOr(err, ERR_NONFINITE);
    }
  }
}

// FACTOR_DIAG, second launch: ell = max term1 + term2 over the ranges, L and the update of q and p in this range.
__global__ void __launch_bounds__(FAC_THREADS) factor_diag_kernel(const PsgdFactorItem* __restrict__ items,
                                                                 const float* __restrict__ hyper,
                                                                 int* __restrict__ err) {
  const PsgdFactorItem& it = items[blockIdx.x / FAC_SPLIT];
  if (it.kind != PSGD_FACTOR_DIAG) return;
  const int c = blockIdx.x % FAC_SPLIT;
  const float lr = hyper[PSGD_HY_LR_PRECOND], betaL = hyper[PSGD_HY_BETA_L];
  float m = it.scratch[0];
  for (int k = 1; k < FAC_SPLIT; ++k) m = fmaxf(m, it.scratch[k]);
  const float ell = m + it.term2;
  const float Lold = it.scratch[FAC_SPLIT];
  const float L = fmaxf(betaL * Lold + (1.f - betaL) * ell, ell);
  const float coef = lr / L;
  int lo, hi;
  split_range(it.n, FAC_SPLIT, c, lo, hi);
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float q = it.q[i] * (1.f - coef * (it.p[i] - it.term2));
    it.q[i] = q;
    it.p[i] = q * q;
  }
  if (c == 0 && threadIdx.x == 0) {
    *it.L = L;
    if (!isfinite(ell) || !isfinite(L)) atomicOr(err, ERR_NONFINITE);
  }
}

// ---- Rn = Q - Q^T ------------------------------------------------------------------------------------------------
// Work entries are pairs of 64 x 64 tiles (TI <= TJ): A = Q[TI, TJ] and B = Q[TJ, TI] are read once into shared
// memory by cp.async (16-byte chunks when n % 4 == 0, a warp request covering two 256-byte tile rows), and both Rn
// tiles, Rn[TI, TJ] = A - B^T and Rn[TJ, TI] = B - A^T, are written (8-byte bf16 stores). The reductions go to the
// 32-wide slot layout of PsgdSkewItem: row sums into slot 2 TJ (or 2 TI), the pair's max and trace share into entry
// (2 TI) * tiles32 + 2 TJ; the slots no block writes stay zero.
constexpr int SK = PSGD_SKEW_TILE;

// Four values as bf16 hi and lo computed together (fewer live registers in the rank-one skew kernel).
PSGD_DEVI void st4_split_both(void* hi, void* lo, long long idx, const float* x, bool vec, int nvalid) {
  __align__(8) __nv_bfloat16 h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) split_bf16(x[i], h[i], l[i]);
  __nv_bfloat16* H = reinterpret_cast<__nv_bfloat16*>(hi) + idx;
  __nv_bfloat16* L = lo ? reinterpret_cast<__nv_bfloat16*>(lo) + idx : nullptr;
  if (vec) {
    *reinterpret_cast<uint2*>(H) = *reinterpret_cast<const uint2*>(h);
    if (L) *reinterpret_cast<uint2*>(L) = *reinterpret_cast<const uint2*>(l);
  } else {
    for (int i = 0; i < nvalid; ++i) {
      H[i] = h[i];
      if (L) L[i] = l[i];
    }
  }
}

// Four values as bf16 hi (two packed conversions) and, only when lo is given, the lo halves bf16(x - hi).
PSGD_DEVI void st4_split(void* hi, void* lo, long long idx, const float* x, bool vec, int nvalid) {
  __align__(8) __nv_bfloat162 h2[2];
  h2[0] = __floats2bfloat162_rn(x[0], x[1]);
  h2[1] = __floats2bfloat162_rn(x[2], x[3]);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(h2);
  __nv_bfloat16* H = reinterpret_cast<__nv_bfloat16*>(hi) + idx;
  if (vec) {
    *reinterpret_cast<uint2*>(H) = *reinterpret_cast<const uint2*>(h2);
  } else {
    for (int i = 0; i < nvalid; ++i) H[i] = h[i];
  }
  if (lo) {
    __align__(8) __nv_bfloat162 l2[2];
    const float2 f0 = __bfloat1622float2(h2[0]), f1 = __bfloat1622float2(h2[1]);
    l2[0] = __floats2bfloat162_rn(x[0] - f0.x, x[1] - f0.y);
    l2[1] = __floats2bfloat162_rn(x[2] - f1.x, x[3] - f1.y);
    const __nv_bfloat16* l = reinterpret_cast<const __nv_bfloat16*>(l2);
    __nv_bfloat16* L = reinterpret_cast<__nv_bfloat16*>(lo) + idx;
    if (vec) {
      *reinterpret_cast<uint2*>(L) = *reinterpret_cast<const uint2*>(l2);
    } else {
      for (int i = 0; i < nvalid; ++i) L[i] = l[i];
    }
  }
}

// Q[row][col0 .. col0 + 3] (zero outside the matrix).
PSGD_DEVI float4 load4q(const float* __restrict__ q, int n, int row, int col0, bool vec) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row >= n) return v;
  const float* src = q + (long long)row * n + col0;
  if (vec && col0 + 3 < n) return *reinterpret_cast<const float4*>(src);
  if (col0 < n) v.x = src[0];
  if (col0 + 1 < n) v.y = src[1];
  if (col0 + 2 < n) v.z = src[2];
  if (col0 + 3 < n) v.w = src[3];
  return v;
}

// Q[row][col0 .. col0 + 3] = v (the in-range elements).
PSGD_DEVI void store4q(float* __restrict__ q, int n, int row, int col0, bool vec, float4 v) {
  if (row >= n) return;
  float* dst = q + (long long)row * n + col0;
  if (vec && col0 + 3 < n) {
    *reinterpret_cast<float4*>(dst) = v;
    return;
  }
  if (col0 < n) dst[0] = v.x;
  if (col0 + 1 < n) dst[1] = v.y;
  if (col0 + 2 < n) dst[2] = v.z;
  if (col0 + 3 < n) dst[3] = v.w;
}

PSGD_DEVI float ldbf(const void* p, long long idx) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
}

// Shared-memory tile of the skew kernel: row r of a 64 x 64 fp32 tile starts at float r * 64 + (r & ~3) (a
// 16-byte gap after every four rows), so 16-byte cp.async chunks stay aligned and the transposed reads of a warp
// (16 columns x 2 rows) fall into 16 distinct banks.
constexpr int SK_TILE = SK * SK + SK;  // floats per staged tile
constexpr int SK_STAGES = 2;           // entries in flight per block: the next pair loads while this one computes
constexpr int SK_SMEM = SK_STAGES * 2 * SK_TILE * (int)sizeof(float);
PSGD_DEVI int sk_off(int r, int c) { return r * SK + (r & ~3) + c; }

PSGD_DEVI void cp_async16(float* dst, const float* src, bool ok) {  // zero-fills dst when !ok (src not read)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
PSGD_DEVI void cp_async4(float* dst, const float* src, bool ok) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(ok ? 4 : 0)
               : "memory");
}
PSGD_DEVI void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
PSGD_DEVI void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Requests work entry w's tiles into one stage: A = Q[TI, TJ] at stage[0 ..), B = Q[TJ, TI] at stage[SK_TILE ..)
// (not loaded on the diagonal, where B = A). Elements outside the matrix arrive as zeros. A warp covers two
// 256-byte tile rows per request.
PSGD_DEVI void skew_issue(const PsgdSkewItem* __restrict__ items, const uint32_t* __restrict__ work, int w,
                          float* stage, int t) {
  const PsgdSkewItem& it = items[work[2 * w]];
  const int ti = work[2 * w + 1] >> 16, tj = work[2 * w + 1] & 0xFFFF;
  const int n = it.n, i0 = ti * SK, j0 = tj * SK, nload = ti == tj ? 4 : 8;
  const float* q = it.q;
  const int c = 4 * (t & 15), r0 = t >> 4;
  if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {  // whole 16-byte chunks: each is inside the
    // matrix or wholly outside
    for (int j = 0; j < nload; ++j) {
      const int tile = j >> 2, r = r0 + 16 * (j & 3);
      const int gr = (tile ? j0 : i0) + r, gc = (tile ? i0 : j0) + c;
      const bool ok = gr < n && gc < n;
      cp_async16(stage + tile * SK_TILE + sk_off(r, c), ok ? q + (long long)gr * n + gc : q, ok);
    }
  } else {
    for (int j = 0; j < nload; ++j) {
      const int tile = j >> 2, r = r0 + 16 * (j & 3);
      const int gr = (tile ? j0 : i0) + r, gc = (tile ? i0 : j0) + c;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = gr < n && gc + e < n;
        cp_async4(stage + tile * SK_TILE + sk_off(r, c + e), ok ? q + (long long)gr * n + gc + e : q, ok);
      }
    }
  }
}

// The element-wise form runs the 1-D factors (psgd_skew_rank1, R1 = true: the items carry the rank-one q update,
// u_hi != NULL, applied to the staged tiles first); the 2-D factors take skew2_kernel below. Entries of a block are
// pipelined through SK_STAGES shared-memory stages (cp.async): entry k + SK_STAGES is requested as soon as entry k's
// tiles have been read.
template <bool R1>
__global__ void __launch_bounds__(256, 3) skew_kernel(const PsgdSkewItem* __restrict__ items,
                                                      const uint32_t* __restrict__ work, int nwork) {
  extern __shared__ __align__(16) float sk_stage[];
  __shared__ float red[8][2];
  // R1: u at the rows of A (i0 ..) and of B (j0 ..), v at the columns of A (j0 ..) and of B (i0 ..); hi and lo
  __shared__ float suv[R1 ? 4 : 1][2][SK];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int rr = t >> 4, c4 = (t & 15) * 4;  // this thread: rows rr + 16 m, columns c4 .. c4 + 3 of a tile
  int wnext = blockIdx.x;
  for (int st = 0; st < SK_STAGES; ++st, wnext += gridDim.x) {
    if (wnext < nwork) skew_issue(items, work, wnext, sk_stage + st * 2 * SK_TILE, t);
    cp_async_commit();
  }
  int st = 0;
  for (int w = blockIdx.x; w < nwork; w += gridDim.x, wnext += gridDim.x, st = st + 1 == SK_STAGES ? 0 : st + 1) {
    const PsgdSkewItem& it = items[work[2 * w]];
    const int ti = work[2 * w + 1] >> 16, tj = work[2 * w + 1] & 0xFFFF;
    const int n = it.n, i0 = ti * SK, j0 = tj * SK;
    const bool diag = ti == tj;
    const bool vec = (n % 4) == 0 && (reinterpret_cast<uintptr_t>(it.q) & 15) == 0;
    float* const sA = sk_stage + st * 2 * SK_TILE;
    float* const sB = diag ? sA : sA + SK_TILE;
    const bool r1 = R1 && it.u_hi != nullptr;
    if (r1) {  // the four 64-element segments of u and v this pair uses, one element per thread
      const int seg = t >> 6, e = t & 63;
      const int base = (seg == 0 || seg == 3) ? i0 : j0;
      const int idx = min(base + e, n - 1);
      const void* h = seg < 2 ? it.u_hi : it.v_hi;
      const void* l = seg < 2 ? it.u_lo : it.v_lo;
      const long long ld = seg < 2 ? it.ldu : it.ldv;
      suv[seg][0][e] = ldbf(h, (long long)idx * ld);
      suv[seg][1][e] = l ? ldbf(l, (long long)idx * ld) : 0.f;
    }
    cp_async_wait<SK_STAGES - 1>();  // this entry's group is complete (later groups may still be in flight)
    __syncthreads();
    float4 a[4], b[4];  // this thread's rows of A and B: the untransposed operands of the differences below
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      a[m] = *reinterpret_cast<const float4*>(sA + sk_off(rr + 16 * m, c4));
      b[m] = *reinterpret_cast<const float4*>(sB + sk_off(rr + 16 * m, c4));
    }
    float mx = 0.f, dsum = 0.f;
    const int tiles32 = (n + 31) / 32;
    // FULL: both tiles lie inside the matrix and every access is a whole vector: no bounds tests per element
    const bool full = vec && i0 + SK <= n && j0 + SK <= n && (it.ldr % 4) == 0 && (!r1 || (it.ldqt % 4) == 0);
    auto body = [&](auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
      if (r1) {  // the rank-one q update of this pair of tiles, written back before Rn is formed from it
        const float al = *it.alpha, be = *it.beta;
        float vha[4], vla[4], vhb[4], vlb[4];  // v at A's columns j0 + c4 + k and at B's columns i0 + c4 + k
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          vha[k] = suv[2][0][c4 + k];
          vla[k] = suv[2][1][c4 + k];
          vhb[k] = suv[3][0][c4 + k];
          vlb[k] = suv[3][1][c4 + k];
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int ia = i0 + rr + 16 * m, ib = j0 + rr + 16 * m;
          const float uha = suv[0][0][rr + 16 * m], ula = suv[0][1][rr + 16 * m];
          const float uhb = suv[1][0][rr + 16 * m], ulb = suv[1][1][rr + 16 * m];
          float xa[4] = {a[m].x, a[m].y, a[m].z, a[m].w}, xb[4] = {b[m].x, b[m].y, b[m].z, b[m].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // the K = 1 product as the tensor cores form it (hi * hi, then + hi * lo, then + lo * hi), then the
            // q-update epilogue: alpha * acc + beta * q
            float acc = uha * vha[k];
            acc = fmaf(uha, vla[k], acc);
            acc = fmaf(ula, vha[k], acc);
            xa[k] = (FULL || (ia < n && j0 + c4 + k < n)) ? fmaf(be, xa[k], acc * al) : 0.f;
            float bcc = uhb * vhb[k];
            bcc = fmaf(uhb, vlb[k], bcc);
            bcc = fmaf(ulb, vhb[k], bcc);
            xb[k] = (FULL || (ib < n && i0 + c4 + k < n)) ? fmaf(be, xb[k], bcc * al) : 0.f;
          }
          a[m] = make_float4(xa[0], xa[1], xa[2], xa[3]);
          b[m] = diag ? a[m] : make_float4(xb[0], xb[1], xb[2], xb[3]);
          if (FULL)
            *reinterpret_cast<float4*>(it.q + (long long)ia * n + j0 + c4) = a[m];
          else
            store4q(it.q, n, ia, j0 + c4, vec, a[m]);
          *reinterpret_cast<float4*>(sA + sk_off(rr + 16 * m, c4)) = a[m];
          if (!diag) {
            if (FULL)
              *reinterpret_cast<float4*>(it.q + (long long)ib * n + i0 + c4) = b[m];
            else
              store4q(it.q, n, ib, i0 + c4, vec, b[m]);
            *reinterpret_cast<float4*>(sB + sk_off(rr + 16 * m, c4)) = b[m];
          }
        }
        __syncthreads();
      }
      for (int half = 0; half < (diag ? 1 : 2); ++half) {
        // half 0: Rn[TI, TJ] rows i0 + r = A[r][c] - B[c][r]; half 1: Rn[TJ, TI] rows j0 + r = B[r][c] - A[c][r]
        const float* Y = half == 0 ? sB : sA;
        const int gr0 = half == 0 ? i0 : j0, gj0 = (half == 0 ? j0 : i0) + c4;
        const int slot = 2 * (half == 0 ? tj : ti);
        const int nv = FULL ? 4 : max(0, min(4, n - gj0));
        const bool vs = FULL || (nv == 4 && (it.ldr % 4) == 0);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int r = rr + 16 * m, gi = gr0 + r;
          const float4 xv = half == 0 ? a[m] : b[m];
          const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
          float yv[4], v[4], rs = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const bool ok = FULL || (gi < n && gj0 + k < n);
            const float x = xs[k];
            yv[k] = Y[sk_off(c4 + k, r)];
            v[k] = ok ? x - yv[k] : 0.f;
            rs += v[k] * v[k];
            mx = fmaxf(mx, fabsf(v[k]));
          }
          // sum Rn o Q = sum over (i, j) of (Q_ij - Q_ji) Q_ij = (1/2) sum Rn^2: over a pair of tiles that is the
          // sum of squares of one of its two Rn tiles (half 0), or half of it for a tile on the diagonal
          if (half == 0) dsum += diag ? 0.5f * rs : rs;
          if (FULL || (gi < n && nv > 0)) {
            if constexpr (R1) st4_split_both(it.r_hi, it.r_lo, (long long)gi * it.ldr + gj0, v, vs, nv);
            else st4_split(it.r_hi, it.r_lo, (long long)gi * it.ldr + gj0, v, vs, nv);
          }
          if (r1 && (FULL || (gi < n && nv > 0)))  // q^T of the updated q: row gi is the transposed operand above
            st4_split_both(it.qt_hi, it.qt_lo, (long long)gi * it.ldqt + gj0, yv,
                           FULL || (nv == 4 && (it.ldqt % 4) == 0), nv);
          rs += __shfl_xor_sync(0xffffffffu, rs, 1);
          rs += __shfl_xor_sync(0xffffffffu, rs, 2);
          rs += __shfl_xor_sync(0xffffffffu, rs, 4);
          rs += __shfl_xor_sync(0xffffffffu, rs, 8);
          if ((t & 15) == 0 && (FULL || gi < n)) it.part_row[(long long)slot * n + gi] = rs;
        }
      }
    };
    if (full)
      body(std::true_type());
    else
      body(std::false_type());
    mx = warp_max(mx);
    dsum = warp_sum(dsum);
    if (lane == 0) {
      red[wid][0] = mx;
      red[wid][1] = dsum;
    }
    __syncthreads();  // every thread is done with this stage: refill it
    if (wnext < nwork) skew_issue(items, work, wnext, sA, t);
    cp_async_commit();
    if (t == 0) {
      float m = 0.f, d = 0.f;
      for (int k = 0; k < 8; ++k) {
        m = fmaxf(m, red[k][0]);
        d += red[k][1];
      }
      it.part_max[(long long)(2 * ti) * tiles32 + 2 * tj] = m;
      it.part_dot[(long long)(2 * ti) * tiles32 + 2 * tj] = d;
    }
  }
  cp_async_wait<0>();
}

// ---- Rn = Q - Q^T, block form (2-D factors without the rank-one update) -------------------------------------------
// The same work entries, outputs and reductions as skew_kernel, with each thread owning whole 4 x 4 blocks: thread
// (bi, bj) = (t / 16, t % 16) forms block (bi, bj) of D = Rn[TI, TJ] = A - B^T from rows 4 bi .. 4 bi + 3 of A and
// rows 4 bj .. 4 bj + 3 of B (eight 16-byte shared-memory reads, the transposition in registers) and writes it and
// its mirror -D^T, block (bj, bi) of Rn[TJ, TI]. No element is read transposed from shared memory. The staged tiles
// keep 256-byte rows with their 16-byte chunks permuted (chunk c of row r at position c ^ ((r / 4) mod 16)), which
// makes the cp.async writes, the row reads of A and the block reads of B all free of bank conflicts. Row sums of
// squares go through shared memory (partials per 4-column block, summed in a fixed order). Entries are pipelined
// through SK2_STAGES stages; two blocks share an SM. D's rows leave straight from the registers (16 lanes write one
// 128-byte row); the mirror's rows are spread over all warps, so it passes through an 8 KB block (MIR) first.
constexpr int SK2_STAGES = 3;
constexpr int SK2_TILE = SK * SK;                                  // floats per staged tile
constexpr int SK2_SQ = SK * 17;                                    // one partial array: 64 rows x 16 (+1 pad)
constexpr int SK2_MIR = SK * SK * 2;                               // bytes: one bf16 64 x 64 tile
constexpr int SK2_SMEM = (SK2_STAGES * 2 * SK2_TILE + 2 * SK2_SQ) * (int)sizeof(float) + SK2_MIR;
PSGD_DEVI int sk2_off(int r, int chunk) { return r * SK + ((chunk ^ ((r >> 2) & 15)) << 2); }

// The fields of a work entry the block needs (read one iteration ahead of use, so the dependent loads of the work
// list and the item do not stall the block at the start of an entry).
struct Sk2Meta {
  const float* q;
  void* r_hi;
  void* r_lo;
  float* part_row;
  float* part_max;
  float* part_dot;
  long long ldr;
  int n, ti, tj;
};
PSGD_DEVI Sk2Meta sk2_meta(const PsgdSkewItem* __restrict__ items, const uint32_t* __restrict__ work, int w,
                           int nwork) {
  Sk2Meta m{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, 0, 0, 0};
  if (w < nwork) {
    const uint32_t e = work[2 * w + 1];
    const PsgdSkewItem& it = items[work[2 * w]];
    m = Sk2Meta{it.q, it.r_hi, it.r_lo, it.part_row, it.part_max, it.part_dot, it.ldr, it.n, (int)(e >> 16),
                (int)(e & 0xFFFF)};
  }
  return m;
}

PSGD_DEVI void skew2_issue(const Sk2Meta& m, float* stage, int t) {
  const int n = m.n, i0 = m.ti * SK, j0 = m.tj * SK, nload = m.ti == m.tj ? 4 : 8;
  const float* q = m.q;
  const int ch = t & 15, r0 = t >> 4;
  const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0;
  for (int j = 0; j < nload; ++j) {
    const int tile = j >> 2, r = r0 + 16 * (j & 3);
    const int gr = (tile ? j0 : i0) + r, gc = (tile ? i0 : j0) + 4 * ch;
    float* dst = stage + tile * SK2_TILE + sk2_off(r, ch);
    if (vec) {  // whole 16-byte chunks: each is inside the matrix or wholly outside (zero-filled)
      const bool ok = gr < n && gc < n;
      cp_async16(dst, ok ? q + (long long)gr * n + gc : q, ok);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = gr < n && gc + e < n;
        cp_async4(dst + e, ok ? q + (long long)gr * n + gc + e : q, ok);
      }
    }
  }
}

// Mirror staging (interior pairs with 16-byte aligned rows): the bf16 mirror -D^T is written into MIR (128-byte rows
// of sixteen 8-byte units, unit u of row r at u ^ ((r / 4) mod 16), free of bank conflicts for both the block writes
// and the row reads) and leaves in 16-byte row chunks; in fp32 mode its lo half takes a second round through MIR.
PSGD_DEVI int sk2_unit(int r, int u) { return r * 16 + (u ^ ((r >> 2) & 15)); }  // in 8-byte units

PSGD_DEVI uint2 pack4_bf16(const float* x) {
  const __nv_bfloat162 h0 = __floats2bfloat162_rn(x[0], x[1]), h1 = __floats2bfloat162_rn(x[2], x[3]);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
}
PSGD_DEVI void lo4(const float* x, float* lo) {  // x - bf16(x), as the split stores it
#pragma unroll
  for (int i = 0; i < 4; ++i) lo[i] = x[i] - __bfloat162float(__float2bfloat16_rn(x[i]));
}

// Writes rows R = t / 8 and t / 8 + 32 of the 64 x 64 bf16 tile held in MIR, 16 bytes (chunk t % 8) each.
PSGD_DEVI void sk2_mirror_out(const uint8_t* mir, __nv_bfloat16* dst, long long ld, int row0, int col0, int t) {
  const int k = t & 7;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int R = (t >> 3) + 32 * h, f = (R >> 2) & 15;
    uint4 v = reinterpret_cast<const uint4*>(mir)[R * 8 + (k ^ (f >> 1))];
    if (f & 1) v = make_uint4(v.z, v.w, v.x, v.y);
    *reinterpret_cast<uint4*>(dst + (long long)(row0 + R) * ld + col0 + 8 * k) = v;
  }
}

__global__ void __launch_bounds__(256, 2) skew2_kernel(const PsgdSkewItem* __restrict__ items,
                                                       const uint32_t* __restrict__ work, int nwork) {
  extern __shared__ __align__(16) float sk2_smem[];
  float* const sq0 = sk2_smem + SK2_STAGES * 2 * SK2_TILE;  // [row of D][bj]: row sums over 4-column blocks
  float* const sq1 = sq0 + SK2_SQ;                          // [row of -D^T][bi]
  uint8_t* const mir = reinterpret_cast<uint8_t*>(sq1 + SK2_SQ);
  __shared__ float red[8][2];
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int bi = t >> 4, bj = t & 15;
  int wnext = blockIdx.x;
  for (int st = 0; st < SK2_STAGES; ++st, wnext += gridDim.x) {
    if (wnext < nwork) skew2_issue(sk2_meta(items, work, wnext, nwork), sk2_smem + st * 2 * SK2_TILE, t);
    cp_async_commit();
  }
  int st = 0;
  Sk2Meta it = sk2_meta(items, work, blockIdx.x, nwork);  // this entry's fields
  for (int w = blockIdx.x; w < nwork; w += gridDim.x, wnext += gridDim.x, st = st + 1 == SK2_STAGES ? 0 : st + 1) {
    // requested now, used after the entry's barrier (the entry refilling this stage) and in the next iteration
    const Sk2Meta im = sk2_meta(items, work, wnext, nwork);
    const Sk2Meta nm = sk2_meta(items, work, w + gridDim.x, nwork);
    const int ti = it.ti, tj = it.tj;
    const int n = it.n, i0 = ti * SK, j0 = tj * SK;
    const bool diag = ti == tj;
    float* const sA = sk2_smem + st * 2 * SK2_TILE;
    const float* const sB = diag ? sA : sA + SK2_TILE;
    // this entry's group is complete (later groups may still be in flight); the previous entry's reads of MIR, the
    // partials and red are done
    cp_async_wait<SK2_STAGES - 1>();
    __syncthreads();
    float d[4][4];  // d[r][c] = A[4 bi + r][4 bj + c] - B[4 bj + c][4 bi + r]
    {
      float4 a[4], b[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r] = *reinterpret_cast<const float4*>(sA + sk2_off(4 * bi + r, bj));
#pragma unroll
      for (int c = 0; c < 4; ++c) b[c] = *reinterpret_cast<const float4*>(sB + sk2_off(4 * bj + c, bi));
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float ar[4] = {a[r].x, a[r].y, a[r].z, a[r].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float bc[4] = {b[c].x, b[c].y, b[c].z, b[c].w};
          d[r][c] = ar[c] - bc[r];
        }
      }
    }
    // elements outside the matrix were staged as zeros on both sides, so they contribute 0 to every reduction
    float mx = 0.f, rsum[4], csum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      rsum[r] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float v2 = d[r][c] * d[r][c];
        rsum[r] += v2;
        csum[c] += v2;
        mx = fmaxf(mx, fabsf(d[r][c]));
      }
    }
    // sum Rn o Q over the pair = (1/2) sum Rn^2 over its two tiles = sum D^2 (a tile on the diagonal: half of it)
    float dsum = ((rsum[0] + rsum[1]) + rsum[2]) + rsum[3];
    if (diag) dsum *= 0.5f;
#pragma unroll
    for (int r = 0; r < 4; ++r) sq0[(4 * bi + r) * 17 + bj] = rsum[r];
    if (!diag) {
#pragma unroll
      for (int c = 0; c < 4; ++c) sq1[(4 * bj + c) * 17 + bi] = csum[c];
    }
    mx = warp_max(mx);
    dsum = warp_sum(dsum);
    if (lane == 0) {
      red[wid][0] = mx;
      red[wid][1] = dsum;
    }
    const bool lo = it.r_lo != nullptr;
    // Rn[TI, TJ] rows i0 + 4 bi + r, columns j0 + 4 bj .. (16 lanes cover one 128-byte row)
    const bool full = i0 + SK <= n && j0 + SK <= n;
    {
      const int col = j0 + 4 * bj, nv = full ? 4 : max(0, min(4, n - col));
      const bool vs = nv == 4 && (it.ldr % 4) == 0;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = i0 + 4 * bi + r;
        if (full || (row < n && nv > 0)) st4_split(it.r_hi, it.r_lo, (long long)row * it.ldr + col, d[r], vs, nv);
      }
    }
    // Rn[TJ, TI] rows j0 + 4 bj + c, columns i0 + 4 bi ..: through MIR when the rows take 16-byte chunks
    const bool staged = !diag && full && (it.ldr % 8) == 0 && (reinterpret_cast<uintptr_t>(it.r_hi) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(it.r_lo) & 15) == 0;
    uint2* const mu = reinterpret_cast<uint2*>(mir);
    if (staged) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float m[4] = {-d[0][c], -d[1][c], -d[2][c], -d[3][c]};
        mu[sk2_unit(4 * bj + c, bi)] = pack4_bf16(m);
      }
    } else if (!diag) {
      const int col = i0 + 4 * bi, nv = max(0, min(4, n - col));
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int row = j0 + 4 * bj + c;
        const float m[4] = {-d[0][c], -d[1][c], -d[2][c], -d[3][c]};
        if (row < n && nv > 0)
          st4_split(it.r_hi, it.r_lo, (long long)row * it.ldr + col, m, nv == 4 && (it.ldr % 4) == 0, nv);
      }
    }
    __syncthreads();  // the stage's tiles are dead; MIR, the partials and red are complete
    if (wnext < nwork) skew2_issue(im, sA, t);  // refill the stage with a later entry
    cp_async_commit();
    if (staged) {
      sk2_mirror_out(mir, reinterpret_cast<__nv_bfloat16*>(it.r_hi), it.ldr, j0, i0, t);
      if (lo) {  // second round through MIR for the lo half
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float m[4] = {-d[0][c], -d[1][c], -d[2][c], -d[3][c]};
          float l[4];
          lo4(m, l);
          mu[sk2_unit(4 * bj + c, bi)] = pack4_bf16(l);
        }
        __syncthreads();
        sk2_mirror_out(mir, reinterpret_cast<__nv_bfloat16*>(it.r_lo), it.ldr, j0, i0, t);
      }
    }
    if (t < 2 * SK) {  // row sums: threads 0..63 the rows of Rn[TI, TJ], 64..127 those of Rn[TJ, TI]
      const int h = t >> 6, r = t & (SK - 1);
      const int gi = (h ? j0 : i0) + r;
      if ((h == 0 || !diag) && gi < n) {
        const float* p = (h ? sq1 : sq0) + r * 17;
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) acc += p[k];
        it.part_row[(long long)(2 * (h ? ti : tj)) * n + gi] = acc;
      }
    }
    if (t == 0) {
      const int tiles32 = (n + 31) / 32;
      float m = 0.f, dd = 0.f;
      for (int k = 0; k < 8; ++k) {
        m = fmaxf(m, red[k][0]);
        dd += red[k][1];
      }
      it.part_max[(long long)(2 * ti) * tiles32 + 2 * tj] = m;
      it.part_dot[(long long)(2 * ti) * tiles32 + 2 * tj] = dd;
    }
    it = nm;
  }
  cp_async_wait<0>();
}

// ---- M = a Rn / s + a^2 / 2 (S / s) / s ----------------------------------------------------------------------------
// Rows of the padded n x ld bf16 arrays, 8 values (16 bytes) per vector; padding columns are zero and stay zero.
// Work entries: (item, first row of a block of ROT_ROWS rows). Each thread takes up to ROT_VEC vectors per pass
// and requests all their inputs before the first use.
constexpr int ROT_ROWS = PSGD_ROT_ROWS;
constexpr int ROT_VEC = 4;

PSGD_DEVI void unpack8(const uint4& u, float* f) {
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = __bfloat162float(h[i]);
}

// LO: the operands carry lo halves (fp32 mode); without them that code is compiled out (fewer registers, more
// blocks per SM).
template <bool LO>
__global__ void __launch_bounds__(256, LO ? 2 : 3) rot_kernel(const PsgdRotItem* __restrict__ items,
                                                 const uint32_t* __restrict__ work, int nwork) {
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdRotItem& it = items[work[2 * w]];
    const int r0 = (int)work[2 * w + 1];
    const float a = *it.alpha, inv_s = *it.beta, half_a2 = 0.5f * a * a;
    const int nvec = (int)(it.ldr / 8);
    const int total = min(ROT_ROWS, it.n - r0) * nvec;
    const float inv_nvec = 1.f / (float)nvec;
    __nv_bfloat16* rbase_h = reinterpret_cast<__nv_bfloat16*>(it.r_hi);
    __nv_bfloat16* rbase_l = LO ? reinterpret_cast<__nv_bfloat16*>(it.r_lo) : nullptr;
    const __nv_bfloat16* sbase_h = reinterpret_cast<const __nv_bfloat16*>(it.s_hi);
    const __nv_bfloat16* sbase_l = LO ? reinterpret_cast<const __nv_bfloat16*>(it.s_lo) : nullptr;
    for (int k0 = threadIdx.x; k0 < total; k0 += ROT_VEC * blockDim.x) {
      uint4 rh[ROT_VEC], sh[ROT_VEC], rl[ROT_VEC], sl[ROT_VEC];
      long long ro[ROT_VEC], so[ROT_VEC];
#pragma unroll
      for (int u = 0; u < ROT_VEC; ++u) {
        const int k = k0 + u * blockDim.x;
        const int rloc = div_small(k, nvec, inv_nvec);
        const long long row = r0 + rloc, col = (long long)(k - rloc * nvec) * 8;
        ro[u] = row * it.ldr + col;
        so[u] = row * it.lds + col;
        if (k < total) {
          rh[u] = *reinterpret_cast<const uint4*>(rbase_h + ro[u]);
          sh[u] = *reinterpret_cast<const uint4*>(sbase_h + so[u]);
          if (LO && rbase_l) rl[u] = *reinterpret_cast<const uint4*>(rbase_l + ro[u]);
          if (LO && sbase_l) sl[u] = *reinterpret_cast<const uint4*>(sbase_l + so[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < ROT_VEC; ++u) {
        if (k0 + u * blockDim.x >= total) continue;
        float rv[8], sv[8];
        unpack8(rh[u], rv);
        unpack8(sh[u], sv);
        if (LO && rbase_l) {
          float l[8];
          unpack8(rl[u], l);
#pragma unroll
          for (int i = 0; i < 8; ++i) rv[i] += l[i];
        }
        if (LO && sbase_l) {
          float l[8];
          unpack8(sl[u], l);
#pragma unroll
          for (int i = 0; i < 8; ++i) sv[i] += l[i];
        }
        __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) split_bf16(a * (rv[i] * inv_s) + half_a2 * ((sv[i] * inv_s) * inv_s), h[i], l[i]);
        *reinterpret_cast<uint4*>(rbase_h + ro[u]) = *reinterpret_cast<const uint4*>(h);
        if (LO && rbase_l) *reinterpret_cast<uint4*>(rbase_l + ro[u]) = *reinterpret_cast<const uint4*>(l);
      }
    }
  }
}

// ---- trace of S o Q ----------------------------------------------------------------------------------------------
// Work entries (item, first row of TRACE_ROWS rows). 8-element vectors of S (16-byte bf16 loads) and Q (two 16-byte
// loads), TRACE_VEC vectors per thread requested before the first use; rows whose Q vectors are not 16-byte aligned
// (n % 4 != 0) and the tail columns of n % 8 != 0 go element by element.
constexpr int TRACE_ROWS = PSGD_TRACE_ROWS;
constexpr int TRACE_VEC = 4;

// LO: the items carry lo halves of S (fp32 mode); without them that code is compiled out (fewer registers, more
// blocks per SM).
template <bool LO>
__global__ void __launch_bounds__(256, LO ? 2 : 3) trace_kernel(const PsgdTraceItem* __restrict__ items,
                                                               const uint32_t* __restrict__ work, int nwork) {
  __shared__ float red[8];
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdTraceItem& it = items[work[2 * w]];
    const int r0 = (int)work[2 * w + 1], n = it.n;
    const int rows = min(TRACE_ROWS, n - r0);
    const __nv_bfloat16* sh = reinterpret_cast<const __nv_bfloat16*>(it.s_hi);
    const __nv_bfloat16* sl = LO ? reinterpret_cast<const __nv_bfloat16*>(it.s_lo) : nullptr;
    const bool vec = (n % 4) == 0 && (reinterpret_cast<uintptr_t>(it.q) & 15) == 0 && (it.lds % 8) == 0 &&
                     (reinterpret_cast<uintptr_t>(sh) & 15) == 0 && (reinterpret_cast<uintptr_t>(sl) & 15) == 0;
    const int nv = vec ? n / 8 : 0, total = rows * nv;
    const float inv_nv = nv > 0 ? 1.f / (float)nv : 0.f;
    float acc = 0.f;
    for (int k0 = threadIdx.x; k0 < total; k0 += TRACE_VEC * blockDim.x) {
      uint4 hv[TRACE_VEC], lv[LO ? TRACE_VEC : 1];
      float4 qa[TRACE_VEC], qb[TRACE_VEC];
#pragma unroll
      for (int u = 0; u < TRACE_VEC; ++u) {
        const int k = k0 + u * blockDim.x;
        if (k < total) {
          const int rl = div_small(k, nv, inv_nv);
          const long long row = r0 + rl, col = (long long)(k - rl * nv) * 8;
          hv[u] = *reinterpret_cast<const uint4*>(sh + row * it.lds + col);
          if (LO && sl) lv[LO ? u : 0] = *reinterpret_cast<const uint4*>(sl + row * it.lds + col);
          const float4* qp = reinterpret_cast<const float4*>(it.q + row * n + col);
          qa[u] = qp[0];
          qb[u] = qp[1];
        }
      }
#pragma unroll
      for (int u = 0; u < TRACE_VEC; ++u) {
        if (k0 + u * blockDim.x >= total) continue;
        float sv[8];
        unpack8(hv[u], sv);
        if (LO && sl) {
          float l[8];
          unpack8(lv[LO ? u : 0], l);
#pragma unroll
          for (int i = 0; i < 8; ++i) sv[i] += l[i];
        }
        const float qv[8] = {qa[u].x, qa[u].y, qa[u].z, qa[u].w, qb[u].x, qb[u].y, qb[u].z, qb[u].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(sv[i], qv[i], acc);
      }
    }
    // elements not covered by whole vectors: every column of a row (vec false) or the n % 8 tail
    const int c0 = nv * 8, ntail = n - c0;
    for (int k = threadIdx.x; k < rows * ntail; k += blockDim.x) {
      const int rl = k / ntail;
      const long long row = r0 + rl, col = c0 + (k - rl * ntail);
      float sv = __bfloat162float(sh[row * it.lds + col]);
      if (LO && sl) sv += __bfloat162float(sl[row * it.lds + col]);
      acc = fmaf(sv, it.q[row * n + col], acc);
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
      it.part[r0 / TRACE_ROWS] = t;
    }
    __syncthreads();
  }
}

// ---- clip + apply ------------------------------------------------------------------------------------------------
// torch.clamp(x, -me, me) (psgd_pro.py:380): NaN stays NaN (fminf / fmaxf alone would drop it), +-Inf clamps.
__device__ __forceinline__ float clip_elem(float x, float me) { return isnan(x) ? x : fminf(fmaxf(x, -me), me); }

__global__ void __launch_bounds__(256) clip_scale_kernel(const PsgdApplyItem* __restrict__ items,
                                                        const float* __restrict__ hyper) {
  const PsgdApplyItem& it = items[blockIdx.x];
  __shared__ float red[8];
  float s = 0.f;
  for (int t = threadIdx.x; t < it.nparts; t += blockDim.x) s += it.part[t];
  const float tot = block_sum(s, red);
  if (threadIdx.x == 0) {
    const float avg = sqrtf(tot / (float)it.numel);
    // psgd_pro.py:374-376: the scale is max_avg / avg only when avg > max_avg (a NaN avg leaves it 1, as the
    // reference's comparison does; an infinite avg gives 0, and Inf * 0 = NaN then reaches the parameter)
    const float max_avg = hyper[PSGD_HY_MAX_AVG];
    *it.scale = avg > max_avg ? max_avg / avg : 1.f;
  }
}

__global__ void __launch_bounds__(256) apply_kernel(const PsgdApplyItem* __restrict__ items,
                                                   const uint32_t* __restrict__ work, int nwork,
                                                   const float* __restrict__ hyper) {
  const float lr = hyper[PSGD_HY_LR_PARAMS], me = hyper[PSGD_HY_MAX_ELEM];
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdApplyItem& it = items[work[2 * w]];
    const long long base = (long long)work[2 * w + 1] * PSGD_APPLY_CHUNK;
    const float sc = *it.scale;
    const long long end = min(base + (long long)PSGD_APPLY_CHUNK, it.numel);
    const bool vec = ((reinterpret_cast<uintptr_t>(it.pg) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(it.param) & (it.param_bf16 ? 7 : 15)) == 0);
    if (vec) {  // whole 4-element vectors (chunk bases are multiples of 4), then the tail
      const long long vend = base + ((end - base) / 4) * 4;
      for (long long k = base + 4 * threadIdx.x; k < vend; k += 4 * blockDim.x) {
        const float4 g4 = *reinterpret_cast<const float4*>(it.pg + k);
        float g[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) g[i] = clip_elem(g[i] * sc, me);
        if (it.param_bf16) {
          uint2* pp = reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(it.param) + k);
          uint2 u = *pp;
          __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&u);
#pragma unroll
          for (int i = 0; i < 4; ++i) h[i] = __float2bfloat16_rn(__bfloat162float(h[i]) - lr * g[i]);
          *pp = u;
        } else {
          float4* pp = reinterpret_cast<float4*>(reinterpret_cast<float*>(it.param) + k);
          float4 p = *pp;
          p.x -= lr * g[0]; p.y -= lr * g[1]; p.z -= lr * g[2]; p.w -= lr * g[3];
          *pp = p;
        }
      }
      for (long long k = vend + threadIdx.x; k < end; k += blockDim.x) {
        const float g = clip_elem(it.pg[k] * sc, me);
        if (it.param_bf16) {
          __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(it.param);
          p[k] = __float2bfloat16_rn(__bfloat162float(p[k]) - lr * g);
        } else {
          float* p = reinterpret_cast<float*>(it.param);
          p[k] = p[k] - lr * g;
        }
      }
      continue;
    }
    for (long long k = base + threadIdx.x; k < end; k += blockDim.x) {
      const float g = clip_elem(it.pg[k] * sc, me);
      if (it.param_bf16) {
        __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(it.param);
        p[k] = __float2bfloat16_rn(__bfloat162float(p[k]) - lr * g);
      } else {
        float* p = reinterpret_cast<float*>(it.param);
        p[k] = p[k] - lr * g;
      }
    }
  }
}

// ---- factor balancing (psgd_pro.py:96-105) --------------------------------------------------------------------------
// max |q| per chunk of a factor's values, then per parameter gmean / max, then one pass that rescales Q (fp32),
// rewrites Q^T (transposed, bf16 hi/lo) and P = Q^T Q (times c^2), or q and p = q^2 for a diagonal factor.
__global__ void __launch_bounds__(256) absmax_kernel(const PsgdBalanceFactor* __restrict__ fs,
                                                    const uint32_t* __restrict__ work, int nwork) {
  __shared__ float red[8];
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdBalanceFactor& f = fs[work[2 * w]];
    const long long numel = f.dense ? (long long)f.n * f.n : f.n;
    const long long base = (long long)work[2 * w + 1] * PSGD_APPLY_CHUNK;
    const long long end = min(base + (long long)PSGD_APPLY_CHUNK, numel);
    float m = 0.f;
    for (long long k = base + threadIdx.x; k < end; k += blockDim.x) m = fmaxf(m, fabsf(f.q[k]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int i = 0; i < 8; ++i) t = fmaxf(t, red[i]);
      f.part[work[2 * w + 1]] = t;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(32) balance_scale_kernel(const PsgdBalanceFactor* __restrict__ fs,
                                                          const PsgdBalanceParam* __restrict__ ps) {
  const PsgdBalanceParam& p = ps[blockIdx.x];
  if (threadIdx.x != 0) return;
  float norms[8];
  float prod = 1.f;
  const int nf = min(p.nf, 8);
  for (int k = 0; k < nf; ++k) {
    const PsgdBalanceFactor& f = fs[p.f0 + k];
    float m = 0.f;
    for (int i = 0; i < f.nparts; ++i) m = fmaxf(m, f.part[i]);
    norms[k] = m;
    prod *= m;
  }
  const float gmean = powf(prod, 1.f / (float)nf);
  for (int k = 0; k < nf; ++k) *fs[p.f0 + k].scale = gmean / norms[k];
}

__global__ void __launch_bounds__(256) balance_apply_kernel(const PsgdBalanceFactor* __restrict__ fs,
                                                           const uint32_t* __restrict__ work, int nwork) {
  __shared__ float tile[TT][TT + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const PsgdBalanceFactor& f = fs[work[2 * w]];
    const float c = *f.scale;
    if (!f.dense) {
      const long long base = (long long)work[2 * w + 1] * PSGD_APPLY_CHUNK;
      const long long end = min(base + (long long)PSGD_APPLY_CHUNK, (long long)f.n);
      for (long long k = base + threadIdx.x; k < end; k += blockDim.x) {
        const float q = f.q[k] * c;
        f.q[k] = q;
        f.pdiag[k] = q * q;
      }
      continue;
    }
    const int ti = work[2 * w + 1] >> 16, tj = work[2 * w + 1] & 0xFFFF;
    const int n = f.n, i0 = ti * TT, j0 = tj * TT;
    const float c2 = c * c;
#pragma unroll
    for (int u = 0; u < TT / TROWS; ++u) {
      const int i = i0 + ty + u * TROWS, j = j0 + tx;
      float q = 0.f;
      if (i < n && j < n) {
        q = f.q[(long long)i * n + j] * c;
        f.q[(long long)i * n + j] = q;
        const float pv = load_split(f.p_hi, f.p_lo, (long long)i * f.ldp + j) * c2;
        store_split(f.p_hi, f.p_lo, (long long)i * f.ldp + j, pv);
      }
      tile[ty + u * TROWS][tx] = q;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < TT / TROWS; ++u) {  // Q^T[j][i] = Q[i][j]
      const int jj = j0 + ty + u * TROWS, ii = i0 + tx;
      if (jj < n && ii < n) store_split(f.qt_hi, f.qt_lo, (long long)jj * f.ldqt + ii, tile[tx][ty + u * TROWS]);
    }
    __syncthreads();
  }
}

// Grid of a grid-stride kernel: every block resident at once (SMs x the blocks per SM that the kernel's registers
// and shared memory allow), so no second partial wave runs its share of the work alone at the end.
template <typename Kernel>
static int grid_for(Kernel kernel, int threads, int nwork, int smem = 0) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int cap = sms * per_sm;
  return nwork < cap ? nwork : cap;
}

static int launched() { return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH; }

// Raises the skew kernel's dynamic shared-memory limit once per device (before any graph capture that uses it).
template <bool R1>
static bool skew_smem_attr() {
  static bool done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(skew_kernel<R1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM) != cudaSuccess)
      return false;
    done[dev] = true;
  }
  return true;
}

}  // namespace psgd

using namespace psgd;

extern "C" int psgd_prep(const PsgdPrepItem* items, const uint32_t* work, int nwork, const float* hyper, int* dev_err,
                         cudaStream_t stream) {
  if (!items || !work || !hyper || nwork < 0) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  prep_kernel<false><<<grid_for(prep_kernel<false>, 256, nwork, PREP_SMEM), 256, PREP_SMEM, stream>>>(items, work,
                                                                                                       nwork, hyper);
  return launched();
}

extern "C" int psgd_prep_momentum(const PsgdPrepItem* items, const uint32_t* work, int nwork, const float* hyper,
                                  int* dev_err, cudaStream_t stream) {
  if (!items || !work || !hyper || nwork < 0) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  prep_kernel<true><<<grid_for(prep_kernel<true>, 256, nwork, PREP_SMEM), 256, PREP_SMEM, stream>>>(items, work,
                                                                                                     nwork, hyper);
  return launched();
}

extern "C" int psgd_nlb_prep(const PsgdNlbPrepItem* items, int nitems, int* dev_err, cudaStream_t stream) {
  if (!items || nitems < 0) return PSGD_EINVAL;
  if (nitems == 0) return PSGD_OK;
  nlb_prep_kernel<<<nitems, NLB_THREADS, 0, stream>>>(items);
  return launched();
}

extern "C" int psgd_factor_update(const PsgdFactorItem* items, int nitems, const float* hyper, int* dev_err,
                                  cudaStream_t stream) {
  if (!items || !hyper || nitems < 0 || !dev_err) return PSGD_EINVAL;
  if (nitems == 0) return PSGD_OK;
  factor_kernel<<<nitems * FAC_SPLIT, FAC_THREADS, 0, stream>>>(items, hyper, dev_err);
  factor_diag_kernel<<<nitems * FAC_SPLIT, FAC_THREADS, 0, stream>>>(items, hyper, dev_err);
  return launched();
}

extern "C" int psgd_skew(const PsgdSkewItem* items, const uint32_t* work, int nwork, int* dev_err,
                         cudaStream_t stream) {
  if (!items || !work || nwork < 0) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  static std::atomic<bool> attr_done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PSGD_ELAUNCH;
  if (!attr_done[dev].load()) {  // the dynamic shared-memory limit, once per device (before any graph capture)
    if (cudaFuncSetAttribute(skew2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SK2_SMEM) != cudaSuccess)
      return PSGD_ELAUNCH;
    attr_done[dev].store(true);
  }
  skew2_kernel<<<grid_for(skew2_kernel, 256, nwork, SK2_SMEM), 256, SK2_SMEM, stream>>>(items, work, nwork);
  return launched();
}

extern "C" int psgd_skew_rank1(const PsgdSkewItem* items, const uint32_t* work, int nwork, int* dev_err,
                               cudaStream_t stream) {
  if (!items || !work || nwork < 0) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  if (!skew_smem_attr<true>()) return PSGD_ELAUNCH;
  skew_kernel<true><<<grid_for(skew_kernel<true>, 256, nwork, SK_SMEM), 256, SK_SMEM, stream>>>(items, work, nwork);
  return launched();
}

extern "C" int psgd_rot(const PsgdRotItem* items, const uint32_t* work, int nwork, int has_lo, int* dev_err,
                        cudaStream_t stream) {
  if (!items || !work || nwork < 0) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  if (has_lo) rot_kernel<true><<<grid_for(rot_kernel<true>, 256, nwork), 256, 0, stream>>>(items, work, nwork);
  else rot_kernel<false><<<grid_for(rot_kernel<false>, 256, nwork), 256, 0, stream>>>(items, work, nwork);
  return launched();
}

extern "C" int psgd_trace(const PsgdTraceItem* items, const uint32_t* work, int nwork, int has_lo, int* dev_err,
                          cudaStream_t stream) {
  if (!items || !work || nwork < 0) return PSGD_EINVAL;
  if (nwork == 0) return PSGD_OK;
  if (has_lo) trace_kernel<true><<<grid_for(trace_kernel<true>, 256, nwork), 256, 0, stream>>>(items, work, nwork);
  else trace_kernel<false><<<grid_for(trace_kernel<false>, 256, nwork), 256, 0, stream>>>(items, work, nwork);
  return launched();
}

extern "C" int psgd_apply(const PsgdApplyItem* items, int nitems, const uint32_t* work, int nwork,
                          const float* hyper, int* dev_err, cudaStream_t stream) {
  if (!items || !work || !hyper || nitems < 0 || nwork < 0) return PSGD_EINVAL;
  if (nitems == 0) return PSGD_OK;
  clip_scale_kernel<<<nitems, 256, 0, stream>>>(items, hyper);
  int rc = launched();
  if (rc) return rc;
  if (nwork == 0) return PSGD_OK;
  apply_kernel<<<grid_for(apply_kernel, 256, nwork), 256, 0, stream>>>(items, work, nwork, hyper);
  return launched();
}

extern "C" int psgd_balance(const PsgdBalanceFactor* factors, const PsgdBalanceParam* params, int nparams,
                            const uint32_t* work_max, int nwork_max, const uint32_t* work_apply, int nwork_apply,
                            int* dev_err, cudaStream_t stream) {
  if (!factors || !params || nparams < 0 || nwork_max < 0 || nwork_apply < 0) return PSGD_EINVAL;
  if (nparams == 0) return PSGD_OK;
  if (nwork_max) absmax_kernel<<<grid_for(absmax_kernel, 256, nwork_max), 256, 0, stream>>>(factors, work_max, nwork_max);
  int rc = launched();
  if (rc) return rc;
  balance_scale_kernel<<<nparams, 32, 0, stream>>>(factors, params);
  if ((rc = launched())) return rc;
  if (nwork_apply) balance_apply_kernel<<<grid_for(balance_apply_kernel, 256, nwork_apply), 256, 0, stream>>>(factors, work_apply, nwork_apply);
  return launched();
}
