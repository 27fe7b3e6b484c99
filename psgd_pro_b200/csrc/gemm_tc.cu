// Persistent, warp-specialised tcgen05 GEMM for sm_100a with fused epilogues (the dense contractions of the
// PSGD-Kron step: Gram products Q^T Q, term1 = Pg Pg^T, the preconditioner applications P1 G P2, the Q update
// term1 q, the Procrustes products, and the skinny subspace products V A of the norm lower bounds).
//
// CTA layout (192 threads, one CTA per SM):
//   warp 0        TMA producer: 128x64 A tile and bn x 64 B tile (plus their lo copies in split mode) per stage,
//                 128-byte swizzled, into a STAGES-deep ring of shared-memory buffers.
//   warp 1        MMA issuer: one thread issues tcgen05.mma (M = 128, N = bn, K = 16 per instruction) into one
//                 of two TMEM accumulators; tcgen05.commit releases stages and hands finished accumulators over.
//   warps 2..5    epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)...), the fused
//                 element-wise transform, stores, and deterministic per-tile reductions.
// Two accumulators let the epilogue of tile i overlap the MMAs of tile i+1. Every wait is bounded in time.
#include "common.cuh"
#include "psgd_b200.h"

#include <float.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <atomic>
#include <queue>
#include <type_traits>
#include <vector>

namespace psgd {

constexpr int BM = 128, BK = 64;
constexpr int GEMM_THREADS = 192;

struct __align__(64) GemmDesc {
  CUtensorMap ta[2];  // A hi, lo
  CUtensorMap tb[2];  // B hi, lo
  CUtensorMap tt;     // the transposed bf16 output (out_hi_t; the mirror half of out_hi in SYRK mode), 32 x 32 boxes
  PsgdGemmSpec s;
  int tiles_m, tiles_n;
  int fast;    // EPI_* kind of the fast epilogue for interior tiles (0: generic only)
  int tstore;  // the fast epilogue writes the transposed bf16 output through tt (TMA stores of 32 x 32 blocks)
};

// Transposed-output blocks of the TMA-store path: one 32 x 32 bf16 block (2 KB, 64-byte rows with the 64-byte
// swizzle) per epilogue warp, after the staging blocks. Only one-MMA (bf16) kernels have them.
constexpr int TBLK_BYTES = 32 * 32 * 2;
constexpr int tblk_offset(int bytes_before) { return (bytes_before + 1023) & ~1023; }

template <int SPLIT, int BNMAX, int STAGES>
struct GemmCfg {
  static constexpr int NOPS = SPLIT == 1 ? 1 : 2;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BNMAX * BK * 2;
  // Narrow tiles (memory-bound streams of the A panel) take KSUB consecutive 64-deep K blocks per stage, so every
  // A row is read in KSUB * 128-byte runs.
  static constexpr int KSUB = (SPLIT == 1 && BNMAX <= 64) ? 4 : 1;
  static constexpr int SUB_BYTES = NOPS * (A_BYTES + B_BYTES);
  static constexpr int STAGE_BYTES = KSUB * SUB_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BNMAX;
  static constexpr int CTRL_BYTES = 256;  // barriers, TMEM slot, abort flag
  static constexpr int RED_FLOATS = 4 * BNMAX + BNMAX + 32 + 4 * 32 * 36;  // + the staging blocks
  static constexpr int TBLK_OFF = tblk_offset(TILE_BYTES + CTRL_BYTES + RED_FLOATS * 4);
  static constexpr int SMEM_BYTES = 1024 + (SPLIT == 1 ? TBLK_OFF + 4 * TBLK_BYTES : TILE_BYTES + CTRL_BYTES +
                                                                                       RED_FLOATS * 4);
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
  static_assert(SMEM_BYTES <= 232448, "shared memory beyond the 227 KB per block");
};

// ---- epilogue ------------------------------------------------------------------------------------------------
// Each epilogue warp owns 32 accumulator rows (its TMEM lane quadrant) and walks them in 32-column chunks. A chunk
// is loaded from TMEM one row per lane, scaled by alpha and staged in a 32 x 36 shared-memory block (16-byte rows,
// float4 traffic without bank conflicts), then read back in two layouts so every global access is a 16- or
// 8-byte vector on contiguous addresses:
//   column pass (lane = 4 columns of rows rs, rs+4, ...): aux term, row / column scales, row-major stores, row and
//     column sums of squares, and for SYRK the direct (upper-triangle) stores, trace share and diagonal;
//   transposed pass (lane = 4 consecutive rows of one column): transposed stores, and for SYRK the mirrored
//     stores and the mirrored trace share.
constexpr int STG = 36;  // staging pitch in floats

PSGD_DEVI float4 ld4(const float* p, int n, bool vec) {
  if (vec) return *reinterpret_cast<const float4*>(p);
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (n > 0) r.x = p[0];
  if (n > 1) r.y = p[1];
  if (n > 2) r.z = p[2];
  if (n > 3) r.w = p[3];
  return r;
}

// Tails use fully unrolled, predicated loops: a runtime index into x would force the value arrays into local
// memory for the whole hot loop.
PSGD_DEVI void st4f(float* p, const float* x, int n, bool vec) {
  if (vec) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < n) p[i] = x[i];
  }
}

// Row-major packed upper triangle of an n x n matrix: (r, c >= r) at r n - r (r - 1) / 2 + c - r.
PSGD_DEVI long long packed_off(long long r, long long c, long long n) { return r * n - (r * (r - 1)) / 2 + (c - r); }

PSGD_DEVI uint32_t pack_bf16x2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}

// Four values as bf16 hi (and lo) at hi[0..3] / lo[0..3]; one 8-byte store each when vec.
PSGD_DEVI void st4b(__nv_bfloat16* hi, __nv_bfloat16* lo, const float* x, int n, bool vec) {
  __nv_bfloat16 h0, h1, h2, h3, l0, l1, l2, l3;
  split_bf16(x[0], h0, l0);
  split_bf16(x[1], h1, l1);
  split_bf16(x[2], h2, l2);
  split_bf16(x[3], h3, l3);
  if (vec) {
    *reinterpret_cast<uint2*>(hi) = make_uint2(pack_bf16x2(h0, h1), pack_bf16x2(h2, h3));
    if (lo) *reinterpret_cast<uint2*>(lo) = make_uint2(pack_bf16x2(l0, l1), pack_bf16x2(l2, l3));
  } else {
    if (n > 0) hi[0] = h0;
    if (n > 1) hi[1] = h1;
    if (n > 2) hi[2] = h2;
    if (n > 3) hi[3] = h3;
    if (lo) {
      if (n > 0) lo[0] = l0;
      if (n > 1) lo[1] = l1;
      if (n > 2) lo[2] = l2;
      if (n > 3) lo[3] = l3;
    }
  }
}

// PACKED: the packed-triangle store is compiled in (only the kernels that can meet a problem with out_packed: the
// general and packed-SYRK kinds; encoding keeps such problems out of groups of other kinds, whose register budget
// it would otherwise take).
template <int BNMAX, bool PACKED>
__device__ __forceinline__ void epilogue_tile(const GemmDesc& d, int tm, int tn, uint32_t tacc, int q, int lane, float* red,
                              float* cs, float* misc, float* stage) {
  // Every descriptor field the loops use is copied into a register first: the staging stores go through
  // pointers the compiler cannot separate from the descriptor, so reading d.s.* inside the loops would reload
  // each field from memory on every iteration.
  const PsgdGemmSpec& sd = d.s;
  const long long s_M = sd.M, s_N = sd.N;
  const float* __restrict__ s_aux = sd.aux;
  const long long s_ld_aux = sd.ld_aux;
  const float* __restrict__ s_row_scale = sd.row_scale;
  const float* __restrict__ s_col_scale = sd.col_scale;
  float* __restrict__ s_out_f32 = sd.out_f32;
  const long long s_ld_f32 = sd.ld_f32;
  void* s_out_hi = sd.out_hi;
  void* s_out_lo = sd.out_lo;
  const long long s_ld_b = sd.ld_b;
  void* s_out_hi_t = sd.out_hi_t;
  void* s_out_lo_t = sd.out_lo_t;
  const long long s_ld_bt = sd.ld_bt;
  float* __restrict__ s_part_tile = sd.part_tile;
  float* __restrict__ s_part_col = sd.part_col;
  float* __restrict__ s_part_row = sd.part_row;
  float* __restrict__ s_diag_out = sd.diag_out;
  const float* __restrict__ s_dot_aux = sd.dot_aux;
  const long long s_ld_dot = sd.ld_dot;
  float* __restrict__ s_part_dot = sd.part_dot;
  const float* __restrict__ s_cs_part = sd.cs_part;
  const int s_cs_T = sd.cs_T, s_cs_mode = sd.cs_mode, s_mode = sd.mode, s_bn = sd.bn;
  const float* s_cs_nf = sd.cs_nf;
  const float s_alpha = sd.alpha, s_beta = sd.beta;
  const float* s_alpha_ptr = sd.alpha_ptr;
  const float* s_beta_ptr = sd.beta_ptr;
  float* __restrict__ s_out_packed = sd.out_packed;
  const int d_tiles_n = d.tiles_n;

  const int bn = s_bn;
  const long long m0 = (long long)tm * BM, n0 = (long long)tn * bn;
  const long long row0 = m0 + q * 32;  // first row of this warp
  const int et = q * 32 + lane;        // 0..127 among the epilogue threads
  const bool syrk = s_mode == PSGD_GEMM_SYRK;

  const float alpha = s_alpha * (s_alpha_ptr ? __ldg(s_alpha_ptr) : 1.f);
  const float beta = s_beta * (s_beta_ptr ? __ldg(s_beta_ptr) : 1.f);
  // Column scales. For the subspace products (cs_mode) the value is (D * 1/(|W_c| + tiny)) * 1/nf: two separate
  // multiplications in the reference's order (normalise V, then multiply by A / nf), so a zero matrix (nf = tiny)
  // gives zeros instead of 0 * inf.
  const bool has_cs = s_col_scale != nullptr || s_cs_mode != 0;
  const float inv_nf = s_cs_mode ? 1.f / *s_cs_nf : 1.f;
  if (has_cs) {
    for (int c = et; c < bn; c += 128) {
      const long long gc = n0 + c;
      float v = 1.f;
      if (gc < s_N) {
        if (s_col_scale) {
          v = s_col_scale[gc];
        } else if (s_cs_mode == 2) {
          float acc = 0.f;
          for (int t = 0; t < s_cs_T; ++t) acc += s_cs_part[(long long)t * s_N + gc];
          v = 1.f / (sqrtf(acc) + FLT_MIN);
        }
      }
      cs[c] = v;
    }
  }
  named_sync(1, 128);

  const bool need_col = s_part_col != nullptr || (syrk && s_part_row != nullptr);
  const bool tpass = syrk || s_out_hi_t != nullptr;
  __nv_bfloat16* out_hi = (__nv_bfloat16*)s_out_hi;
  __nv_bfloat16* out_lo = (__nv_bfloat16*)s_out_lo;
  const bool vf32 = s_out_f32 && (s_ld_f32 % 4 == 0) && ((reinterpret_cast<uintptr_t>(s_out_f32) & 15) == 0);
  const bool vb16 = out_hi && (s_ld_b % 4 == 0) && ((reinterpret_cast<uintptr_t>(out_hi) & 7) == 0) &&
                    (!out_lo || (reinterpret_cast<uintptr_t>(out_lo) & 7) == 0);
  const bool vaux = s_aux && (s_ld_aux % 4 == 0) && ((reinterpret_cast<uintptr_t>(s_aux) & 15) == 0);
  const bool vdot = s_dot_aux && (s_ld_dot % 4 == 0) && ((reinterpret_cast<uintptr_t>(s_dot_aux) & 15) == 0);

  // column-pass lane mapping: rows rs + 4 * it (it = 0..7), columns 4 * cg .. 4 * cg + 3 of the chunk
  const int rs = lane >> 3, cg = lane & 7;
  float rowacc[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) rowacc[it] = 0.f;
  float tsum = 0.f, dsum = 0.f;

  // The column pass's second input (aux, or dot_aux in SYRK mode): a chunk's loads are all issued before use.
  const float* pre_src = syrk ? s_dot_aux : s_aux;
  const long long pre_ld = syrk ? s_ld_dot : s_ld_aux;
  const bool pre_vec = syrk ? vdot : vaux;
  auto load_pre = [&](int cc, float4* out) {
    const long long gb = n0 + cc + 4 * cg;
    const int wn = (bn - cc) >= 32 ? 32 : 16;
    const int nv = (4 * cg < wn) ? (int)max(0LL, min(4LL, (long long)s_N - gb)) : 0;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const long long gr = row0 + rs + 4 * it;
      out[it] = (gr < s_M && nv > 0) ? ld4(pre_src + gr * pre_ld + gb, nv, pre_vec && nv == 4)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  for (int c0 = 0; c0 < bn; c0 += 32) {
    float4 pv[8];
    if (pre_src) load_pre(c0, pv);
    float v[32];
    const int w = (bn - c0) >= 32 ? 32 : 16;
    if (w == 32) {
      tmem_ld32(tacc + (uint32_t)c0, v);
    } else {
      tmem_ld16(tacc + (uint32_t)c0, v);
#pragma unroll
      for (int j = 16; j < 32; ++j) v[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(stage + lane * STG + j) =
          make_float4(v[j] * alpha, v[j + 1] * alpha, v[j + 2] * alpha, v[j + 3] * alpha);
    __syncwarp();

    // ---- column pass ----
    const long long gcb = n0 + c0 + 4 * cg;
    const int ncv = (4 * cg < w) ? (int)max(0LL, min(4LL, (long long)s_N - gcb)) : 0;
    float csc[4] = {1.f, 1.f, 1.f, 1.f};
    if (has_cs)
#pragma unroll
      for (int i = 0; i < 4; ++i) csc[i] = (i < ncv) ? cs[c0 + 4 * cg + i] : 1.f;
    float csq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = rs + 4 * it;
      const long long gr = row0 + r;
      const bool rok = gr < s_M;
      const float4 sv = *reinterpret_cast<const float4*>(stage + r * STG + 4 * cg);
      float x[4] = {sv.x, sv.y, sv.z, sv.w};
      if (s_aux) {
        x[0] += beta * pv[it].x;
        x[1] += beta * pv[it].y;
        x[2] += beta * pv[it].z;
        x[3] += beta * pv[it].w;
      }
      const float rsc = (s_row_scale && rok) ? s_row_scale[gr] : 1.f;
      float rpart = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool ok = rok && i < ncv;
        float xi = x[i] * rsc;
        if (has_cs) xi = (xi * csc[i]) * inv_nf;
        xi = ok ? xi : 0.f;
        x[i] = xi;
        const float x2 = xi * xi;
        if (!syrk) {
          rpart += x2;
          csq[i] += x2;
        } else {
          const long long gc = gcb + i;
          if (gc >= gr) rpart += x2;
          if (gc > gr) csq[i] += x2;  // mirrored element (gc, gr) belongs to row gc
          if (ok && gc == gr && s_diag_out) s_diag_out[gr] = xi;
        }
      }
      tsum += rpart;
      rowacc[it] += rpart;
      if (rok && ncv > 0) {
        if (!syrk) {
          if (s_out_f32) st4f(s_out_f32 + gr * s_ld_f32 + gcb, x, ncv, vf32 && ncv == 4);
          if (out_hi) st4b(out_hi + gr * s_ld_b + gcb, out_lo ? out_lo + gr * s_ld_b + gcb : nullptr, x, ncv,
                           vb16 && ncv == 4);
        } else {
          const int first = (int)max(0LL, min(4LL, gr - gcb));  // elements i >= first have gc >= gr
          if (first < ncv) {
            const bool full = first == 0 && ncv == 4;
            if (s_out_f32) {
              if (full) {
                st4f(s_out_f32 + gr * s_ld_f32 + gcb, x, 4, vf32);
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  if (i >= first && i < ncv) s_out_f32[gr * s_ld_f32 + gcb + i] = x[i];
              }
            }
            if (out_hi) {
              if (full) {
                st4b(out_hi + gr * s_ld_b + gcb, out_lo ? out_lo + gr * s_ld_b + gcb : nullptr, x, 4, vb16);
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  if (i >= first && i < ncv) {
                    __nv_bfloat16 h, l;
                    split_bf16(x[i], h, l);
                    out_hi[gr * s_ld_b + gcb + i] = h;
                    if (out_lo) out_lo[gr * s_ld_b + gcb + i] = l;
                  }
                }
              }
            }
            if (s_dot_aux) {
              const float dd[4] = {pv[it].x, pv[it].y, pv[it].z, pv[it].w};
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (i >= first && i < ncv) dsum += x[i] * dd[i];
            }
            if (PACKED && s_out_packed) {
              const long long pb = packed_off(gr, gcb, s_N);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (i >= first && i < ncv) s_out_packed[pb + i] = x[i];
            }
          }
        }
      }
      *reinterpret_cast<float4*>(stage + r * STG + 4 * cg) = make_float4(x[0], x[1], x[2], x[3]);
    }
    if (need_col) {  // column sums over the warp's 32 rows: reduce over the 4 lanes that share cg
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float t = csq[i];
        t += __shfl_xor_sync(0xffffffffu, t, 8);
        t += __shfl_xor_sync(0xffffffffu, t, 16);
        csq[i] = t;
      }
      if (rs == 0)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[q * BNMAX + c0 + 4 * cg + i] = csq[i];
    }
    __syncwarp();

    // ---- transposed pass: lane = rows 4 rg .. 4 rg + 3 of column 4 it + cs_ ----
    if (tpass) {
      const int cs_ = lane >> 3, rg = lane & 7;
      const long long gr0 = row0 + 4 * rg;
      const int nrv = (int)max(0LL, min(4LL, (long long)s_M - gr0));
      __nv_bfloat16* ht = (__nv_bfloat16*)s_out_hi_t;
      __nv_bfloat16* lt = (__nv_bfloat16*)s_out_lo_t;
      const bool vt = ht && (s_ld_bt % 4 == 0) && ((reinterpret_cast<uintptr_t>(ht) & 7) == 0) &&
                      (!lt || (reinterpret_cast<uintptr_t>(lt) & 7) == 0);
      float4 md[8];  // mirrored trace operand dot_aux[gc][gr0 ..], all issued before use
      if (syrk && s_dot_aux) {
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int c = 4 * it + cs_;
          const long long gc = n0 + c0 + c;
          const int lim = (c < w && gc < s_N) ? (int)max(0LL, min((long long)nrv, gc - gr0)) : 0;
          md[it] = lim > 0 ? ld4(s_dot_aux + gc * s_ld_dot + gr0, lim, vdot && lim == 4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int c = 4 * it + cs_;
        const long long gc = n0 + c0 + c;
        if (c >= w || gc >= s_N || nrv == 0) continue;
        float x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = stage[(4 * rg + i) * STG + c];
        if (!syrk) {
          st4b(ht + gc * s_ld_bt + gr0, lt ? lt + gc * s_ld_bt + gr0 : nullptr, x, nrv, vt && nrv == 4);
        } else {
          // mirrors (gc, gr) of the elements with gc > gr: rows gr0 + i < gc
          const int lim = (int)max(0LL, min((long long)nrv, gc - gr0));
          if (lim > 0) {
            const bool full = lim == 4;
            if (s_out_f32) {
              st4f(s_out_f32 + gc * s_ld_f32 + gr0, x, lim, vf32 && full);
            }
            if (out_hi) st4b(out_hi + gc * s_ld_b + gr0, out_lo ? out_lo + gc * s_ld_b + gr0 : nullptr, x, lim,
                             vb16 && full);
            if (s_dot_aux) {
              const float dd[4] = {md[it].x, md[it].y, md[it].z, md[it].w};
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (i < lim) dsum += x[i] * dd[i];
            }
          }
        }
      }
    }
    __syncwarp();
  }

  // ---- reductions over the 128 epilogue threads (fixed order) ----
  // row sums: reduce over the 8 lanes that share rs (their 4-column partials)
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    float t = rowacc[it];
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 4);
    rowacc[it] = t;
  }
  if (s_part_tile || s_part_dot) {
    const float t1 = warp_sum(tsum), t2 = warp_sum(dsum);
    if (lane == 0) {
      misc[q] = t1;
      misc[4 + q] = t2;
    }
  }
  named_sync(1, 128);
  const long long tile_lin = (long long)tm * d_tiles_n + tn;
  if (et == 0) {
    if (s_part_tile) s_part_tile[tile_lin] = ((misc[0] + misc[1]) + misc[2]) + misc[3];
    if (s_part_dot) s_part_dot[tile_lin] = ((misc[4] + misc[5]) + misc[6]) + misc[7];
  }
  if (s_part_row && cg == 0) {  // direct share: slot tn
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const long long gr = row0 + rs + 4 * it;
      if (gr < s_M) s_part_row[(long long)tn * s_M + gr] = rowacc[it];
    }
  }
  if (need_col) {
    for (int c = et; c < bn; c += 128) {
      const long long gcc = n0 + c;
      if (gcc >= s_N) continue;
      const float t = ((red[c] + red[BNMAX + c]) + red[2 * BNMAX + c]) + red[3 * BNMAX + c];
      if (!syrk) {
        s_part_col[(long long)tm * s_N + gcc] = t;
      } else {  // mirrored share of row gcc: slot tiles_n + tm
        s_part_row[((long long)d_tiles_n + tm) * s_M + gcc] = t;
      }
    }
  }
  named_sync(1, 128);  // red/cs/misc are reused by the next tile
}

// ---- fast epilogue for interior tiles -------------------------------------------------------------------------------
// Interior tiles (all 128 rows and bn columns inside the matrix) of problems whose pointers and leading dimensions
// allow vector accesses take a specialised path per epilogue kind: no tail handling, one instruction stream per
// kind. The column pass is epilogue_tile's; the transposed pass keeps one accumulator row per lane (the TMEM
// layout) so each warp store writes 32 consecutive elements of a transposed row, and reads no shared memory in
// SYRK mode. SYRK tiles that meet the diagonal mask only the one 32 x 32 chunk per warp that the diagonal crosses.
// EPI_SYRKP: SYRK whose only output is the packed upper triangle (no mirror, no reductions).
enum : int { EPI_GENERIC = 0, EPI_AUX = 1, EPI_NLB = 2, EPI_PLAIN = 3, EPI_SYRK = 4, EPI_SYRKP = 5 };

// One 32 x 32 chunk of the transposed bf16 output through a TMA store: lane L packs column L of the warp's staging
// block (scaled) as row L of the warp's transposed block (64-byte rows, 16-byte groups placed by the 64-byte swizzle,
// which also keeps the warp's shared-memory writes free of bank conflicts), then one lane stores the block at
// (x, y) = (first accumulator row, first chunk column) of the map. The block is rewritten only after the previous
// store from it has finished reading it.
__device__ __forceinline__ void tstore_chunk(const CUtensorMap* tt, uint8_t* tblk, const float* stage, int lane,
                                             float scale, long long x, long long y) {
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(stage[(2 * i) * STG + lane] * scale,
                                                   stage[(2 * i + 1) * STG + lane] * scale);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  uint8_t* rowp = tblk + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    *reinterpret_cast<uint4*>(rowp + ((k ^ sw) << 4)) = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tt, tblk, (int)x, (int)y);
    bulk_commit();
  }
}

template <int KIND, int BNMAX, bool DG>
__device__ __forceinline__ void epilogue_fast(const GemmDesc& d, int tm, int tn, uint32_t tacc, int q, int lane, float* red,
                              float* cs, float* misc, float* stage, uint8_t* tblk) {
  static_assert(!DG || KIND == EPI_SYRK || KIND == EPI_SYRKP, "diagonal tiles exist in SYRK mode only");
  const PsgdGemmSpec& sd = d.s;
  const long long s_M = sd.M, s_N = sd.N;
  const int bn = sd.bn;
  const float* __restrict__ s_aux = sd.aux;
  const long long s_ld_aux = sd.ld_aux;
  const float* __restrict__ s_row_scale = sd.row_scale;
  float* __restrict__ s_out_f32 = sd.out_f32;
  const long long s_ld_f32 = sd.ld_f32;
  __nv_bfloat16* out_hi = (__nv_bfloat16*)sd.out_hi;
  __nv_bfloat16* out_lo = (__nv_bfloat16*)sd.out_lo;
  const long long s_ld_b = sd.ld_b;
  __nv_bfloat16* ht = (__nv_bfloat16*)sd.out_hi_t;
  __nv_bfloat16* lt = (__nv_bfloat16*)sd.out_lo_t;
  const long long s_ld_bt = sd.ld_bt;
  float* __restrict__ s_part_tile = sd.part_tile;
  float* __restrict__ s_part_col = sd.part_col;
  float* __restrict__ s_part_row = sd.part_row;
  // (the fast kinds never carry a dot operand: SYRK problems with one take the general epilogue, which keeps the
  // registers of the dot's loads out of the hot SYRK path; part_dot is then left as it is)
  float* __restrict__ s_part_dot = sd.part_dot;
  float* __restrict__ s_diag_out = sd.diag_out;
  float* __restrict__ s_out_packed = sd.out_packed;
  const int d_tiles_n = d.tiles_n;
  const long long m0 = (long long)tm * BM, n0 = (long long)tn * bn;
  const long long row0 = m0 + q * 32;
  const int et = q * 32 + lane;
  const float alpha = sd.alpha * (sd.alpha_ptr ? __ldg(sd.alpha_ptr) : 1.f);
  const float beta = sd.beta * (sd.beta_ptr ? __ldg(sd.beta_ptr) : 1.f);
  // the transposed bf16 output (the mirror in SYRK mode) leaves through TMA stores of the staging block
  const bool tma_t = tblk != nullptr && d.tstore;
  float inv_nf = 1.f;
  if (KIND == EPI_NLB) {  // column scales of the subspace products, in the reference's division order
    inv_nf = 1.f / *sd.cs_nf;
    for (int c = et; c < bn; c += 128) {
      float v = 1.f;
      if (sd.cs_mode == 2) {
        float acc = 0.f;
        for (int t = 0; t < sd.cs_T; ++t) acc += sd.cs_part[(long long)t * s_N + n0 + c];
        v = 1.f / (sqrtf(acc) + FLT_MIN);
      }
      cs[c] = v;
    }
  }
  named_sync(1, 128);

  const int rs = lane >> 3, cg = lane & 7;  // column pass: rows rs + 4 it, columns 4 cg .. 4 cg + 3
  const long long rr = row0 + lane;         // transposed pass: one accumulator row per lane
  float rowacc[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) rowacc[it] = 0.f;
  float tsum = 0.f, dsum = 0.f;
  // The column-pass operand (aux) of the next chunk is requested while the
  // current one is processed.
  const float* pre_src = KIND == EPI_AUX ? s_aux : nullptr;
  const long long pre_ld = s_ld_aux;
  // The transposed pass reads the transformed values back from the staging block, except in SYRK mode where they
  // are alpha times the accumulator registers themselves.
  const bool writeback = KIND != EPI_SYRK && ht != nullptr;
  // SYRK tiles on the diagonal: for this warp's 32 rows the chunks left of column row0 hold no direct or mirrored
  // element (every offset is a multiple of 32), the chunk starting at row0 is masked per element (MASK), and the
  // chunks to its right are above the diagonal.
  // (In a 256-row pair tile the second CTA's rows can lie wholly below the diagonal: c_first >= bn.)
  const int c_first = DG ? (int)min(row0 - n0, (long long)bn) : 0;
  float4 pv[8];
  if (pre_src && c_first < bn) {
#pragma unroll
    for (int it = 0; it < 8; ++it)
      pv[it] = *reinterpret_cast<const float4*>(pre_src + (row0 + rs + 4 * it) * pre_ld + n0 + c_first + 4 * cg);
  }
  if (DG && s_part_row && rs == 0) {  // the skipped chunks' column sums of squares are zero
    for (int c0 = 0; c0 < c_first; c0 += 32)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[q * BNMAX + c0 + 4 * cg + i] = 0.f;
  }

  // Each chunk parks its accumulator columns in the staging block, and everything after that reads the staging
  // block. PIPE (the aux and norm-bound kinds): the columns of chunk c + 1 are loaded from TMEM while chunk c is
  // processed, into the same registers. (For the plain and SYRK kinds the 32 registers in flight cost more in spills
  // than the hidden latency gains: term1 and the Pg products 7% slower, the aux products 2% faster.)
  constexpr bool PIPE = KIND == EPI_AUX || KIND == EPI_NLB;
  uint32_t ra[32];
  if (PIPE && c_first < bn) tmem_ld32_issue(tacc + (uint32_t)c_first, ra);
  auto chunk = [&](const int c0, auto mask_tag) {
    constexpr bool MASK = decltype(mask_tag)::value;
    if (!PIPE) tmem_ld32_issue(tacc + (uint32_t)c0, ra);
    tmem_ld32_wait(ra);
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(stage + lane * STG + j) =
          make_float4(__uint_as_float(ra[j]), __uint_as_float(ra[j + 1]), __uint_as_float(ra[j + 2]),
                      __uint_as_float(ra[j + 3]));
    __syncwarp();
    if (PIPE && c0 + 32 < bn) tmem_ld32_issue(tacc + (uint32_t)(c0 + 32), ra);
    const long long colb = n0 + c0 + 4 * cg;
    float csc[4] = {1.f, 1.f, 1.f, 1.f};
    if (KIND == EPI_NLB) {
#pragma unroll
      for (int i = 0; i < 4; ++i) csc[i] = cs[c0 + 4 * cg + i];
    }
    float csq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = rs + 4 * it;
      const long long row = row0 + r;
      const float4 sv = *reinterpret_cast<const float4*>(stage + r * STG + 4 * cg);
      float x[4] = {sv.x * alpha, sv.y * alpha, sv.z * alpha, sv.w * alpha};
      if (KIND == EPI_AUX) {
        x[0] += beta * pv[it].x;
        x[1] += beta * pv[it].y;
        x[2] += beta * pv[it].z;
        x[3] += beta * pv[it].w;
        *reinterpret_cast<float4*>(s_out_f32 + row * s_ld_f32 + colb) = make_float4(x[0], x[1], x[2], x[3]);
      } else if (KIND == EPI_NLB) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[i] = (x[i] * csc[i]) * inv_nf;
          csq[i] += x[i] * x[i];
        }
      } else if (KIND == EPI_PLAIN) {
        if (s_row_scale) {
          const float rsc = s_row_scale[row];
#pragma unroll
          for (int i = 0; i < 4; ++i) x[i] *= rsc;
        }
        float rp = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float x2 = x[i] * x[i];
          rp += x2;
          csq[i] += x2;
        }
        tsum += rp;
        rowacc[it] += rp;
        if (s_out_f32)
          *reinterpret_cast<float4*>(s_out_f32 + row * s_ld_f32 + colb) = make_float4(x[0], x[1], x[2], x[3]);
        if (out_hi) st4b(out_hi + row * s_ld_b + colb, out_lo ? out_lo + row * s_ld_b + colb : nullptr, x, 4, true);
      } else if (KIND == EPI_SYRKP) {  // packed upper triangle only: four consecutive values of row `row`
        float* pp = s_out_packed + packed_off(row, colb, s_N);  // (unaligned offsets: scalar stores)
        const int first = MASK ? (int)max(0LL, min(4LL, row - colb)) : 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i >= first) pp[i] = x[i];
      } else if (!MASK) {  // EPI_SYRK above the diagonal: every element is direct and has a mirror
        float rp = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float x2 = x[i] * x[i];
          rp += x2;
          csq[i] += x2;
        }
        tsum += rp;
        rowacc[it] += rp;
        if (s_out_f32)
          *reinterpret_cast<float4*>(s_out_f32 + row * s_ld_f32 + colb) = make_float4(x[0], x[1], x[2], x[3]);
        if (out_hi) st4b(out_hi + row * s_ld_b + colb, out_lo ? out_lo + row * s_ld_b + colb : nullptr, x, 4, true);
      } else {  // EPI_SYRK on the diagonal: element i is direct when colb + i >= row, mirrored when >
        const int first = (int)max(-1LL, min(4LL, row - colb));
        float rp = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float x2 = x[i] * x[i];
          const bool direct = i >= first;
          rp += direct ? x2 : 0.f;
          csq[i] += (i > first) ? x2 : 0.f;
          if (i == first && s_diag_out) s_diag_out[row] = x[i];
          if (direct) {
            if (s_out_f32) s_out_f32[row * s_ld_f32 + colb + i] = x[i];
            if (out_hi) {
              __nv_bfloat16 h, l;
              split_bf16(x[i], h, l);
              out_hi[row * s_ld_b + colb + i] = h;
              if (out_lo) out_lo[row * s_ld_b + colb + i] = l;
            }
          }
        }
        tsum += rp;
        rowacc[it] += rp;
      }
      if (writeback) *reinterpret_cast<float4*>(stage + r * STG + 4 * cg) = make_float4(x[0], x[1], x[2], x[3]);
    }
    if ((KIND == EPI_NLB || KIND == EPI_PLAIN) ? (s_part_col != nullptr) : (KIND == EPI_SYRK && s_part_row)) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float t = csq[i];
        t += __shfl_xor_sync(0xffffffffu, t, 8);
        t += __shfl_xor_sync(0xffffffffu, t, 16);
        csq[i] = t;
      }
      if (rs == 0)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[q * BNMAX + c0 + 4 * cg + i] = csq[i];
    }
    __syncwarp();
    if (pre_src && c0 + 32 < bn) {  // the next chunk's column-pass operand
#pragma unroll
      for (int it = 0; it < 8; ++it)
        pv[it] = *reinterpret_cast<const float4*>(pre_src + (row0 + rs + 4 * it) * pre_ld + n0 + c0 + 32 + 4 * cg);
    }
    // transposed pass: the chunk's column j goes to row n0 + c0 + j of the transposed output (for SYRK, the
    // mirror), so each warp store covers 32 consecutive rows: 64 contiguous bytes (bf16) or 128 (fp32).
    if (KIND == EPI_SYRK) {
      if (out_hi && !MASK && tma_t) {
        tstore_chunk(&d.tt, tblk, stage, lane, alpha, row0, n0 + c0);
      } else if (out_hi) {
#pragma unroll
        for (int j4 = 0; j4 < 32; j4 += 4) {  // this lane's accumulator row, four columns at a time
          const float4 t4 = *reinterpret_cast<const float4*>(stage + lane * STG + j4);
          const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const long long col = n0 + c0 + j4 + i;
            if (MASK && col <= rr) continue;  // on the diagonal only elements with col > row have a mirror
            __nv_bfloat16 h, l;
            split_bf16(alpha * tv[i], h, l);
            out_hi[col * s_ld_b + rr] = h;
            if (out_lo) out_lo[col * s_ld_b + rr] = l;
          }
        }
      }
      if (s_out_f32) {
#pragma unroll
        for (int j4 = 0; j4 < 32; j4 += 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(stage + lane * STG + j4);
          const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const long long col = n0 + c0 + j4 + i;
            if (MASK && col <= rr) continue;
            s_out_f32[col * s_ld_f32 + rr] = alpha * tv[i];
          }
        }
      }
    } else if (ht && tma_t) {
      __syncwarp();
      tstore_chunk(&d.tt, tblk, stage, lane, 1.f, row0, n0 + c0);
    } else if (ht) {
      __syncwarp();
      float y[32];
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(stage + lane * STG + j);
        y[j] = t.x;
        y[j + 1] = t.y;
        y[j + 2] = t.z;
        y[j + 3] = t.w;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        __nv_bfloat16 h, l;
        split_bf16(y[j], h, l);
        ht[(n0 + c0 + j) * s_ld_bt + rr] = h;
        if (lt) lt[(n0 + c0 + j) * s_ld_bt + rr] = l;
      }
    }
    __syncwarp();
  };

  int c0 = c_first;
  if (DG && c0 < bn) {
    chunk(c0, std::integral_constant<bool, true>());
    c0 += 32;
  }
  for (; c0 < bn; c0 += 32) chunk(c0, std::integral_constant<bool, false>());

  // ---- reductions (fixed order, as epilogue_tile) ----
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    float t = rowacc[it];
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 4);
    rowacc[it] = t;
  }
  if (s_part_tile || s_part_dot) {
    const float t1 = warp_sum(tsum), t2 = warp_sum(dsum);
    if (lane == 0) {
      misc[q] = t1;
      misc[4 + q] = t2;
    }
  }
  named_sync(1, 128);
  const long long tile_lin = (long long)tm * d_tiles_n + tn;
  if (et == 0) {
    if (s_part_tile) s_part_tile[tile_lin] = ((misc[0] + misc[1]) + misc[2]) + misc[3];
    if (s_part_dot) s_part_dot[tile_lin] = ((misc[4] + misc[5]) + misc[6]) + misc[7];
  }
  if ((KIND == EPI_PLAIN || KIND == EPI_SYRK) && s_part_row && cg == 0) {
#pragma unroll
    for (int it = 0; it < 8; ++it) s_part_row[(long long)tn * s_M + row0 + rs + 4 * it] = rowacc[it];
  }
  const bool col_out = (KIND == EPI_NLB || KIND == EPI_PLAIN) ? (s_part_col != nullptr) : (KIND == EPI_SYRK && s_part_row);
  if (col_out) {
    for (int c = et; c < bn; c += 128) {
      const float t = ((red[c] + red[BNMAX + c]) + red[2 * BNMAX + c]) + red[3 * BNMAX + c];
      if (KIND == EPI_SYRK) s_part_row[((long long)d_tiles_n + tm) * s_M + n0 + c] = t;
      else s_part_col[(long long)tm * s_N + n0 + c] = t;
    }
  }
  named_sync(1, 128);
}

// First K block a tile reduces over: 0, or in TRMM mode (A upper triangular, M == K) the block holding the tile's
// first row, m0 / kblock (the blocks before it multiply zeros). m0 < M = K, so every tile has at least one block.
PSGD_HD int first_kblock(const PsgdGemmSpec& s, long long m0, int kblock) {
  return s.mode == PSGD_GEMM_TRMM ? (int)(m0 / kblock) : 0;
}

// Grouped tile lists start with a header of uint32 values: the number of segments S (one per CTA), then S + 1
// offsets; segment b holds the tiles of CTA b, entries [off_b, off_(b+1)) of the (problem, tm << 16 | tn) pairs
// that follow the header.
PSGD_HD int tile_header_pairs(int nseg) { return (nseg + 3) / 2; }

// Tile t of a launch: from the explicit list (grouped launch) or, with no list, the t-th tile of problem 0 in
// row-major order (upper tiles only for SYRK).
PSGD_DEVI void get_tile(const GemmDesc* descs, const uint32_t* tiles, int t, int& p, int& tm, int& tn) {
  if (tiles) {
    p = (int)tiles[2 * t];
    tm = (int)(tiles[2 * t + 1] >> 16);
    tn = (int)(tiles[2 * t + 1] & 0xFFFF);
    return;
  }
  p = 0;
  const GemmDesc& d = descs[0];
  if (d.s.mode == PSGD_GEMM_SYRK) {  // row tm holds the tiles tn >= tm * BM / bn (they reach the upper triangle)
    int row = 0, rem = t;
    while (rem >= d.tiles_n - row * BM / d.s.bn) {
      rem -= d.tiles_n - row * BM / d.s.bn;
      ++row;
    }
    tm = row;
    tn = row * BM / d.s.bn + rem;
  } else {
    tm = t / d.tiles_n;
    tn = t % d.tiles_n;
  }
}

// Shared-memory descriptors of the issue loops: the 128-byte-swizzle descriptor of the stage ring's base, with a tile's
// start address reached by adding its offset (in 16-byte units) to the low word. Every offset of the ring keeps the
// start-address field below 2^14 (shared-memory addresses stay under 256 KB), so no carry leaves the field.
struct DescBase {
  uint32_t lo, hi;
  PSGD_DEVI explicit DescBase(const void* base) {
    const uint64_t d = sdesc_k_sw128(smem_u32(base));
    lo = (uint32_t)d;
    hi = (uint32_t)(d >> 32);
  }
  PSGD_DEVI uint64_t at(uint32_t byte_off) const { return ((uint64_t)hi << 32) | (lo + (byte_off >> 4)); }
};

// Position in the stage ring (stage index and the phase parity of its barriers), advanced once per K block.
template <int STAGES>
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  PSGD_DEVI void next() {
    if (++s == STAGES) {
      s = 0;
      ph ^= 1;
    }
  }
};

// The fields of its tiles the producer and the MMA issuer need, requested one tile ahead (and the tile-list entry two tiles ahead),
// so the global-memory latency of the next tile's metadata is hidden behind the current tile's MMAs instead of
// idling the tensor pipe between tiles. (The loads stay where they are written: every mbarrier wait and MMA
// between them is an asm statement with a memory clobber.)
struct TileMeta {
  long long K;
  int mode, bn, p, tm, tn;
};
struct TileAhead {
  const GemmDesc* descs;
  const uint32_t* tiles;
  int t, t_end, t_step;
  uint32_t e0, e1;  // list entry of tile t (when there is a list)
  TileMeta m;       // fields of the tile before t
  PSGD_DEVI TileAhead(const GemmDesc* d, const uint32_t* tl, int t0, int t1, int step)
      : descs(d), tiles(tl), t(t0), t_end(t1), t_step(step), e0(0), e1(0), m{0, 0, 0, 0, 0, 0} {
    if (t < t_end) {
      if (tiles) {
        e0 = tiles[2 * t];
        e1 = tiles[2 * t + 1];
      }
      m = fetch();
      advance_entry();
    }
  }
  PSGD_DEVI TileMeta fetch() const {
    int p, tm, tn;
    if (tiles) {
      p = (int)e0;
      tm = (int)(e1 >> 16);
      tn = (int)(e1 & 0xFFFF);
    } else {
      get_tile(descs, nullptr, t, p, tm, tn);
    }
    const PsgdGemmSpec& s = descs[p].s;
    return TileMeta{s.K, s.mode, s.bn, p, tm, tn};
  }
  PSGD_DEVI void advance_entry() {  // t moves to the next tile; its list entry is requested
    t += t_step;
    if (tiles && t < t_end) {
      e0 = tiles[2 * t];
      e1 = tiles[2 * t + 1];
    }
  }
  // Returns the current tile's fields and requests the next tile's (and the entry of the one after it).
  PSGD_DEVI TileMeta next() {
    const TileMeta cur = m;
    if (t < t_end) {
      m = fetch();
      advance_entry();
    }
    return cur;
  }
};

// ---- the kernel body ------------------------------------------------------------------------------------------
template <int SPLIT, int BNMAX, int STAGES, int KIND>
__device__ __forceinline__ void gemm_body(const GemmDesc* __restrict__ descs, const uint32_t* __restrict__ tiles,
                                          int ntiles, int* err, unsigned long long wait_ns) {
  using C = GemmCfg<SPLIT, BNMAX, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::TILE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + C::TILE_BYTES + C::CTRL_BYTES);
  float* cs = red + 4 * BNMAX;
  float* misc = cs + BNMAX;
  volatile int* epi_ok = reinterpret_cast<volatile int*>(misc + 16);
  float* stage_all = misc + 32;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // This CTA's tiles: a segment of the grouped tile list (per-CTA offsets in its header), or every gridDim-th tile
  // of the single problem.
  int t_begin = blockIdx.x, t_end = ntiles, t_step = gridDim.x;
  if (tiles) {
    const int nseg = (int)tiles[0];
    t_begin = blockIdx.x < nseg ? (int)tiles[1 + blockIdx.x] : 0;
    t_end = blockIdx.x < nseg ? (int)tiles[2 + blockIdx.x] : 0;
    t_step = 1;
    tiles += 2 * tile_header_pairs(nseg);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      Ring<STAGES> ring;
      uint32_t armed[STAGES];  // phases armed per stage, to drain in-flight copies on abort
#pragma unroll
      for (int s = 0; s < STAGES; ++s) armed[s] = 0;
      TileAhead ta(descs, tiles, t_begin, t_end, t_step);
      for (int t = t_begin; t < t_end && !*abort; t += t_step) {
        const TileMeta cur = ta.next();
        const GemmDesc& d = descs[cur.p];  // (only its tensor maps' addresses are taken below)
        const int tm = cur.tm, tn = cur.tn, bn = cur.bn;
        const long long K = cur.K;
        const int nk = (int)((K + BK * C::KSUB - 1) / (BK * C::KSUB));
        const int kb0 = cur.mode == PSGD_GEMM_TRMM ? (int)((long long)tm * BM / (BK * C::KSUB)) : 0;
        const uint32_t sub_bytes = C::NOPS * (C::A_BYTES + bn * BK * 2);
        for (int kb = kb0; kb < nk; ++kb, ring.next()) {
          const int s = ring.s;
          const uint32_t ph = ring.ph;
          // 64-deep blocks of this stage that hold any of K (no copy is issued past the end)
          const int nsub = (int)min((long long)C::KSUB, (K - (long long)kb * BK * C::KSUB + BK - 1) / BK);
          if (!mbar_wait_for(&empty[s], ph ^ 1, abort, wait_ns)) break;
          mbar_arrive_expect_tx(&full[s], sub_bytes * (uint32_t)nsub);
          armed[s] += 1;
          for (int j = 0; j < nsub; ++j) {
            uint8_t* sa = smem + s * C::STAGE_BYTES + j * C::SUB_BYTES;
            uint8_t* sb = sa + C::NOPS * C::A_BYTES;
            const int x = (kb * C::KSUB + j) * BK;
            tma_load_2d(sa, &d.ta[0], &full[s], x, tm * BM);
            tma_load_2d(sb, &d.tb[0], &full[s], x, tn * bn);
            if (SPLIT != 1) {
              tma_load_2d(sa + C::A_BYTES, &d.ta[1], &full[s], x, tm * BM);
              tma_load_2d(sb + C::B_BYTES, &d.tb[1], &full[s], x, tn * bn);
            }
          }
        }
      }
      if (*abort) {  // let every armed copy land before the CTA releases its shared memory
        for (int s = 0; s < STAGES; ++s) {
          if (armed[s] == 0) continue;
          volatile int never = 0;
          mbar_wait(&full[s], (armed[s] - 1) & 1, &never);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      Ring<STAGES> ring;
      const DescBase db(smem);
      uint32_t i = 0;
      bool issued = false;
      TileAhead ta(descs, tiles, t_begin, t_end, t_step);
      for (int t = t_begin; t < t_end; t += t_step, ++i) {
        const TileMeta cur = ta.next();  // this tile's fields; the next tile's are requested here
        const long long K = cur.K;
        const int nk = (int)((K + BK * C::KSUB - 1) / (BK * C::KSUB));
        const int kb0 = cur.mode == PSGD_GEMM_TRMM ? (int)((long long)cur.tm * BM / (BK * C::KSUB)) : 0;
        const int bn = cur.bn;
        const uint32_t acc = i & 1, aph = (i >> 1) & 1;
        if (!mbar_wait_for(&tempty[acc], aph ^ 1, abort, wait_ns)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + acc * BNMAX;
        const uint32_t idesc = idesc_bf16_m128(bn);
        bool ok = true;
        for (int kb = kb0; kb < nk; ++kb, ring.next()) {
          const int s = ring.s;
          if (!mbar_wait_for(&full[s], ring.ph, abort, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nsub = (int)min((long long)C::KSUB, (K - (long long)kb * BK * C::KSUB + BK - 1) / BK);
          for (int j = 0; j < nsub; ++j) {
            const uint32_t a_off = (uint32_t)(s * C::STAGE_BYTES + j * C::SUB_BYTES);
            const uint32_t b_off = a_off + C::NOPS * C::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad = db.at(a_off + kk * 32), bd = db.at(b_off + kk * 32);
              umma_bf16(dt, ad, bd, idesc, ((kb - kb0) | j | kk) != 0);
              if (SPLIT != 1) {
                umma_bf16(dt, ad, db.at(b_off + C::B_BYTES + kk * 32), idesc, 1);
                umma_bf16(dt, db.at(a_off + C::A_BYTES + kk * 32), bd, idesc, 1);
              }
            }
          }
          issued = true;
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (*abort && issued) {  // every issued MMA must finish before TMEM and shared memory are released
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;
    uint32_t i = 0;
    for (int t = t_begin; t < t_end; t += t_step, ++i) {
      int p, tm, tn;
      get_tile(descs, tiles, t, p, tm, tn);
      const GemmDesc& d = descs[p];
      const uint32_t acc = i & 1, aph = (i >> 1) & 1;
      // the four epilogue warps agree on success before any named barrier, so none can be left waiting there
      const bool ok = mbar_wait_for(&tfull[acc], aph, abort, wait_ns);
      if (lane == 0) epi_ok[q] = ok ? 1 : 0;
      named_sync(1, 128);
      const bool all_ok = epi_ok[0] && epi_ok[1] && epi_ok[2] && epi_ok[3];
      named_sync(1, 128);
      if (!all_ok) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BNMAX;
      float* stg = stage_all + q * 32 * STG;
      uint8_t* tb = SPLIT == 1 ? smem + C::TBLK_OFF + q * TBLK_BYTES : nullptr;
      const long long m0 = (long long)tm * BM, n0 = (long long)tn * d.s.bn;
      const bool interior = m0 + BM <= d.s.M && n0 + d.s.bn <= d.s.N;
      // the launch's kind (template) picks the one fast path compiled into this kernel; problems of another
      // kind, edge tiles and SYRK tiles on the diagonal take the generic epilogue
      const bool fast = KIND != EPI_GENERIC && d.fast == KIND && interior;
      if constexpr (KIND == EPI_SYRK || KIND == EPI_SYRKP) {
        if (fast && n0 >= m0 + BM) epilogue_fast<KIND, BNMAX, false>(d, tm, tn, tacc, q, lane, red, cs, misc, stg, tb);
        else if (fast) epilogue_fast<KIND, BNMAX, true>(d, tm, tn, tacc, q, lane, red, cs, misc, stg, tb);
        else epilogue_tile<BNMAX, KIND == EPI_GENERIC || KIND == EPI_SYRKP>(d, tm, tn, tacc, q, lane, red, cs, misc, stg);
      } else {
        if (fast) epilogue_fast<KIND, BNMAX, false>(d, tm, tn, tacc, q, lane, red, cs, misc, stg, tb);
        else epilogue_tile<BNMAX, KIND == EPI_GENERIC || KIND == EPI_SYRKP>(d, tm, tn, tacc, q, lane, red, cs, misc, stg);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait_all();  // this warp's TMA stores have completed before the block exits
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort) atomicOr(err, ERR_TIMEOUT_FULL);
}

template <int SPLIT, int BNMAX, int STAGES, int KIND>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_group_kernel(const GemmDesc* __restrict__ descs, const uint32_t* __restrict__ tiles, int ntiles, int* err,
                      unsigned long long wait_ns) {
  gemm_body<SPLIT, BNMAX, STAGES, KIND>(descs, tiles, ntiles, err, wait_ns);
}

// Single problem: the descriptor is a __grid_constant__ parameter and the tile list is implicit.
template <int SPLIT, int BNMAX, int STAGES, int KIND>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_single_kernel(const __grid_constant__ GemmDesc desc, const uint32_t* __restrict__ tiles, int ntiles,
                       int* err, unsigned long long wait_ns) {
  gemm_body<SPLIT, BNMAX, STAGES, KIND>(&desc, tiles, ntiles, err, wait_ns);
}

// ---- the pair kernel (tcgen05 cta_group::2) ------------------------------------------------------------------------
// A cluster of two CTAs on neighbouring SMs computes 256 x bn tiles: each CTA stages its 128 rows of A and its half
// (bn / 2 rows) of B, the leader (cluster rank 0) issues M = 256 MMAs that read both CTAs' shared memory, and each
// CTA's TMEM receives its 128 accumulator rows, which its own epilogue warps store. Per SM this halves the B
// operand's shared-memory and L2 traffic against the one-CTA kernel. Handshakes (all waits bounded):
//   full[s]  (leader)   both CTAs' TMA copies of stage s land here (cta_group::2 copies signal the leader's barrier);
//                       the leader's producer sets the expected bytes of both CTAs;
//   go[s]    (peer)     the leader's producer arrives when it has armed full[s] for the round, so the peer never
//                       issues copies the leader does not count (on abort the leader drains every armed round);
//   empty[s] (both)     the leader's MMA commit, multicast to both CTAs, frees stage s;
//   tfull[a] (both)     the leader's commit, multicast, hands accumulator a to both epilogues;
//   tempty[a] (leader)  four epilogue warps of each CTA arrive (the peer's remotely) when accumulator a is drained.
// A stage holds PAIR_KS consecutive 64-deep K blocks (sub-blocks of A_BYTES + B_BYTES each): every barrier round
// and every wait of the MMA issuer covers 4 * PAIR_KS MMAs.
constexpr int PAIR_BN = 256, PAIR_STAGES = 3, PAIR_KS = 2;
template <int BNMAX, int STAGES>
struct PairCfg {
  static constexpr int KS = PAIR_KS;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BNMAX / 2) * BK * 2;
  static constexpr int SUB_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = KS * SUB_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BNMAX;
  static constexpr int CTRL_BYTES = 512;
  static constexpr int RED_FLOATS = 4 * BNMAX + BNMAX + 32 + 4 * 32 * 36;
  static constexpr int TBLK_OFF = tblk_offset(TILE_BYTES + CTRL_BYTES + RED_FLOATS * 4);
  static constexpr int SMEM_BYTES = 1024 + TBLK_OFF + 4 * TBLK_BYTES;
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
  static_assert((3 * STAGES + 5) * 8 + 8 <= CTRL_BYTES, "barriers must fit the control block");
  static_assert(SMEM_BYTES <= 232448, "shared memory beyond the 227 KB per block");
};
constexpr int PBM = 2 * BM;  // rows of a pair tile

template <int BNMAX, int STAGES, int KIND>
__device__ __forceinline__ void gemm_pair_body(const GemmDesc* __restrict__ descs, const uint32_t* __restrict__ tiles,
                                               int* err, unsigned long long wait_ns) {
  using C = PairCfg<BNMAX, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::TILE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* go = empty + STAGES;
  uint64_t* tfull = go + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + C::TILE_BYTES + C::CTRL_BYTES);
  float* cs = red + 4 * BNMAX;
  float* misc = cs + BNMAX;
  volatile int* epi_ok = reinterpret_cast<volatile int*>(misc + 16);
  float* stage_all = misc + 32;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: leader
  // This cluster's segment of the tile list.
  const int nseg = (int)tiles[0], cl = (int)(blockIdx.x >> 1);
  const int t_begin = cl < nseg ? (int)tiles[1 + cl] : 0;
  const int t_end = cl < nseg ? (int)tiles[2 + cl] : 0;
  tiles += 2 * tile_header_pairs(nseg);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&go[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive or copy signal
  if (warp == 1) {
    __syncwarp();
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      Ring<STAGES> ring;
      uint32_t armed[STAGES];  // rounds the leader armed per stage, drained on abort
#pragma unroll
      for (int s = 0; s < STAGES; ++s) armed[s] = 0;
      TileAhead ta(descs, tiles, t_begin, t_end, 1);
      for (int t = t_begin; t < t_end && !*abort; ++t) {
        const TileMeta cur = ta.next();
        const GemmDesc& d = descs[cur.p];  // (only its tensor maps' addresses are taken below)
        const int tm = cur.tm, tn = cur.tn, bn = cur.bn;
        const long long K = cur.K;
        const int nk = (int)((K + BK * C::KS - 1) / (BK * C::KS));
        const int kb0 = cur.mode == PSGD_GEMM_TRMM ? (int)((long long)tm * PBM / (BK * C::KS)) : 0;
        const int half = bn / 2;
        const uint32_t sub_bytes = 2u * (uint32_t)(C::A_BYTES + half * BK * 2);  // both CTAs' copies
        for (int kb = kb0; kb < nk; ++kb, ring.next()) {
          const int s = ring.s;
          const uint32_t ph = ring.ph;
          // 64-deep blocks of this stage that hold any of K (no copy is issued past the end)
          const int nsub = (int)min((long long)C::KS, (K - (long long)kb * BK * C::KS + BK - 1) / BK);
          if (!mbar_wait_for(&empty[s], ph ^ 1, abort, wait_ns)) break;
          if (rank == 0) {
            mbar_arrive_expect_tx(&full[s], sub_bytes * (uint32_t)nsub);
            armed[s] += 1;
            mbar_arrive_cluster_relaxed(mapa_shared(&go[s], 1));
          } else if (!mbar_wait_for(&go[s], ph, abort, wait_ns)) {
            break;
          }
          const uint32_t fb = mapa_shared(&full[s], 0);
          for (int j = 0; j < nsub; ++j) {
            uint8_t* sa = smem + s * C::STAGE_BYTES + j * C::SUB_BYTES;
            const int x = (kb * C::KS + j) * BK;
            tma_load_2d_pair(sa, &d.ta[0], fb, x, tm * PBM + (int)rank * BM);
            tma_load_2d_pair(sa + C::A_BYTES, &d.tb[0], fb, x, tn * bn + (int)rank * half);
          }
        }
      }
      if (*abort && rank == 0) {  // every armed round (both CTAs' copies) lands before shared memory is released
        for (int s = 0; s < STAGES; ++s) {
          if (armed[s] == 0) continue;
          volatile int never = 0;
          mbar_wait(&full[s], (armed[s] - 1) & 1, &never);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader) ----------------
      Ring<STAGES> ring;
      const DescBase db(smem);
      uint32_t i = 0;
      bool issued = false;
      TileAhead ta(descs, tiles, t_begin, t_end, 1);
      for (int t = t_begin; t < t_end; ++t, ++i) {
        const TileMeta cur = ta.next();  // this tile's fields; the next tile's are requested here
        const long long K = cur.K;
        const int nk = (int)((K + BK * C::KS - 1) / (BK * C::KS));
        const int kb0 = cur.mode == PSGD_GEMM_TRMM ? (int)((long long)cur.tm * PBM / (BK * C::KS)) : 0;
        const uint32_t acc = i & 1, aph = (i >> 1) & 1;
        if (!mbar_wait_for(&tempty[acc], aph ^ 1, abort, wait_ns)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + acc * BNMAX;
        const uint32_t idesc = idesc_bf16_m256(cur.bn);
        bool ok = true;
        for (int kb = kb0; kb < nk; ++kb, ring.next()) {
          const int s = ring.s;
          if (!mbar_wait_for(&full[s], ring.ph, abort, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nsub = (int)min((long long)C::KS, (K - (long long)kb * BK * C::KS + BK - 1) / BK);
#pragma unroll
          for (int j = 0; j < C::KS; ++j) {
            if (j >= nsub) break;
            const uint32_t a_off = (uint32_t)(s * C::STAGE_BYTES + j * C::SUB_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_bf16_pair(dt, db.at(a_off + kk * 32), db.at(a_off + C::A_BYTES + kk * 32), idesc,
                             ((kb - kb0) | j | kk) != 0);
          }
          issued = true;
          umma_commit_pair(&empty[s], 3);
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 3);
      }
      if (*abort && issued) {  // every issued MMA (it reads both CTAs' shared memory) finishes first
        umma_commit_pair(drain, 1);
        volatile int never = 0;
        mbar_wait(drain, 0, &never);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;
    const uint32_t tempty_leader0 = mapa_shared(&tempty[0], 0), tempty_leader1 = mapa_shared(&tempty[1], 0);
    uint32_t i = 0;
    for (int t = t_begin; t < t_end; ++t, ++i) {
      int p, tm, tn;
      get_tile(descs, tiles, t, p, tm, tn);
      const GemmDesc& d = descs[p];
      const int tm128 = 2 * tm + (int)rank;  // this CTA's 128 rows of the pair tile
      const uint32_t acc = i & 1, aph = (i >> 1) & 1;
      const bool ok = mbar_wait_for(&tfull[acc], aph, abort, wait_ns);
      if (lane == 0) epi_ok[q] = ok ? 1 : 0;
      named_sync(1, 128);
      const bool all_ok = epi_ok[0] && epi_ok[1] && epi_ok[2] && epi_ok[3];
      named_sync(1, 128);
      if (!all_ok) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BNMAX;
      float* stg = stage_all + q * 32 * STG;
      uint8_t* tb = smem + C::TBLK_OFF + q * TBLK_BYTES;
      const long long m0 = (long long)tm128 * BM, n0 = (long long)tn * d.s.bn;
      if (m0 < d.s.M) {
        const bool interior = m0 + BM <= d.s.M && n0 + d.s.bn <= d.s.N;
        const bool fast = KIND != EPI_GENERIC && d.fast == KIND && interior;
        if constexpr (KIND == EPI_SYRK || KIND == EPI_SYRKP) {
          if (fast && n0 >= m0 + BM) epilogue_fast<KIND, BNMAX, false>(d, tm128, tn, tacc, q, lane, red, cs, misc, stg, tb);
          else if (fast) epilogue_fast<KIND, BNMAX, true>(d, tm128, tn, tacc, q, lane, red, cs, misc, stg, tb);
          else epilogue_tile<BNMAX, KIND == EPI_GENERIC || KIND == EPI_SYRKP>(d, tm128, tn, tacc, q, lane, red, cs, misc, stg);
        } else {
          if (fast) epilogue_fast<KIND, BNMAX, false>(d, tm128, tn, tacc, q, lane, red, cs, misc, stg, tb);
          else epilogue_tile<BNMAX, KIND == EPI_GENERIC || KIND == EPI_SYRKP>(d, tm128, tn, tacc, q, lane, red, cs, misc, stg);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&tempty[acc]);
        else mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's TMA stores have completed before the block exits
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA releases shared memory or TMEM while the other may still use them
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort) atomicOr(err, ERR_TIMEOUT_FULL);
}

template <int BNMAX, int STAGES, int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    gemm_pair_kernel(const GemmDesc* __restrict__ descs, const uint32_t* __restrict__ tiles, int* err,
                     unsigned long long wait_ns) {
  gemm_pair_body<BNMAX, STAGES, KIND>(descs, tiles, err, wait_ns);
}

// ---- host side --------------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;  // resolved once; the driver entry point never changes
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// bf16 row-major matrix (rows x cols, leading dimension ld) as TMA tiles of box_rows x 64, 128-byte swizzled.
static int encode_bf16(CUtensorMap* tm, const void* ptr, int rows, int cols, long long ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return PSGD_ETMAP;
  if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) || (ld % 8) || ld < cols || rows < 1 || cols < 1)
    return PSGD_EINVAL;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PSGD_OK : PSGD_ETMAP;
}

// Store map of a row-major bf16 matrix (rows x cols, leading dimension ld) in 32 x 32 boxes with the 64-byte
// swizzle (one box row is 64 bytes).
static int encode_store_bf16(CUtensorMap* tm, const void* ptr, long long rows, long long cols, long long ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return PSGD_ETMAP;
  if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) || (ld % 8) || ld < cols || rows < 1 || cols < 1)
    return PSGD_EINVAL;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PSGD_OK : PSGD_ETMAP;
}

static bool valid_bn(int bn, int split) {
  const int bnmax = split == 1 ? 256 : 128;
  return (bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256) && bn <= bnmax;
}

static int check_spec(const PsgdGemmSpec& s, int split) {
  if (split != 1 && split != 3) return PSGD_EINVAL;
  if (s.M < 1 || s.N < 1 || s.K < 1 || !valid_bn(s.bn, split)) return PSGD_EINVAL;
  if (split == 3 && (s.a_lo == nullptr || s.b_lo == nullptr)) return PSGD_EINVAL;
  if (s.mode == PSGD_GEMM_SYRK && (s.M != s.N || s.bn < 128)) return PSGD_EINVAL;
  if (s.mode == PSGD_GEMM_TRMM && s.M != s.K) return PSGD_EINVAL;
  if (s.mode != PSGD_GEMM_PLAIN && s.mode != PSGD_GEMM_SYRK && s.mode != PSGD_GEMM_TRMM) return PSGD_EINVAL;
  if (s.out_packed && s.mode != PSGD_GEMM_SYRK) return PSGD_EINVAL;
  if (s.cs_mode && (s.cs_nf == nullptr || (s.cs_mode == 2 && (s.cs_part == nullptr || s.cs_T < 1)))) return PSGD_EINVAL;
  if (s.M > 65535 * BM || s.N > 65535 * s.bn) return PSGD_EINVAL;
  return PSGD_OK;
}

static bool al(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// The fast epilogue kind a problem qualifies for: vector-aligned pointers and leading dimensions, and only the
// epilogue terms that kind implements (every other problem, and every edge tile, uses the generic epilogue).
static int fast_kind(const PsgdGemmSpec& s) {
  const bool f32_ok = !s.out_f32 || (al(s.out_f32, 16) && s.ld_f32 % 4 == 0);
  const bool b_ok = !s.out_hi || (al(s.out_hi, 8) && (!s.out_lo || al(s.out_lo, 8)) && s.ld_b % 4 == 0);
  const bool t_ok = !s.out_hi_t || (al(s.out_hi_t, 8) && (!s.out_lo_t || al(s.out_lo_t, 8)) && s.ld_bt % 4 == 0);
  const bool aux_ok = !s.aux || (al(s.aux, 16) && s.ld_aux % 4 == 0);
  const bool dot_ok = !s.dot_aux || (al(s.dot_aux, 16) && s.ld_dot % 4 == 0);
  // the fast epilogue walks whole 32-column chunks: narrower tiles (bn = 16) would run past the output
  if (s.bn % 32 != 0) return EPI_GENERIC;
  if (!(f32_ok && b_ok && t_ok && aux_ok && dot_ok) || s.col_scale) return EPI_GENERIC;
  if (s.mode == PSGD_GEMM_SYRK) {
    if (s.row_scale || s.aux || s.cs_mode || s.out_hi_t || s.dot_aux) return EPI_GENERIC;
    if (s.out_packed)  // the packed triangle alone has its own fast path; with other outputs the general one
      return (s.out_f32 || s.out_hi || s.dot_aux || s.diag_out || s.part_row || s.part_tile) ? EPI_GENERIC : EPI_SYRKP;
    return EPI_SYRK;
  }
  if (s.aux)
    return (s.out_f32 && s.out_hi_t && !s.out_hi && !s.row_scale && !s.cs_mode && !s.part_tile && !s.part_col &&
            !s.part_row && !s.dot_aux) ? EPI_AUX : EPI_GENERIC;
  if (s.cs_mode)
    return (!s.out_f32 && !s.out_hi && !s.row_scale && !s.part_tile && !s.part_row && !s.dot_aux) ? EPI_NLB
                                                                                                  : EPI_GENERIC;
  if (s.dot_aux || s.diag_out) return EPI_GENERIC;
  return EPI_PLAIN;
}

// pair: the B map's box is the half of a tile's bn rows that each CTA of a pair stages.
static int fill_desc(GemmDesc* d, const PsgdGemmSpec& s, int split, bool pair = false) {
  int rc = check_spec(s, split);
  if (rc) return rc;
  memset(d, 0, sizeof(GemmDesc));
  d->s = s;
  d->tiles_m = (s.M + BM - 1) / BM;
  d->tiles_n = (s.N + s.bn - 1) / s.bn;
  d->fast = fast_kind(s);
  if ((rc = encode_bf16(&d->ta[0], s.a_hi, s.M, s.K, s.lda, BM))) return rc;
  if ((rc = encode_bf16(&d->tb[0], s.b_hi, s.N, s.K, s.ldb, pair ? s.bn / 2 : s.bn))) return rc;
  if (split != 1) {
    if ((rc = encode_bf16(&d->ta[1], s.a_lo, s.M, s.K, s.lda, BM))) return rc;
    if ((rc = encode_bf16(&d->tb[1], s.b_lo, s.N, s.K, s.ldb, s.bn))) return rc;
  } else {
    d->ta[1] = d->ta[0];
    d->tb[1] = d->tb[0];
    // bf16 kernels store the transposed output of the fast epilogue with TMA where its alignment allows
    const void* tp = nullptr;
    long long trows = 0, tcols = 0, tld = 0;
    if ((d->fast == EPI_AUX || d->fast == EPI_PLAIN) && s.out_hi_t && !s.out_lo_t) {
      tp = s.out_hi_t, trows = s.N, tcols = s.M, tld = s.ld_bt;
    } else if (d->fast == EPI_SYRK && s.out_hi && !s.out_lo) {
      tp = s.out_hi, trows = s.N, tcols = s.N, tld = s.ld_b;
    }
    const char* env = getenv("PSGD_GEMM_TSTORE");  // "0": the per-lane stores of the transposed output instead
    const bool want = !(env && env[0] == '0');
    if (want && tp && al(tp, 16) && tld % 8 == 0 && encode_store_bf16(&d->tt, tp, trows, tcols, tld) == PSGD_OK)
      d->tstore = 1;
  }
  return PSGD_OK;
}

// Tiles of one problem, rows of height bm (BM for one CTA, PBM for a pair); SYRK: upper tiles only.
static int spec_tiles(const PsgdGemmSpec& s, int bm = BM) {
  const int tmn = (s.M + bm - 1) / bm, tnn = (s.N + s.bn - 1) / s.bn;
  if (s.mode == PSGD_GEMM_SYRK) {
    int n = 0;
    for (int tm = 0; tm < tmn; ++tm) n += tnn - tm * bm / s.bn;
    return n;
  }
  return tmn * tnn;
}

// Tile order of one problem: blocks of RASTER_W tile columns, each walked row by row, so the tiles that run at the
// same time (neighbours in this order) share a few B panels and a band of A panels that stay resident in L2.
constexpr int RASTER_W = 8;

// Width of the column blocks: RASTER_W, or PSGD_GEMM_RASTER from the environment (a positive count of tile columns;
// 0 walks whole rows), read at encoding time.
static int raster_width() {
  const char* env = getenv("PSGD_GEMM_RASTER");
  if (env && env[0]) {
    const int w = atoi(env);
    return w > 0 ? w : 1 << 30;
  }
  return RASTER_W;
}

static void append_tiles(const PsgdGemmSpec& s, uint32_t p, uint32_t* out, int& k, int bm = BM) {
  const int tmn = (s.M + bm - 1) / bm, tnn = (s.N + s.bn - 1) / s.bn;
  const bool syrk = s.mode == PSGD_GEMM_SYRK;
  const int rw = raster_width();
  for (int c0 = 0; c0 < tnn; c0 += rw)
    for (int tm = 0; tm < tmn; ++tm) {
      const int lo = syrk ? max(c0, tm * bm / s.bn) : c0;
      for (int tn = lo; tn < min(c0 + rw, tnn); ++tn) {
        out[2 * k] = p;
        out[2 * k + 1] = ((uint32_t)tm << 16) | (uint32_t)tn;
        ++k;
      }
    }
}

static int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

// Limit of the GEMM kernels' waits for work (a TMA stage, a free stage, an accumulator), passed to every launch:
// WAIT_LIMIT_NS unless psgd_set_wait_limit_ns changed it. The waits of an aborting CTA for its own copies and MMAs
// in flight keep WAIT_LIMIT_NS whatever this is, so shared memory and TMEM are never released under them.
static std::atomic<unsigned long long> g_wait_limit_ns{WAIT_LIMIT_NS};
static unsigned long long wait_limit() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

// Raises the dynamic shared-memory limit of a kernel once per device (never inside a graph capture afterwards).
static bool smem_attr_once(const void* fn, int bytes) {
  static const void* done[64][32] = {};  // per device: kernels already configured
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  for (int i = 0; i < 32; ++i)
    if (done[dev][i] == fn) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  for (int i = 0; i < 32; ++i)
    if (done[dev][i] == nullptr) {
      done[dev][i] = fn;
      break;
    }
  return true;
}

template <int SPLIT, int BNMAX, int STAGES, int KIND>
static int launch_group(const GemmDesc* descs, const uint32_t* tiles, int ntiles, int* err, cudaStream_t st) {
  using C = GemmCfg<SPLIT, BNMAX, STAGES>;
  auto k = gemm_group_kernel<SPLIT, BNMAX, STAGES, KIND>;
  if (!smem_attr_once(reinterpret_cast<const void*>(k), C::SMEM_BYTES)) return PSGD_ELAUNCH;
  const int grid = num_sms();  // one CTA per segment of the tile list
  k<<<grid, GEMM_THREADS, C::SMEM_BYTES, st>>>(descs, tiles, ntiles, err, wait_limit());
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}

template <int SPLIT, int BNMAX, int STAGES, int KIND>
static int launch_single(const GemmDesc& desc, const uint32_t* tiles, int ntiles, int* err, cudaStream_t st) {
  using C = GemmCfg<SPLIT, BNMAX, STAGES>;
  auto k = gemm_single_kernel<SPLIT, BNMAX, STAGES, KIND>;
  if (!smem_attr_once(reinterpret_cast<const void*>(k), C::SMEM_BYTES)) return PSGD_ELAUNCH;
  const int grid = ntiles < num_sms() ? ntiles : num_sms();
  k<<<grid, GEMM_THREADS, C::SMEM_BYTES, st>>>(desc, tiles, ntiles, err, wait_limit());
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}

// ---- pair kernel launch: one cluster of two CTAs per segment of the tile list ----
constexpr int KIND_PAIR = 8;     // flag in the encoded kind: the group runs on the pair kernel
constexpr int KIND_NARROW = 16;  // flag: every tile is at most 64 columns wide (one-CTA kernel, long K stages)

// Clusters a pair launch uses on the current device: as many as can be resident at once (at most SMs / 2).
static int pair_clusters() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms() / 2;
  if (cached[dev] > 0) return cached[dev];
  using C = PairCfg<PAIR_BN, PAIR_STAGES>;
  auto k = gemm_pair_kernel<PAIR_BN, PAIR_STAGES, EPI_GENERIC>;
  int n = num_sms() / 2;
  if (smem_attr_once(reinterpret_cast<const void*>(k), C::SMEM_BYTES)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * n);
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = 2;
    at.val.clusterDim.y = 1;
    at.val.clusterDim.z = 1;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, reinterpret_cast<const void*>(k), &cfg) == cudaSuccess && active > 0 &&
        active < n)
      n = active;
  }
  cached[dev] = n;
  return n;
}

template <int KIND>
static int launch_pair(const GemmDesc* descs, const uint32_t* tiles, int* err, cudaStream_t st) {
  using C = PairCfg<PAIR_BN, PAIR_STAGES>;
  auto k = gemm_pair_kernel<PAIR_BN, PAIR_STAGES, KIND>;
  if (!smem_attr_once(reinterpret_cast<const void*>(k), C::SMEM_BYTES)) return PSGD_ELAUNCH;
  k<<<2 * pair_clusters(), GEMM_THREADS, C::SMEM_BYTES, st>>>(descs, tiles, err, wait_limit());
  return cudaGetLastError() == cudaSuccess ? PSGD_OK : PSGD_ELAUNCH;
}

static int launch_pair_kind(const GemmDesc* d, const uint32_t* tiles, int kind, int* err, cudaStream_t st) {
  switch (kind) {
    case EPI_AUX: return launch_pair<EPI_AUX>(d, tiles, err, st);
    case EPI_NLB: return launch_pair<EPI_NLB>(d, tiles, err, st);
    case EPI_PLAIN: return launch_pair<EPI_PLAIN>(d, tiles, err, st);
    case EPI_SYRK: return launch_pair<EPI_SYRK>(d, tiles, err, st);
    case EPI_SYRKP: return launch_pair<EPI_SYRKP>(d, tiles, err, st);
    default: return launch_pair<EPI_GENERIC>(d, tiles, err, st);
  }
}

// A group runs on the pair kernel when every problem is one-MMA (bf16, no lo operands), its tiles are 128 or 256
// columns wide, neither CTA of a pair tile ever stages a wholly out-of-range box (rows past the last full 128-row
// half, columns past the last bn/2 half), and its reductions are long. PSGD_GEMM_PAIR=0 in the environment keeps
// every group on the one-CTA kernel; PSGD_GEMM_PAIR=1 drops the length rule.
static bool pair_eligible(const PsgdGemmSpec* specs, int nspecs) {
  const char* env = getenv("PSGD_GEMM_PAIR");
  if (env && env[0] == '0') return false;
  // Pairs pay off on long reductions (measured: up to +9% at K >= 4096, -8% at K = 1024, where the epilogue bounds
  // the tile): the group's flop-weighted K decides unless PSGD_GEMM_PAIR=1 forces pairs.
  if (!(env && env[0] == '1')) {
    double fl = 0.0, flk = 0.0;
    for (int i = 0; i < nspecs; ++i) {
      const double f = (double)specs[i].M * specs[i].N * specs[i].K;
      fl += f;
      flk += f * specs[i].K;
    }
    if (fl <= 0.0 || flk / fl < 2048.0) return false;
  }
  for (int i = 0; i < nspecs; ++i) {
    const PsgdGemmSpec& s = specs[i];
    if (s.a_lo || s.b_lo) return false;
    if (s.bn != 128 && s.bn != 256) return false;
    const int rm = s.M % PBM, rn = s.N % s.bn;
    if (rm != 0 && rm <= BM) return false;
    if (rn != 0 && rn <= s.bn / 2) return false;
  }
  return true;
}

template <int SPLIT, int BNMAX, int STAGES>
static int launch_group_kind(const GemmDesc* d, const uint32_t* tiles, int ntiles, int kind, int* err,
                             cudaStream_t st) {
  switch (kind) {
    case EPI_AUX: return launch_group<SPLIT, BNMAX, STAGES, EPI_AUX>(d, tiles, ntiles, err, st);
    case EPI_NLB: return launch_group<SPLIT, BNMAX, STAGES, EPI_NLB>(d, tiles, ntiles, err, st);
    case EPI_PLAIN: return launch_group<SPLIT, BNMAX, STAGES, EPI_PLAIN>(d, tiles, ntiles, err, st);
    case EPI_SYRK: return launch_group<SPLIT, BNMAX, STAGES, EPI_SYRK>(d, tiles, ntiles, err, st);
    case EPI_SYRKP: return launch_group<SPLIT, BNMAX, STAGES, EPI_SYRKP>(d, tiles, ntiles, err, st);
    default: return launch_group<SPLIT, BNMAX, STAGES, EPI_GENERIC>(d, tiles, ntiles, err, st);
  }
}

template <int SPLIT, int BNMAX, int STAGES>
static int launch_single_kind(const GemmDesc& d, int ntiles, int* err, cudaStream_t st) {
  switch (d.fast) {
    case EPI_AUX: return launch_single<SPLIT, BNMAX, STAGES, EPI_AUX>(d, nullptr, ntiles, err, st);
    case EPI_NLB: return launch_single<SPLIT, BNMAX, STAGES, EPI_NLB>(d, nullptr, ntiles, err, st);
    case EPI_PLAIN: return launch_single<SPLIT, BNMAX, STAGES, EPI_PLAIN>(d, nullptr, ntiles, err, st);
    case EPI_SYRK: return launch_single<SPLIT, BNMAX, STAGES, EPI_SYRK>(d, nullptr, ntiles, err, st);
    case EPI_SYRKP: return launch_single<SPLIT, BNMAX, STAGES, EPI_SYRKP>(d, nullptr, ntiles, err, st);
    default: return launch_single<SPLIT, BNMAX, STAGES, EPI_GENERIC>(d, nullptr, ntiles, err, st);
  }
}

}  // namespace psgd

using namespace psgd;

extern "C" int psgd_num_sms(void) { return num_sms(); }

extern "C" unsigned long long psgd_set_wait_limit_ns(unsigned long long ns) {
  if (ns == 0) ns = WAIT_LIMIT_NS;
  return g_wait_limit_ns.exchange(ns);
}

extern "C" size_t psgd_gemm_table_bytes(int nspecs) { return (size_t)(nspecs > 0 ? nspecs : 0) * sizeof(GemmDesc); }

extern "C" int psgd_gemm_count_tiles(const PsgdGemmSpec* specs, int nspecs) {
  if (!specs || nspecs < 0) return PSGD_EINVAL;
  long long n = tile_header_pairs(num_sms());
  for (int i = 0; i < nspecs; ++i) {
    if (specs[i].M < 1 || specs[i].N < 1 || !valid_bn(specs[i].bn, 1)) return PSGD_EINVAL;
    n += spec_tiles(specs[i]);
  }
  return n > 0x7fffffff ? PSGD_EINVAL : (int)n;
}

// Estimated cycles a tile holds its CTA: the slower of its MMAs (one 128 x 256 x 64 block step ~730 cycles at the
// tensor-core rate, three MMAs per step in split mode) and its epilogue (per 32-column chunk; the general epilogue
// is several times dearer than the specialised ones). The accumulators are double-buffered, so the two overlap.
static double tile_cost(const GemmDesc& d, int tm, int tn, int kind, int bm) {
  const PsgdGemmSpec& s = d.s;
  const double nk = (double)((s.K + BK - 1) / BK - first_kblock(s, (long long)tm * bm, BK));
  const double mma = nk * 730.0 * (s.bn / 256.0) * ((s.a_lo && s.b_lo) ? 3.0 : 1.0) + 1500.0;
  const long long m0 = (long long)tm * bm, n0 = (long long)tn * s.bn;
  const bool interior = m0 + bm <= s.M && n0 + s.bn <= s.N;
  const bool fast = kind != EPI_GENERIC && d.fast == kind && interior;
  const double epi = (s.bn / 32.0) * (fast ? 3000.0 : 12000.0);
  return mma > epi ? mma : epi;
}

extern "C" int psgd_gemm_encode(const PsgdGemmSpec* specs, int nspecs, void* host_table, size_t table_bytes,
                                uint32_t* host_tiles, int max_tiles, int* ntiles, int* kind) {
  if (!specs || nspecs < 1 || !host_table || !host_tiles || !ntiles || !kind) return PSGD_EINVAL;
  if (table_bytes < psgd_gemm_table_bytes(nspecs) || (reinterpret_cast<uintptr_t>(host_table) & 63)) return PSGD_ESPACE;
  if (nspecs > 65535) return PSGD_EINVAL;
  const int need = psgd_gemm_count_tiles(specs, nspecs);
  if (need < 0) return need;
  if (need > max_tiles) return PSGD_ESPACE;
  GemmDesc* descs = reinterpret_cast<GemmDesc*>(host_table);
  const bool pair = pair_eligible(specs, nspecs);
  const int bm = pair ? PBM : BM;
  // split is a launch-time choice; encode the lo maps whenever lo pointers are present
  for (int i = 0; i < nspecs; ++i) {
    const int split = (specs[i].a_lo && specs[i].b_lo) ? 3 : 1;
    const int rc = fill_desc(&descs[i], specs[i], split == 3 && specs[i].bn > 128 ? 1 : split, pair);
    if (rc) return rc;
  }
  // the group's epilogue kind: the fast kind covering the most tiles (its problems take the fast path)
  long long w[6] = {0, 0, 0, 0, 0, 0};
  for (int i = 0; i < nspecs; ++i) w[descs[i].fast] += spec_tiles(specs[i], bm);
  int best = EPI_GENERIC;
  for (int t = 1; t < 6; ++t)
    if (w[t] > w[best] || (best == EPI_GENERIC && w[t] > 0)) best = t;
  // problems with a packed output only run in kernels that compile the packed store in
  bool any_packed = false, all_syrkp = true;
  for (int i = 0; i < nspecs; ++i) {
    any_packed = any_packed || specs[i].out_packed != nullptr;
    all_syrkp = all_syrkp && descs[i].fast == EPI_SYRKP;
  }
  if (any_packed) best = all_syrkp ? EPI_SYRKP : EPI_GENERIC;
  // Narrow groups (the N = 32 norm-bound products, the rank-one products) are memory-bound streams of their A
  // operand: they run on a configuration for tiles up to 64 wide whose stages hold four 64-deep K blocks.
  bool narrow = !pair;
  for (int i = 0; i < nspecs && narrow; ++i) narrow = specs[i].bn <= 64 && !specs[i].a_lo && !specs[i].b_lo;
  *kind = best | (pair ? KIND_PAIR : 0) | (narrow ? KIND_NARROW : 0);

  // Tiles in their natural order (problems as given, row-major within each), each handed to the CTA with the
  // least estimated work so far: neighbouring tiles (which share operand panels in L2) run at about the same
  // time, and costly tiles (long K, the general epilogue) do not pile up on a few CTAs.
  const int nseg = pair ? pair_clusters() : num_sms();  // one segment per CTA, or per pair of CTAs
  const int hdr = tile_header_pairs(nseg);
  std::vector<uint32_t> all;
  all.reserve(2 * (size_t)(need - hdr));
  for (int i = 0; i < nspecs; ++i) {
    int k = 0;
    std::vector<uint32_t> one(2 * (size_t)spec_tiles(specs[i], bm));
    append_tiles(specs[i], (uint32_t)i, one.data(), k, bm);
    all.insert(all.end(), one.begin(), one.end());
  }
  const int nt = (int)(all.size() / 2);
  std::vector<double> load(nseg, 0.0);
  std::vector<int> owner(nt), count(nseg, 0);
  std::priority_queue<std::pair<double, int>, std::vector<std::pair<double, int>>, std::greater<std::pair<double, int>>> pq;
  for (int b = 0; b < nseg; ++b) pq.push({0.0, b});
  for (int t = 0; t < nt; ++t) {
    const auto top = pq.top();
    pq.pop();
    const int p = (int)all[2 * t], tm = (int)(all[2 * t + 1] >> 16), tn = (int)(all[2 * t + 1] & 0xFFFF);
    owner[t] = top.second;
    count[top.second] += 1;
    pq.push({top.first + tile_cost(descs[p], tm, tn, best, bm), top.second});
  }
  uint32_t* h = host_tiles;  // header: nseg, then nseg + 1 offsets
  h[0] = (uint32_t)nseg;
  h[1] = 0;
  for (int b = 0; b < nseg; ++b) h[2 + b] = h[1 + b] + (uint32_t)count[b];
  if (nseg + 2 < 2 * hdr) h[2 * hdr - 1] = 0;
  std::vector<uint32_t> pos(h + 1, h + 1 + nseg);
  uint32_t* body = host_tiles + 2 * hdr;
  for (int t = 0; t < nt; ++t) {
    const uint32_t j = pos[owner[t]]++;
    body[2 * j] = all[2 * t];
    body[2 * j + 1] = all[2 * t + 1];
  }
  *ntiles = hdr + nt;
  return PSGD_OK;
}

extern "C" int psgd_gemm_launch(const void* dev_table, const uint32_t* dev_tiles, int ntiles, int split, int kind,
                                int* dev_err, cudaStream_t stream) {
  if (!dev_table || !dev_tiles || ntiles < 0 || !dev_err || kind < 0 || (kind & 7) > EPI_SYRKP ||
      (kind & ~(7 | KIND_PAIR | KIND_NARROW)) != 0 || ((kind & KIND_PAIR) && (kind & KIND_NARROW)))
    return PSGD_EINVAL;
  if (ntiles == 0) return PSGD_OK;
  const GemmDesc* d = reinterpret_cast<const GemmDesc*>(dev_table);
  if (kind & KIND_PAIR) return split == 1 ? launch_pair_kind(d, dev_tiles, kind & 7, dev_err, stream) : PSGD_EINVAL;
  if (kind & KIND_NARROW)
    return split == 1 ? launch_group_kind<1, 64, 2>(d, dev_tiles, ntiles, kind & 7, dev_err, stream) : PSGD_EINVAL;
  if (split == 1) return launch_group_kind<1, 256, 4>(d, dev_tiles, ntiles, kind, dev_err, stream);
  if (split == 3) return launch_group_kind<3, 128, 3>(d, dev_tiles, ntiles, kind, dev_err, stream);
  return PSGD_EINVAL;
}

extern "C" int psgd_gemm(const PsgdGemmSpec* spec, int split, int* dev_err, cudaStream_t stream) {
  if (!spec || !dev_err) return PSGD_EINVAL;
  GemmDesc desc;
  int rc = fill_desc(&desc, *spec, split);
  if (rc) return rc;
  if (spec->out_packed && desc.fast != EPI_SYRKP) desc.fast = EPI_GENERIC;
  const int nt = spec_tiles(*spec);
  if (split == 1) return launch_single_kind<1, 256, 4>(desc, nt, dev_err, stream);
  return launch_single_kind<3, 128, 3>(desc, nt, dev_err, stream);
}
