// glue_dev.cuh -- device side of the embedding lookup and the first-index
// argmax, shared by the stand-alone kernels (glue.cu) and the persistent
// decode kernel (decode.cu).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"

namespace shk {
namespace gldev {

// Element e of the embedding row of token `tok`: op_embed, Q4_K and F16
// branches (engine/src/ops.c:533-577), same per-element formula as the
// reference, y = (d * sc) * q - dmin * m, rounded step by step.
__device__ __forceinline__ float embed_elem(const uint8_t* __restrict__ table, uint32_t dtype,
                                            uint32_t tok, uint32_t n_embd, uint32_t e) {
  if (dtype == 1) return ref_half(reinterpret_cast<const uint16_t*>(table)[(size_t)tok * n_embd + e]);
  const uint32_t nb = n_embd / QK;
  const uint8_t* blk = table + ((size_t)tok * nb + e / QK) * Q4K_BYTES;
  const uint32_t l = e % QK, grp = l / 64, w = l % 64, sub = 2 * grp + (w >= 32);
  const float d = ref_half(blk[0] | (blk[1] << 8)), dmin = ref_half(blk[2] | (blk[3] << 8));
  const uint8_t* sc = blk + 4;
  uint32_t s, m;
  if (sub < 4) {
    s = sc[sub] & 63;
    m = sc[sub + 4] & 63;
  } else {
    s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
    m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
  }
  const uint8_t qb = blk[16 + 32 * grp + (w & 31)];
  const uint32_t q = (w >= 32) ? (qb >> 4) : (qb & 0xF);
  const float d1 = d * (float)s, m1 = dmin * (float)m;
  return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

// (v2, i2) beats (v1, i1): larger value, or equal value at a lower index
// (engine/src/engine.c:424-431 keeps the first maximum with a strict >).
// Index 0xFFFFFFFF marks "no element".
__device__ __forceinline__ bool am_better(float v1, uint32_t i1, float v2, uint32_t i2) {
  if (i2 == 0xFFFFFFFFu) return false;
  if (i1 == 0xFFFFFFFFu) return true;
  return v2 > v1 || (v2 == v1 && i2 < i1);
}

// Best (value, index) of x[lo, hi) over NT threads (thread ids 0..NT-1);
// the result is valid in thread 0.  sv/si: NT/32 entries of shared memory.
// sync() synchronises the NT threads.
template <int NT, typename Sync>
__device__ __forceinline__ void am_block(const float* __restrict__ x, uint32_t lo, uint32_t hi,
                                         float* sv, uint32_t* si, Sync sync, float& bv_out,
                                         uint32_t& bi_out) {
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  // 64-bit index: with hi close to 2^32 a 32-bit i + NT would wrap below hi
  for (uint64_t i = (uint64_t)lo + threadIdx.x; i < hi; i += NT) {
    const float v = __ldcg(x + i);  // may have been written earlier in the same launch
    // NaN never wins (the reference's `x[i] > x[best]` is false for it; a NaN
    // at index 0 is handled by the merge); i increases: strict > keeps the first
    if (!isnan(v) && (bi == 0xFFFFFFFFu || v > bv)) {
      bv = v;
      bi = (uint32_t)i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(bv, bi, ov, oi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  sync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < NT / 32; ++w)
      if (am_better(bv, bi, sv[w], si[w])) {
        bv = sv[w];
        bi = si[w];
      }
  }
  bv_out = bv;
  bi_out = bi;
}

// Parallel merge of n per-block partials by the NT threads of the last block
// (sync() synchronises them; sv/si: NT/32 entries); the result is valid in
// thread 0.  (value, index) pairs with no NaN values order totally (larger
// value, then lower index), so the tree gives the sequential answer.  The
// reference's loop (best = 0; x[i] > x[best]) returns 0 when x[0] is NaN --
// x0_nan -- and when every value is NaN.
template <int NT, typename Sync>
__device__ __forceinline__ uint32_t am_merge_par(const float* part_v, const uint32_t* part_i, uint32_t n,
                                                 bool x0_nan, float* sv, uint32_t* si, Sync sync,
                                                 float* v_out = nullptr) {
  float v = -INFINITY;
  uint32_t ix = 0xFFFFFFFFu;
  for (uint32_t b = threadIdx.x; b < n; b += NT) {
    const float ov = __ldcg(&part_v[b]);
    const uint32_t oi = __ldcg(&part_i[b]);
    if (am_better(v, ix, ov, oi)) {
      v = ov;
      ix = oi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
    if (am_better(v, ix, ov, oi)) {
      v = ov;
      ix = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = ix;
  }
  sync();
  if (threadIdx.x == 0)
    for (int w = 1; w < NT / 32; ++w)
      if (am_better(v, ix, sv[w], si[w])) {
        v = sv[w];
        ix = si[w];
      }
  if (x0_nan) {
    v = __int_as_float(0x7fc00000);
    ix = 0;
  }
  if (v_out) *v_out = v;
  return (ix == 0xFFFFFFFFu) ? 0u : ix;
}

}  // namespace gldev
}  // namespace shk
