// gemv.cu -- batch-1 Q4_K / Q6_K dequantise-matvec for sm_100a.
//
// Reference semantics: op_matmul_q4_k / op_matmul_q6_k (engine/src/ops.c:266-314,
// 361-404): y[r] = sum_k dequant(W[r, k]) * x[k] over 256-element super-blocks
// laid out row-major as in GGUF.  Summation order differs (parallel partial sums);
// results agree with the reference to fp32 rounding.
//
// Kernel shape (one CTA per SM, persistent over a byte-balanced row range):
//  * warp 8 is the producer: one lane streams whole-row chunks of the weight
//    matrix into a 4-stage shared-memory ring with cp.async.bulk (TMA, 1-D,
//    no tensor map, no multicast), completion tracked by mbarrier tx-counts;
//  * warps 0-7 are consumers: while the first chunks are in flight they build
//    the input vector in shared memory (optionally RMS-normalised), then decode
//    blocks from the ring.
//
// Dequant arithmetic ("denormal nibble" trick): a quant field is isolated in
// place with one AND, leaving the integer q at bit p of an otherwise-zero word,
// i.e. the fp32 denormal q * 2^(p-149).  The input element was stored
// pre-multiplied by 2^(69-p), so one FFMA gives q * x * 2^-80 exactly rounded,
// with no int->float conversion per weight.  Two weights go per __ffma2_rn.
// Per sub-block the partial sum is rescaled by d*sc*2^80 and the min / -32
// offsets are applied through precomputed sums of x.  Constraint: |x| < 2^58.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"

namespace shk {
namespace {

constexpr int XEXP = 69;
constexpr float BACK = 0x1p80f;  // 2^80

// Bit position at which the Q4_K weight for element e lands after masking
// (see q4k_block): low-nibble half {0,8,16,12}, high-nibble half {4,12,8,16}.
__device__ __forceinline__ int q4_pos(uint32_t e) {
  const uint32_t tab = ((e & 63u) < 32u) ? 0x0C100800u : 0x10080C04u;
  return (int)((tab >> (8u * (e & 3u))) & 0xFFu);
}
// Q6_K: byte k of the combined word at 8k, byte 3 at 16 (after >> 8).
__device__ __forceinline__ int q6_pos(uint32_t e) {
  const uint32_t k = e & 3u;
  return k == 3u ? 16 : (int)(8u * k);
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------- Q4_K ---------------------------------------
// One lane handles 64-element group j (32 quant bytes) of a block: the low
// nibbles are sub-block 2j, the high nibbles sub-block 2j+1.
template <bool DUAL>
__device__ __forceinline__ void q4k_block(const uint8_t* __restrict__ blk_a,
                                          const uint8_t* __restrict__ blk_b, int j,
                                          const float* __restrict__ xb, float2 xsum,
                                          float& acc_a, float& acc_b) {
  const uint4 ha = *reinterpret_cast<const uint4*>(blk_a);
  const uint4 qa0 = *reinterpret_cast<const uint4*>(blk_a + 16 + 32 * j);
  const uint4 qa1 = *reinterpret_cast<const uint4*>(blk_a + 32 + 32 * j);
  uint4 hb = ha, qb0 = qa0, qb1 = qa1;
  if (DUAL) {
    hb = *reinterpret_cast<const uint4*>(blk_b);
    qb0 = *reinterpret_cast<const uint4*>(blk_b + 16 + 32 * j);
    qb1 = *reinterpret_cast<const uint4*>(blk_b + 32 + 32 * j);
  }
  const uint32_t wa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
  const uint32_t wb[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
  float2 alo = make_float2(0.f, 0.f), ahi = alo, blo = alo, bhi = alo;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 xl = *reinterpret_cast<const float4*>(xb + 4 * i);
    const float4 xh = *reinterpret_cast<const float4*>(xb + 32 + 4 * i);
    {
      const uint32_t w = wa[i], w12 = w >> 12;
      alo = ffma2(make_float2(u2f_bits(w & 0xFu), u2f_bits(w & 0xF00u)), make_float2(xl.x, xl.y), alo);
      alo = ffma2(make_float2(u2f_bits(w & 0xF0000u), u2f_bits(w12 & 0xF000u)), make_float2(xl.z, xl.w), alo);
      ahi = ffma2(make_float2(u2f_bits(w & 0xF0u), u2f_bits(w & 0xF000u)), make_float2(xh.x, xh.y), ahi);
      ahi = ffma2(make_float2(u2f_bits(w12 & 0xF00u), u2f_bits(w12 & 0xF0000u)), make_float2(xh.z, xh.w), ahi);
    }
    if (DUAL) {
      const uint32_t w = wb[i], w12 = w >> 12;
      blo = ffma2(make_float2(u2f_bits(w & 0xFu), u2f_bits(w & 0xF00u)), make_float2(xl.x, xl.y), blo);
      blo = ffma2(make_float2(u2f_bits(w & 0xF0000u), u2f_bits(w12 & 0xF000u)), make_float2(xl.z, xl.w), blo);
      bhi = ffma2(make_float2(u2f_bits(w & 0xF0u), u2f_bits(w & 0xF000u)), make_float2(xh.x, xh.y), bhi);
      bhi = ffma2(make_float2(u2f_bits(w12 & 0xF00u), u2f_bits(w12 & 0xF0000u)), make_float2(xh.z, xh.w), bhi);
    }
  }
  // Scales/mins of sub-blocks 2j and 2j+1 (engine/src/ops.c:107-115 get_scale_min_k4).
  const int sh = (j & 1) * 16;
  auto apply = [&](const uint4& h, float2 lo, float2 hi, float& acc) {
    uint32_t scw, mw;
    if (j < 2) {
      scw = h.y & 0x3F3F3F3Fu;
      mw = h.z & 0x3F3F3F3Fu;
    } else {
      scw = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
      mw = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    }
    const float d = ref_half(h.x & 0xFFFFu) * BACK;
    const float dmin = ref_half(h.x >> 16);
    const float sc0 = (float)((scw >> sh) & 0xFFu), sc1 = (float)((scw >> (sh + 8)) & 0xFFu);
    const float m0 = (float)((mw >> sh) & 0xFFu), m1 = (float)((mw >> (sh + 8)) & 0xFFu);
    acc = fmaf(d * sc0, lo.x + lo.y, acc);
    acc = fmaf(d * sc1, hi.x + hi.y, acc);
    acc = fmaf(-(dmin * m0), xsum.x, acc);
    acc = fmaf(-(dmin * m1), xsum.y, acc);
  };
  apply(ha, alo, ahi, acc_a);
  if (DUAL) apply(hb, blo, bhi, acc_b);
}

template <int RG, bool DUAL>
__device__ __forceinline__ void q4k_task(const uint8_t* __restrict__ rows, uint32_t row_stride,
                                         uint32_t nb, int rows_valid, uint32_t dual_off,
                                         const float* __restrict__ x4,
                                         const float* __restrict__ xs32, int lane, float& acc_a,
                                         float& acc_b) {
  constexpr int SPR = 8 / RG;  // block slots per row
  const int slot = lane >> 2, j = lane & 3;
  const int r = slot / SPR, s = slot % SPR;
  acc_a = 0.f;
  acc_b = 0.f;
  if (r < rows_valid) {
    const uint8_t* row = rows + (size_t)r * row_stride;
    for (uint32_t b = s; b < nb; b += SPR) {
      const float2 xsum = *reinterpret_cast<const float2*>(xs32 + b * 8 + 2 * j);
      q4k_block<DUAL>(row + b * Q4K_BYTES, row + dual_off + b * Q4K_BYTES, j,
                      x4 + b * QK + 64 * j, xsum, acc_a, acc_b);
    }
  }
#pragma unroll
  for (int o = 16 / RG; o > 0; o >>= 1) {
    acc_a += __shfl_xor_sync(0xffffffffu, acc_a, o);
    if (DUAL) acc_b += __shfl_xor_sync(0xffffffffu, acc_b, o);
  }
}

// ------------------------------- Q6_K ---------------------------------------
// Blocks are 210 bytes, so a block's offset inside a 16-byte-aligned row is
// 2*b mod 16.  Lanes of a warp always work on blocks b == C (mod 4), which
// share the alignment MU = 2*C mod 8 of every field; MU is a template constant.
template <int MU>
__device__ __forceinline__ void load32(const uint8_t* p, uint32_t o[8]) {
  if (MU == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint2 v = *reinterpret_cast<const uint2*>(p + 8 * i);
      o[2 * i] = v.x;
      o[2 * i + 1] = v.y;
    }
  } else if (MU == 4) {
    o[0] = *reinterpret_cast<const uint32_t*>(p);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint2 v = *reinterpret_cast<const uint2*>(p + 4 + 8 * i);
      o[1 + 2 * i] = v.x;
      o[2 + 2 * i] = v.y;
    }
    o[7] = *reinterpret_cast<const uint32_t*>(p + 28);
  } else if (MU == 2) {
    const uint32_t a = *reinterpret_cast<const uint16_t*>(p);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p + 2);
    const uint2 d0 = *reinterpret_cast<const uint2*>(p + 6);
    const uint2 d1 = *reinterpret_cast<const uint2*>(p + 14);
    const uint2 d2 = *reinterpret_cast<const uint2*>(p + 22);
    const uint32_t z = *reinterpret_cast<const uint16_t*>(p + 30);
    o[0] = __byte_perm(a, w, 0x5410);
    o[1] = __byte_perm(w, d0.x, 0x5432);
    o[2] = __byte_perm(d0.x, d0.y, 0x5432);
    o[3] = __byte_perm(d0.y, d1.x, 0x5432);
    o[4] = __byte_perm(d1.x, d1.y, 0x5432);
    o[5] = __byte_perm(d1.y, d2.x, 0x5432);
    o[6] = __byte_perm(d2.x, d2.y, 0x5432);
    o[7] = __byte_perm(d2.y, z, 0x5432);
  } else {  // MU == 6
    const uint32_t a = *reinterpret_cast<const uint16_t*>(p);
    const uint2 d0 = *reinterpret_cast<const uint2*>(p + 2);
    const uint2 d1 = *reinterpret_cast<const uint2*>(p + 10);
    const uint2 d2 = *reinterpret_cast<const uint2*>(p + 18);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p + 26);
    const uint32_t z = *reinterpret_cast<const uint16_t*>(p + 30);
    o[0] = __byte_perm(a, d0.x, 0x5410);
    o[1] = __byte_perm(d0.x, d0.y, 0x5432);
    o[2] = __byte_perm(d0.y, d1.x, 0x5432);
    o[3] = __byte_perm(d1.x, d1.y, 0x5432);
    o[4] = __byte_perm(d1.y, d2.x, 0x5432);
    o[5] = __byte_perm(d2.x, d2.y, 0x5432);
    o[6] = __byte_perm(d2.y, w, 0x5432);
    o[7] = __byte_perm(w, z, 0x5432);
  }
}

template <int MU>
__device__ __forceinline__ void load8(const uint8_t* p, uint32_t o[2]) {
  if (MU == 0) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    o[0] = v.x;
    o[1] = v.y;
  } else if (MU == 4) {
    o[0] = *reinterpret_cast<const uint32_t*>(p);
    o[1] = *reinterpret_cast<const uint32_t*>(p + 4);
  } else {  // 2 or 6: p+2 is 4-byte aligned
    const uint32_t a = *reinterpret_cast<const uint16_t*>(p);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p + 2);
    const uint32_t z = *reinterpret_cast<const uint16_t*>(p + 6);
    o[0] = __byte_perm(a, w, 0x5410);
    o[1] = __byte_perm(w, z, 0x5432);
  }
}

// One lane handles half n (128 elements) of a Q6_K block
// (engine/src/ops.c:167-193 dequantize_row_q6_k).
template <int MU>
__device__ __forceinline__ void q6k_block(const uint8_t* __restrict__ blk, int n,
                                          const float* __restrict__ xh,
                                          const float* __restrict__ xm, float& acc) {
  uint32_t A[8], B[8], H[8], S[2];
  load32<MU>(blk + 64 * n, A);
  load32<MU>(blk + 64 * n + 32, B);
  load32<MU>(blk + 128 + 32 * n, H);
  load8<MU>(blk + 192 + 8 * n, S);
  const uint32_t dbits = *reinterpret_cast<const uint16_t*>(blk + 208);
  const uint32_t M = 0x0F0F0F0Fu;
  float2 a[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) a[t] = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int is = i >> 2;
    const uint32_t h = H[i];
    // combined 6-bit quants, bits 6-7 of each byte are don't-care
    const uint32_t Q[4] = {lop_sel(A[i], h << 4, M), lop_sel(B[i], h << 2, M),
                           lop_sel(A[i] >> 4, h, M), lop_sel(B[i] >> 4, h >> 2, M)};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float4 xv = *reinterpret_cast<const float4*>(xh + 32 * g + 4 * i);
      const uint32_t q = Q[g], q8 = q >> 8;
      float2& ac = a[2 * g + is];
      ac = ffma2(make_float2(u2f_bits(q & 0x3Fu), u2f_bits(q & 0x3F00u)), make_float2(xv.x, xv.y), ac);
      ac = ffma2(make_float2(u2f_bits(q & 0x3F0000u), u2f_bits(q8 & 0x3F0000u)), make_float2(xv.z, xv.w), ac);
    }
  }
  const float d = ref_half(dbits);
  const float4 m0 = *reinterpret_cast<const float4*>(xm);
  const float4 m1 = *reinterpret_cast<const float4*>(xm + 4);
  const float mm[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
#pragma unroll
    for (int is = 0; is < 2; ++is) {
      const int si = is + 2 * g;  // scale index within this half
      const int sc = (int)(int8_t)((S[si >> 2] >> (8 * (si & 3))) & 0xFFu);
      const float t = fmaf(a[2 * g + is].x + a[2 * g + is].y, BACK, mm[si]);
      acc = fmaf(d * (float)sc, t, acc);
    }
  }
}

template <int C>
__device__ __forceinline__ void q6k_class(const uint8_t* __restrict__ row, uint32_t nb, int s,
                                          int spr, int n, const float* __restrict__ x6,
                                          const float* __restrict__ xm16, float& acc) {
  if (nb <= (uint32_t)C) return;
  const uint32_t nbc = (nb - C + 3) / 4;
  for (uint32_t t = s; t < nbc; t += spr) {
    const uint32_t b = C + 4 * t;
    q6k_block<(2 * C) & 7>(row + (size_t)b * Q6K_BYTES, n, x6 + b * QK + 128 * n,
                           xm16 + b * 16 + 8 * n, acc);
  }
}

template <int RG, bool DUAL>
__device__ __forceinline__ void q6k_task(const uint8_t* __restrict__ rows, uint32_t row_stride,
                                         uint32_t nb, int rows_valid, uint32_t dual_off,
                                         const float* __restrict__ x6,
                                         const float* __restrict__ xm16, int lane, float& acc_a,
                                         float& acc_b) {
  constexpr int SPR = 16 / RG;
  const int slot = lane >> 1, n = lane & 1;
  const int r = slot / SPR, s = slot % SPR;
  acc_a = 0.f;
  acc_b = 0.f;
  if (r < rows_valid) {
    const uint8_t* row = rows + (size_t)r * row_stride;
    q6k_class<0>(row, nb, s, SPR, n, x6, xm16, acc_a);
    q6k_class<1>(row, nb, s, SPR, n, x6, xm16, acc_a);
    q6k_class<2>(row, nb, s, SPR, n, x6, xm16, acc_a);
    q6k_class<3>(row, nb, s, SPR, n, x6, xm16, acc_a);
    if (DUAL) {
      const uint8_t* row2 = row + dual_off;
      q6k_class<0>(row2, nb, s, SPR, n, x6, xm16, acc_b);
      q6k_class<1>(row2, nb, s, SPR, n, x6, xm16, acc_b);
      q6k_class<2>(row2, nb, s, SPR, n, x6, xm16, acc_b);
      q6k_class<3>(row2, nb, s, SPR, n, x6, xm16, acc_b);
    }
  }
#pragma unroll
  for (int o = 16 / RG; o > 0; o >>= 1) {
    acc_a += __shfl_xor_sync(0xffffffffu, acc_a, o);
    if (DUAL) acc_b += __shfl_xor_sync(0xffffffffu, acc_b, o);
  }
}

// ------------------------------ chunk walk ----------------------------------
struct Range {
  uint32_t ub, ue;
};
__device__ __forceinline__ Range seg_units(const GemvArgs& a, int s, uint64_t seg_off, uint64_t lo,
                                           uint64_t hi) {
  const GemvSeg& g = a.seg[s];
  const uint64_t units = (g.m + g.rg - 1) / g.rg;
  auto first_at_or_after = [&](uint64_t c) -> uint64_t {
    if (c <= seg_off) return 0;
    const uint64_t u = (c - seg_off + g.unit_cost - 1) / g.unit_cost;
    return u < units ? u : units;
  };
  return Range{(uint32_t)first_at_or_after(lo), (uint32_t)first_at_or_after(hi)};
}

template <int RG>
__device__ __forceinline__ void run_task(const GemvArgs& a, const GemvSeg& g, const uint8_t* rows,
                                         int rows_valid, uint32_t dual_off, const float* x4,
                                         const float* x6, const float* xs32, const float* xm16,
                                         int lane, float& acc_a, float& acc_b) {
  if (g.qt == T_Q4K) {
    if (RG <= 8) {
      constexpr int R = RG <= 8 ? RG : 8;
      if (g.dual)
        q4k_task<R, true>(rows, g.row_stride, g.nb, rows_valid, dual_off, x4, xs32, lane, acc_a, acc_b);
      else
        q4k_task<R, false>(rows, g.row_stride, g.nb, rows_valid, dual_off, x4, xs32, lane, acc_a, acc_b);
    }
  } else {
    if (g.dual)
      q6k_task<RG, true>(rows, g.row_stride, g.nb, rows_valid, dual_off, x6, xm16, lane, acc_a, acc_b);
    else
      q6k_task<RG, false>(rows, g.row_stride, g.nb, rows_valid, dual_off, x6, xm16, lane, acc_a, acc_b);
  }
}

template <int RG>
__device__ __forceinline__ void task_and_store(const GemvArgs& a, const GemvSeg& g,
                                               const uint8_t* rows, uint32_t row0, int rows_valid,
                                               uint32_t dual_off, const float* x4, const float* x6,
                                               const float* xs32, const float* xm16, int lane) {
  float acc_a, acc_b;
  run_task<RG>(a, g, rows, rows_valid, dual_off, x4, x6, xs32, xm16, lane, acc_a, acc_b);
  constexpr int LPR = 32 / RG;  // lanes per row
  const int r = lane / LPR;
  if (g.epi == EPI_ROPE) {
    const float partner = __shfl_down_sync(0xffffffffu, acc_a, LPR);
    if ((lane % LPR) == 0 && (r & 1) == 0 && r + 1 < rows_valid) {
      const uint32_t row = row0 + r;
      const uint32_t i = row % g.rope_hd;
      const float inv_theta = 1.0f / a.rope_theta;
      const float freq = powf(inv_theta, (float)i / (float)g.rope_hd);
      const float ang = (float)(*a.pos) * freq;
      const float c = cosf(ang), s = sinf(ang);
      g.y[row] = acc_a * c - partner * s;
      g.y[row + 1] = acc_a * s + partner * c;
    }
    return;
  }
  if ((lane % LPR) == 0 && r < rows_valid) {
    const uint32_t row = row0 + r;
    if (g.epi == EPI_STORE) {
      g.y[row] = acc_a;
    } else if (g.epi == EPI_ADD) {
      g.y[row] = g.y[row] + acc_a;
    } else {  // EPI_SWIGLU
      const float gt = acc_a;
      const float sig = 1.0f / (1.0f + expf(-gt));
      g.y[row] = (gt * sig) * acc_b;
    }
  }
}

template <bool HAS4, bool HAS6>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + GEMV_STAGES;
  float* red = reinterpret_cast<float*>(smem + 64);
  float* xbase = red + 32;
  const uint32_t K = a.k;
  float* x4 = xbase;
  float* x6 = x4 + (HAS4 ? K : 0);
  float* xs32 = x6 + (HAS6 ? K : 0);
  float* xm16 = xs32 + (HAS4 ? K / 32 : 0);
  size_t stage_off = (size_t)(reinterpret_cast<uint8_t*>(xm16 + (HAS6 ? K / 16 : 0)) - smem);
  stage_off = (stage_off + 127) & ~(size_t)127;
  uint8_t* stages = smem + stage_off;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < GEMV_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GEMV_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const uint64_t lo = a.total_cost * blockIdx.x / gridDim.x;
  const uint64_t hi = a.total_cost * (blockIdx.x + 1) / gridDim.x;

  if (warp == GEMV_WARPS) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      uint64_t seg_off = 0;
      for (uint32_t s = 0; s < a.nseg && ok; ++s) {
        const GemvSeg& g = a.seg[s];
        const Range rr = seg_units(a, s, seg_off, lo, hi);
        const uint32_t cu = g.chunk_rows / g.rg;
        for (uint32_t u = rr.ub; u < rr.ue && ok; u += cu) {
          const uint32_t r0 = u * g.rg;
          const uint32_t r1 = min(min(u + cu, rr.ue) * g.rg, g.m);
          const uint32_t bytes = (r1 - r0) * g.row_stride;
          const int st = it % GEMV_STAGES;
          if (it >= GEMV_STAGES &&
              !mbar_wait_bounded(&empty[st], ((it / GEMV_STAGES) - 1) & 1, a.err, DERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* dst = stages + (size_t)st * a.stage_bytes;
          mbar_arrive_expect_tx(&full[st], g.dual ? 2 * bytes : bytes);
          bulk_g2s(dst, g.w + (size_t)r0 * g.row_stride, bytes, &full[st]);
          if (g.dual) bulk_g2s(dst + bytes, g.w2 + (size_t)r0 * g.row_stride, bytes, &full[st]);
          ++it;
        }
        seg_off += (uint64_t)((g.m + g.rg - 1) / g.rg) * g.unit_cost;
      }
      // Do not leave the CTA with copies in flight: wait (bounded) for the
      // last issued stages to land.
      const uint32_t n_tail = it < (uint32_t)GEMV_STAGES ? it : (uint32_t)GEMV_STAGES;
      for (uint32_t t = it - n_tail; t < it; ++t)
        mbar_wait_bounded(&full[t % GEMV_STAGES], (t / GEMV_STAGES) & 1, a.err, DERR_TIMEOUT_FULL);
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int ctid = threadIdx.x;  // 0 .. 32*GEMV_WARPS-1
  constexpr int CT = 32 * GEMV_WARPS;
  float inv_rms = 1.0f;
  if (a.norm_w) {
    // RMSNorm prologue (engine/src/ops.c:195-214), fixed-order reduction so
    // every CTA derives the identical scale.
    float ss = 0.f;
    for (uint32_t i = ctid; i < K; i += CT) {
      const float v = a.x[i];
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    named_sync(1, CT);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < GEMV_WARPS; ++w) tot += red[w];
    inv_rms = 1.0f / sqrtf(tot / (float)K + 1e-5f);
  }
  // Build scaled input copies and per-group sums; warp w takes 32-element
  // groups w, w+8, ...
  for (uint32_t g32 = warp; g32 < K / 32; g32 += GEMV_WARPS) {
    const uint32_t i = g32 * 32 + lane;
    float v = a.x[i];
    if (a.norm_w) v = (v * inv_rms) * a.norm_w[i];
    if (HAS4) {
      x4[i] = ldexpf(v, XEXP - q4_pos(i));
      const float s = warp_sum(v);
      if (lane == 0) xs32[g32] = s;
    }
    if (HAS6) {
      x6[i] = ldexpf(v, XEXP - q6_pos(i));
      float s = v;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if ((lane & 15) == 0) xm16[2 * g32 + (lane >> 4)] = -32.0f * s;
    }
  }
  named_sync(1, CT);

  uint32_t it = 0, gtask = 0;
  uint64_t seg_off = 0;
  for (uint32_t s = 0; s < a.nseg; ++s) {
    const GemvSeg& g = a.seg[s];
    const Range rr = seg_units(a, s, seg_off, lo, hi);
    const uint32_t cu = g.chunk_rows / g.rg;
    for (uint32_t u = rr.ub; u < rr.ue; u += cu) {
      const uint32_t r0 = u * g.rg;
      const uint32_t r1 = min(min(u + cu, rr.ue) * g.rg, g.m);
      const uint32_t nrows = r1 - r0;
      const int st = it % GEMV_STAGES;
      if (!mbar_wait_bounded(&full[st], (it / GEMV_STAGES) & 1, a.err, DERR_TIMEOUT_FULL)) return;
      const uint8_t* buf = stages + (size_t)st * a.stage_bytes;
      const uint32_t ntasks = (nrows + g.rg - 1) / g.rg;
      const uint32_t dual_off = nrows * g.row_stride;
      uint32_t t = (uint32_t)((warp - (int)(gtask % GEMV_WARPS) + GEMV_WARPS) % GEMV_WARPS);
      for (; t < ntasks; t += GEMV_WARPS) {
        const int rv = (int)min((uint32_t)g.rg, nrows - t * g.rg);
        const uint8_t* rows = buf + (size_t)t * g.rg * g.row_stride;
        const uint32_t row0 = r0 + t * g.rg;
        switch (g.rg) {
          case 1: task_and_store<1>(a, g, rows, row0, rv, dual_off, x4, x6, xs32, xm16, lane); break;
          case 2: task_and_store<2>(a, g, rows, row0, rv, dual_off, x4, x6, xs32, xm16, lane); break;
          case 4: task_and_store<4>(a, g, rows, row0, rv, dual_off, x4, x6, xs32, xm16, lane); break;
          case 8: task_and_store<8>(a, g, rows, row0, rv, dual_off, x4, x6, xs32, xm16, lane); break;
          default: task_and_store<16>(a, g, rows, row0, rv, dual_off, x4, x6, xs32, xm16, lane); break;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      gtask += ntasks;
      ++it;
    }
    seg_off += (uint64_t)((g.m + g.rg - 1) / g.rg) * g.unit_cost;
  }
}

// --------------------------- generic fallback ---------------------------------
// One warp per row; plain byte loads; used only when rows are not 16-byte
// multiples (e.g. a raw Q6_K tensor whose row has an odd number of 8-block
// groups).  Same per-element dequantisation as the reference.
__global__ void gemv_generic_kernel(uint32_t qt, const uint8_t* __restrict__ w,
                                    const float* __restrict__ x, float* __restrict__ y,
                                    uint32_t m, uint32_t k) {
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const uint32_t nb = k / QK;
  float acc = 0.f;
  if (qt == T_Q4K) {
    const uint8_t* rp = w + (size_t)row * nb * Q4K_BYTES;
    for (uint32_t b = 0; b < nb; ++b) {
      const uint8_t* blk = rp + (size_t)b * Q4K_BYTES;
      const float d = ref_half(blk[0] | (blk[1] << 8)), dmin = ref_half(blk[2] | (blk[3] << 8));
      const uint8_t* sc = blk + 4;
      for (int e = lane; e < QK; e += 32) {
        const int g = e / 64, l = e % 64, sub = 2 * g + (l >= 32);
        const uint8_t qb = blk[16 + 32 * g + (l & 31)];
        const int q = (l >= 32) ? (qb >> 4) : (qb & 0xF);
        int s, mn;
        if (sub < 4) {
          s = sc[sub] & 63;
          mn = sc[sub + 4] & 63;
        } else {
          s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
          mn = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
        }
        acc = fmaf((d * s) * q - dmin * mn, x[b * QK + e], acc);
      }
    }
  } else {
    const uint8_t* rp = w + (size_t)row * nb * Q6K_BYTES;
    for (uint32_t b = 0; b < nb; ++b) {
      const uint8_t* blk = rp + (size_t)b * Q6K_BYTES;
      const float d = ref_half(blk[208] | (blk[209] << 8));
      for (int e = lane; e < QK; e += 32) {
        const int n = e / 128, r = e % 128, grp = r / 32, l = r % 32;
        const uint8_t* ql = blk + 64 * n;
        const uint8_t h = blk[128 + 32 * n + l];
        const uint8_t lq = (grp & 1) ? ql[l + 32] : ql[l];
        const int lo = (grp >= 2) ? (lq >> 4) : (lq & 0xF);
        const int q = (lo | (((h >> (2 * grp)) & 3) << 4)) - 32;
        const int s = (int8_t)blk[192 + 8 * n + l / 16 + 2 * grp];
        acc = fmaf((d * (float)s) * (float)q, x[b * QK + e], acc);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

}  // namespace

int gemv_plan(GemvPlan& p, const GemvMat* mats, int nmats, uint32_t k, const float* x,
              const float* norm_w, const uint32_t* pos, float rope_theta, int* err, int num_sms) {
  if (nmats < 1 || nmats > GEMV_MAX_SEGS || k == 0 || k % QK) return -1;
  GemvArgs& a = p.args;
  a = GemvArgs{};
  a.nseg = nmats;
  a.k = k;
  a.x = x;
  a.norm_w = norm_w;
  a.pos = pos;
  a.rope_theta = rope_theta;
  a.err = err;
  p.has4 = p.has6 = 0;
  const uint32_t nb = k / QK;
  const uint32_t target = 32768;
  uint32_t stage = 0;
  uint64_t total = 0, units_total = 0;
  for (int i = 0; i < nmats; ++i) {
    const GemvMat& mt = mats[i];
    GemvSeg& g = a.seg[i];
    if (mt.qt != T_Q4K && mt.qt != T_Q6K) return -2;
    const uint32_t bb = mt.qt == T_Q4K ? Q4K_BYTES : Q6K_BYTES;
    g.w = static_cast<const uint8_t*>(mt.w);
    g.w2 = static_cast<const uint8_t*>(mt.w2);
    g.y = mt.y;
    g.m = mt.m;
    g.nb = nb;
    g.row_stride = mt.row_stride ? mt.row_stride : nb * bb;
    if (g.row_stride % 16 || g.row_stride < nb * bb) return -3;
    if ((reinterpret_cast<uintptr_t>(g.w) & 15) || (g.w2 && (reinterpret_cast<uintptr_t>(g.w2) & 15)))
      return -3;
    g.qt = (uint8_t)mt.qt;
    g.epi = mt.epi;
    g.dual = mt.w2 ? 1 : 0;
    if (g.dual != (mt.epi == EPI_SWIGLU)) return -1;
    g.rope_hd = mt.rope_hd;
    if (mt.epi == EPI_ROPE && (mt.rope_hd == 0 || (mt.rope_hd & 1) || !pos)) return -1;
    uint32_t rg = 1;
    if (mt.qt == T_Q4K) {
      p.has4 = 1;
      while (rg * 2 <= 8 && rg * 2 * nb <= 8) rg *= 2;
    } else {
      p.has6 = 1;
      const uint32_t nbc = (nb + 3) / 4;
      while (rg * 2 <= 16 && rg * 2 * nbc <= 16) rg *= 2;
    }
    if (mt.epi == EPI_ROPE && rg < 2) rg = 2;
    g.rg = (uint8_t)rg;
    g.unit_cost = rg * g.row_stride * (g.dual ? 2 : 1);
    const uint32_t cu = std::max<uint32_t>(1, target / g.unit_cost);
    g.chunk_rows = cu * rg;
    stage = std::max<uint32_t>(stage, cu * g.unit_cost);
    const uint64_t units = (mt.m + rg - 1) / rg;
    total += units * g.unit_cost;
    units_total += units;
  }
  a.stage_bytes = (stage + 127) & ~127u;
  a.total_cost = total;
  size_t xbytes = 64 + 32 * 4;
  if (p.has4) xbytes += (size_t)k * 4 + (k / 32) * 4;
  if (p.has6) xbytes += (size_t)k * 4 + (k / 16) * 4;
  xbytes = (xbytes + 127) & ~(size_t)127;
  p.smem = xbytes + (size_t)GEMV_STAGES * a.stage_bytes;
  if (p.smem > 227 * 1024) return -4;
  p.grid = (int)std::min<uint64_t>((uint64_t)num_sms, units_total);
  if (p.grid < 1) p.grid = 1;
  return 0;
}

cudaError_t gemv_init() {
  const int mx = 227 * 1024;
  cudaError_t e = cudaFuncSetAttribute(gemv_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  return e;
}

cudaError_t gemv_launch(const GemvPlan& p, cudaStream_t stream) {
  if (p.args.total_cost == 0) return cudaSuccess;
  if (p.has4 && p.has6)
    gemv_kernel<true, true><<<p.grid, GEMV_THREADS, p.smem, stream>>>(p.args);
  else if (p.has4)
    gemv_kernel<true, false><<<p.grid, GEMV_THREADS, p.smem, stream>>>(p.args);
  else
    gemv_kernel<false, true><<<p.grid, GEMV_THREADS, p.smem, stream>>>(p.args);
  return cudaGetLastError();
}

cudaError_t gemv_generic_launch(uint32_t qt, const void* w, const float* x, float* y, uint32_t m,
                                uint32_t k, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  const int rows_per_block = 8;
  gemv_generic_kernel<<<(m + rows_per_block - 1) / rows_per_block, 32 * rows_per_block, 0, stream>>>(
      qt, static_cast<const uint8_t*>(w), x, y, m, k);
  return cudaGetLastError();
}

}  // namespace shk
