// mmv_dev.cuh -- device side of the tensor-core batch-1 dequantise-matvec:
// the tile bodies (mma.sync int8), the x prologue, the item ring and the
// reduction of K slices.  Used by the stand-alone kernel (mmv.cu) and the
// persistent decode kernel.
//
// Reference semantics: op_matmul_q4_k / op_matmul_q6_k (engine/src/ops.c:266-314,
// 361-404) with dequantize_row_q4_k / dequantize_row_q6_k (:117-142, :167-193):
// y[r] = sum_k w[r][k] x[k], w = d*sc*q - dmin*m (Q4_K), d*sc*(q - 32) (Q6_K).
// Summation order differs from the reference's sequential fp32 sum; results
// agree to fp32 rounding.
//
// Arithmetic.  Each 256-element block of x is written as X_b * x_int with X_b a
// power of two from the block's maximum and |x_int| <= 2^22 (relative step
// 2^-22 of the block maximum), and x_int = l0 + 256 l1 + 65536 l2 with signed
// byte limbs l0, l1, l2 (balanced digits).  The weights' integer quants are the
// A operand (unsigned bytes) and the limbs the B operand (signed bytes) of
// mma.sync.m16n8k32.u8.s8.s32: one mma multiplies 16 weight rows by 32
// elements of x into three (Q4_K) or six (Q6_K) limb columns, exactly, in
// int32.  The per-sub-block scales are applied to those sums with IMAD (still
// exact), and each block's result is taken to fp32 with d * X_b.
//
//  * Q4_K: mma k-range = one 32-element sub-block.  Low nibbles (sub-block 2j)
//    are masked in place; high nibbles (2j+1) are masked without a shift, so
//    their sums are 16x and the low sub-blocks' sums are scaled by 16 instead
//    (the block result is divided by 16, exactly).  Limb columns 0-2; the
//    dmin * m * sum(x) term is fp32 from per-sub-block sums of x.
//  * Q6_K: mma k-range = one 32-element group (half n, quarter g4) holding two
//    16-element scale groups; columns 0-2 take the limbs of the first group's
//    elements (zero elsewhere), columns 3-5 the second's.  The accumulator
//    input C starts at -32 * (the group's limb sums), which applies the -32
//    offset, so D = sum (q - 32) * limb per (row, scale group, limb).
//
// Fragment layout (PTX mma.m16n8k32 .u8/.s8): lane = 4 g + t; A registers
// a0 (row g) and a1 (row g+8) hold mma-k 4t..4t+3, a2 / a3 mma-k 16+4t..+3;
// B registers b0 / b1 hold mma-k 4t..+3 / 16+4t..+3 of column g; D holds rows
// g, g+8 x columns 2t, 2t+1.  Here mma-k 4t+i is element 8t+i of the 32 and
// mma-k 16+4t+i element 8t+4+i, so each lane's A bytes are 8 consecutive
// quants of a row and its B bytes 8 consecutive limbs (one 8-byte load).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"
#include "mmv.cuh"

namespace shk {
namespace mdev {

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, int c0, int c1, int c2, int c3) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

// Shared-memory loads by 32-bit shared-window address (ld.shared: no generic
// address resolution).  volatile: the bytes are written by the bulk-copy
// engine, so the loads must stay after the mbarrier waits that publish them.
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

// Signed byte of w picked by a sign-extending PRMT selector (sx_sel(k)).
__host__ __device__ __forceinline__ uint32_t sx_sel(uint32_t k) {
  return k | ((8u | k) << 4) | ((8u | k) << 8) | ((8u | k) << 12);
}
__device__ __forceinline__ int sbyte_sel(uint32_t w, uint32_t sel) {
  int r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
  return r;
}
__device__ __forceinline__ int ubyte(uint32_t w, uint32_t k) { return (int)__byte_perm(w, 0u, 0x4440u | k); }

// --------------------------- x region in shared memory -----------------------
// xl: limbs, [K/32][3][32] bytes (range kr of 32 elements, limb L, element e)
// xb: X_b per 256-block (float)
// xs: Q4_K only -- fp32 sum of x over each 32-element sub-block
// xc: Q6_K only -- [K/32][8] int32, the C input of range kr's mma: columns
//     0-2 = -32 * sum of limb c over elements 0-15, 3-5 = over 16-31, 6-7 = 0
// zero: 16 bytes of zeros (B operand of lanes with no column)
struct XRegion {
  uint8_t* xl;
  float* xb;
  float* xs;
  int* xc;
  uint8_t* zero;
  // the same as shared-window addresses, for the hot loops
  uint32_t a_xl, a_xb, a_xs, a_xc, a_zero;
};

__host__ __device__ __forceinline__ size_t x_bytes(uint32_t K, bool has4, bool has6) {
  size_t b = 16 + (size_t)K / 32 * 96 + ((size_t)K / 256 * 4 + 15) / 16 * 16;
  if (has4) b += (size_t)K / 32 * 4;
  if (has6) b += (size_t)K;  // K/32 ranges x 32 bytes
  return b;
}
__device__ __forceinline__ XRegion x_region(uint8_t* base, uint32_t K, bool has4, bool has6) {
  XRegion r;
  r.zero = base;
  r.xl = base + 16;
  uint8_t* p = r.xl + (size_t)K / 32 * 96;
  r.xb = reinterpret_cast<float*>(p);
  p += ((size_t)K / 256 * 4 + 15) / 16 * 16;
  r.xs = reinterpret_cast<float*>(p);
  if (has4) p += (size_t)K / 32 * 4;
  r.xc = reinterpret_cast<int*>(p);
  r.a_xl = smem_u32(r.xl);
  r.a_xb = smem_u32(r.xb);
  r.a_xs = smem_u32(r.xs);
  r.a_xc = smem_u32(r.xc);
  r.a_zero = smem_u32(r.zero);
  return r;
}

// ------------------------------- the ring -------------------------------------
// Items (one K slice of a 16-row tile, of one or two matrices) live in slots of
// a.stage_bytes; R.chunk (a power of two, at most MMV_MAX_CHUNK) consecutive
// items of a CTA form a chunk, one ring stage: the producer fills a chunk with as few bulk copies as the items'
// contiguity allows (consecutive slices of a segment are consecutive in the
// tiled layout), all completing on the stage's `full` barrier.  Item j (local
// index) is consumed by warp j % MMV_WARPS alone, which arrives on the stage's
// `empty` barrier (chunk arrivals per use) when done.  Chunks keep the
// producer's work per byte small and leave every warp several items in
// flight.  With ns >= ceil(MMV_WARPS / chunk) + 2 stages, a warp waiting for
// item j finds the previous use of its stage filled, so the parity wait is
// unambiguous.
struct MRing {
  uint64_t* full;
  uint64_t* empty;
  uint8_t* stages;
  uint32_t ns;          // chunk stages
  uint32_t slot_bytes;  // bytes of one item slot (a dual item: two halves)
  uint32_t chunk;       // items per chunk
  uint32_t lg_chunk;    // log2(chunk)
};

// Item geometry.
struct Item {
  uint32_t s;    // segment
  uint32_t t;    // row tile
  uint32_t sl;   // K slice
  uint32_t b0;   // first block
  uint32_t nbs;  // blocks in this slice
};
__device__ __forceinline__ Item item_of(const MmvArgs& a, uint32_t i) {
  uint32_t s = 0;
  while (s + 1 < a.nseg && i >= a.seg[s + 1].item0) ++s;
  const MmvSeg& g = a.seg[s];
  const uint32_t li = i - g.item0;
  Item it;
  it.s = s;
  it.t = li / g.ks;
  it.sl = li - it.t * g.ks;
  it.b0 = it.sl * g.sw;
  it.nbs = min((uint32_t)g.sw, g.nb - it.b0);
  return it;
}
// Advance an item by n positions in global order (n smaller than any
// segment's item count is not required: whole segments are skipped).
__device__ __forceinline__ void item_skip(const MmvArgs& a, Item& it, uint32_t n) {
  uint32_t sl = it.sl + n, t = it.t, s = it.s;
  for (;;) {
    const MmvSeg& g = a.seg[s];
    if (sl < g.ks) break;
    sl -= g.ks;
    if (++t == g.ntiles) {
      t = 0;
      if (++s == a.nseg) {  // past the last item: leave `it` at the end
        s = a.nseg - 1;
        break;
      }
    }
  }
  const MmvSeg& h = a.seg[s];
  it.s = s;
  it.t = t;
  it.sl = sl;
  it.b0 = sl * h.sw;
  it.nbs = min((uint32_t)h.sw, h.nb - min(it.b0, h.nb));
}
__device__ __forceinline__ uint32_t tile_bytes(const MmvSeg& g) { return g.qt == T_Q4K ? Q4T_BYTES : Q6T_BYTES; }

// Bytes of one item of segment g (one matrix) and the item's byte offset in
// the tiled matrix: slices evenly divide a row (the planner's sw divides nb),
// so item li of a segment starts at li * sw tiles.
__device__ __forceinline__ uint32_t item_bytes(const MmvSeg& g) { return (uint32_t)g.sw * tile_bytes(g); }

// Offset (within its chunk) of global item i, whose chunk starts at item cs:
// the chunk's items are packed in order, a dual segment's up tiles after all
// of the chunk's gate tiles (dual plans have one segment).
__device__ __forceinline__ uint32_t chunk_off(const MmvArgs& a, uint32_t cs, uint32_t i) {
  uint32_t off = 0;
  for (uint32_t s = 0; s < a.nseg; ++s) {
    const MmvSeg& g = a.seg[s];
    const uint32_t lo = max(cs, g.item0), hi = min(i, g.item0 + g.items);
    if (hi > lo) off += (hi - lo) * item_bytes(g);
  }
  return off;
}

// Producer (one lane): this CTA's items [i0, i1) in chunks, one bulk copy per
// segment run of a chunk (two for a dual segment).  cpos: the ring position
// (chunks issued so far by this CTA, across plans in a persistent launch),
// advanced here.  The first a.pre_items items go out at once; the rest after
// the consumers have their x (xready, nullable).  Returns false if a bounded
// wait ran out.
__device__ __forceinline__ bool mmv_produce(const MmvArgs& a, const MRing& R, uint32_t i0, uint32_t i1,
                                            uint32_t& cpos, uint64_t* xready, uint32_t xready_parity) {
  bool xwaited = xready == nullptr;
  uint32_t st = cpos % R.ns, use = cpos / R.ns, s = 0;
  // one-segment plans (all but the QKV projection): the segment in registers
  const bool single = a.nseg == 1;
  const uint8_t* w1 = a.seg[0].w;
  const uint8_t* w21 = a.seg[0].w2;
  const uint32_t ib1 = item_bytes(a.seg[0]), it01 = a.seg[0].item0;
  const bool dual1 = a.seg[0].dual != 0;
  for (uint32_t i = i0; i < i1;) {
    if (!xwaited && i - i0 >= a.pre_items) {
      if (!mbar_wait_spin(xready, xready_parity, a.err, DERR_TIMEOUT_FULL)) return false;
      xwaited = true;
    }
    if (use > 0 && !mbar_wait_spin(&R.empty[st], (use - 1) & 1u, a.err, DERR_TIMEOUT_EMPTY)) return false;
    const uint32_t n = min(R.chunk, i1 - i);
    if (single) {  // one segment: the chunk is one contiguous run per matrix
      const uint32_t len = n * ib1;
      uint64_t* bar = &R.full[st];
      mbar_arrive_expect_tx(bar, dual1 ? 2 * len : len);
      uint8_t* dst = R.stages + (size_t)st * R.chunk * R.slot_bytes;
      const size_t off = (size_t)(i - it01) * ib1;
      bulk_g2s(dst, w1 + off, len, bar);
      if (dual1) bulk_g2s(dst + R.chunk * ib1, w21 + off, len, bar);
      i += n;
      ++cpos;
      if (++st == R.ns) {
        st = 0;
        ++use;
      }
      continue;
    }
    while (i >= a.seg[s].item0 + a.seg[s].items) ++s;
    // the chunk's bytes first: the barrier must expect them before any land
    uint32_t bytes = 0;
    for (uint32_t q = i, ss = s; q < i + n; ++ss) {
      const MmvSeg& g = a.seg[ss];
      const uint32_t cnt = min(i + n, g.item0 + g.items) - q;
      bytes += cnt * item_bytes(g) * (g.dual ? 2u : 1u);
      q += cnt;
    }
    uint64_t* bar = &R.full[st];
    mbar_arrive_expect_tx(bar, bytes);
    uint8_t* dst = R.stages + (size_t)st * R.chunk * R.slot_bytes;
    for (uint32_t q = i, ss = s; q < i + n; ++ss) {
      const MmvSeg& g = a.seg[ss];
      const uint32_t cnt = min(i + n, g.item0 + g.items) - q;
      const uint32_t len = cnt * item_bytes(g);
      const size_t off = (size_t)(q - g.item0) * item_bytes(g);
      bulk_g2s(dst, g.w + off, len, bar);
      if (g.dual) bulk_g2s(dst + R.chunk * item_bytes(g), g.w2 + off, len, bar);
      dst += len;
      q += cnt;
    }
    i += n;
    ++cpos;
    if (++st == R.ns) {
      st = 0;
      ++use;
    }
  }
  return true;
}

// Wait (bounded) for every chunk the producer issued to land before the CTA
// exits, so no bulk copy is in flight into released shared memory.
__device__ __forceinline__ void mmv_drain(const MRing& R, uint32_t n_chunks, int* err) {
  const uint32_t n = n_chunks < R.ns ? n_chunks : R.ns;
  for (uint32_t c = n_chunks - n; c < n_chunks; ++c)
    mbar_wait_spin(&R.full[c % R.ns], (c / R.ns) & 1u, err, DERR_TIMEOUT_FULL);
}

// ------------------------------ x prologue -------------------------------------
// Blocks per conversion batch (loads of a batch are in flight together).
constexpr int MMV_PU = 4;

struct XPre {  // RMSNorm weights of the first batch, loaded before the PDL wait
  float4 w[MMV_PU][2];
};
__device__ __forceinline__ void x_norm_prefetch(const MmvArgs& a, int warp, int lane, XPre& np) {
  if (!a.norm_w) return;
  const uint32_t NB = a.k / 256;
#pragma unroll
  for (int u = 0; u < MMV_PU; ++u) {
    const uint32_t kb = warp + u * MMV_WARPS;
    np.w[u][0] = np.w[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (kb < NB) {
      const float4* wn = reinterpret_cast<const float4*>(a.norm_w + 256 * (size_t)kb + 8 * lane);
      np.w[u][0] = __ldg(wn);
      np.w[u][1] = __ldg(wn + 1);
    }
  }
}

// Balanced base-256 digits of |v| <= 2^22: v = l0 + 256 l1 + 65536 l2, each a signed byte.
__device__ __forceinline__ void limbs3(int v, int& l0, int& l1, int& l2) {
  l0 = (int)(int8_t)(v & 0xFF);
  const int r = (v - l0) >> 8;
  l1 = (int)(int8_t)(r & 0xFF);
  l2 = (r - l1) >> 8;
}
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) |
         ((uint32_t)(d & 0xFF) << 24);
}

// Consumers (warps 0..MMV_WARPS-1): x (optionally x * norm_w) -> limbs and the
// per-range tables.  Warp w converts blocks w, w + MMV_WARPS, ...; lane l holds
// elements 8l..8l+7 of a block.  x is read with ld.global.cg (it may come from
// other CTAs of the same persistent launch).  Returns the output scale:
// inv_rms = 1/sqrt(mean(x^2) + 1e-5) with RMSNorm (engine/src/ops.c:195-214),
// else 1; W (x * inv_rms * w) = inv_rms * W (x * w).  Ends with a
// consumer-only barrier (id 1); `red`: MMV_WARPS floats of shared memory.
template <bool HAS4, bool HAS6>
__device__ __forceinline__ float mmv_prologue(const MmvArgs& a, const XRegion& X, float* red, int warp, int lane,
                                              const XPre* np) {
  const uint32_t K = a.k, NB = K / 256;
  const float* nw = a.norm_w;
  float ss = 0.f;
  if (warp == 0 && lane < 4) reinterpret_cast<uint32_t*>(X.zero)[lane] = 0u;
#pragma unroll 1
  for (uint32_t kb0 = warp, it = 0; kb0 < NB; kb0 += MMV_PU * MMV_WARPS, ++it) {
    const uint32_t nu = min((uint32_t)MMV_PU, (NB - kb0 + MMV_WARPS - 1) / MMV_WARPS);
    float v[MMV_PU][8];
#pragma unroll
    for (int u = 0; u < MMV_PU; ++u) {
      if ((uint32_t)u >= nu) break;
      const float4* src = reinterpret_cast<const float4*>(a.x + 256 * (size_t)(kb0 + u * MMV_WARPS) + 8 * lane);
      const float4 t0 = __ldcg(src), t1 = __ldcg(src + 1);
      v[u][0] = t0.x; v[u][1] = t0.y; v[u][2] = t0.z; v[u][3] = t0.w;
      v[u][4] = t1.x; v[u][5] = t1.y; v[u][6] = t1.z; v[u][7] = t1.w;
    }
#pragma unroll
    for (int u = 0; u < MMV_PU; ++u) {
      if ((uint32_t)u >= nu) break;
      const uint32_t kb = kb0 + u * MMV_WARPS;
      if (nw) {
        float4 w0, w1;
        if (it == 0 && np) {
          w0 = np->w[u][0];
          w1 = np->w[u][1];
        } else {
          const float4* wn = reinterpret_cast<const float4*>(nw + 256 * (size_t)kb + 8 * lane);
          w0 = __ldg(wn);
          w1 = __ldg(wn + 1);
        }
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ss = fmaf(v[u][e], v[u][e], ss);
          v[u][e] *= w[e];
        }
      }
      float amax = 0.f;
      bool fin = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        amax = fmaxf(amax, fabsf(v[u][e]));
        fin = fin && isfinite(v[u][e]);
      }
      amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
      fin = __all_sync(0xffffffffu, fin);
      // X_b = 2^(f-21) with amax in [2^f, 2^(f+1)): |x / X_b| < 2^22.  Maxima
      // below 2^-104 are treated as 2^-104; powers of two built from bits.
      const int e8 = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
      const int f = amax > 0.f ? max(e8 - 127, -104) : 0;
      const float xbv = fin ? __uint_as_float((uint32_t)(f - 21 + 127) << 23) : __int_as_float(0x7fc00000);
      const float inv_xb = __uint_as_float((uint32_t)(21 - f + 127) << 23);
      if (lane == 0) X.xb[kb] = xbv;
      int L[3][8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int xi = fin ? __float2int_rn(v[u][e] * inv_xb) : 0;
        limbs3(xi, L[0][e], L[1][e], L[2][e]);
      }
      const uint32_t kr = 8 * kb + (lane >> 2);
      uint8_t* dst = X.xl + (size_t)kr * 96 + 8 * (lane & 3);
#pragma unroll
      for (int l = 0; l < 3; ++l)
        *reinterpret_cast<uint2*>(dst + 32 * l) =
            make_uint2(pack4(L[l][0], L[l][1], L[l][2], L[l][3]), pack4(L[l][4], L[l][5], L[l][6], L[l][7]));
      if (HAS4) {  // fp32 sum of x per 32-element sub-block (4 lanes)
        float sm = ((v[u][0] + v[u][1]) + (v[u][2] + v[u][3])) + ((v[u][4] + v[u][5]) + (v[u][6] + v[u][7]));
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        if ((lane & 3) == 0) X.xs[kr] = sm;
      }
      if (HAS6) {  // -32 x limb sums per 16-element group (lane pairs)
        int s3[3];
#pragma unroll
        for (int l = 0; l < 3; ++l) {
          int s = 0;
#pragma unroll
          for (int e = 0; e < 8; ++e) s += L[l][e];
          s += __shfl_xor_sync(0xffffffffu, s, 1);
          s3[l] = -32 * s;
        }
        int* c = X.xc + (size_t)kr * 8;
        if ((lane & 3) == 0) {
          c[0] = s3[0];
          c[1] = s3[1];
          c[2] = s3[2];
        } else if ((lane & 3) == 2) {
          c[3] = s3[0];
          c[4] = s3[1];
          c[5] = s3[2];
          c[6] = 0;
          c[7] = 0;
        }
      }
    }
  }
  if (nw) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
  }
  named_sync(1, 32 * MMV_WARPS);
  if (!nw) return 1.0f;
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < MMV_WARPS; ++w) tot += red[w];
  return 1.0f / sqrtf(tot / (float)K + 1e-5f);
}

// --------------------------------- bodies --------------------------------------
// Per-lane accumulators of one matrix of an item: rows g and g+8, columns 2t
// and 2t+1 (F), and the Q4_K min term of rows g and g+8 (M).
struct Acc {
  float F[4];
  float M[2];
};

// One Q4_K tile (16 rows x 256), tile bytes T in shared memory: [0, 256) the
// 16 rows' GGUF block headers (d, dmin, scales[12]); [256, 2304) quants,
// [chunk j][lane][16 B] = row g bytes 32j+8t..+7, then row g+8's.
// bl[j], bh[j]: B operands of sub-blocks 2j, 2j+1.  xsp: this lane's two
// sub-block sums (sub-blocks 2t, 2t+1), xbv: X_b.
__device__ __forceinline__ void q4_tile(uint32_t T, const uint2 (&bl)[4], const uint2 (&bh)[4],
                                        float2 xsp, float xbv, int g, int t, int lane, Acc& acc) {
  const uint4 h0 = lds128(T + 16 * g), h1 = lds128(T + 16 * (g + 8));
  const uint32_t M4 = 0x0F0F0F0Fu;
  // 6-bit scales and mins (engine/src/ops.c:107-115 get_scale_min_k4), four per word
  const uint32_t scl0 = h0.y & 0x3F3F3F3Fu, scl1 = h1.y & 0x3F3F3F3Fu;
  const uint32_t sch0 = (h0.w & M4) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t sch1 = (h1.w & M4) | ((h1.y >> 2) & 0x30303030u);
  int Il[4] = {0, 0, 0, 0}, Ih[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 q = lds128(T + 256 + 512 * j + 16 * lane);
    int D[4];
    mma_u8s8(D, q.x & M4, q.z & M4, q.y & M4, q.w & M4, bl[j].x, bl[j].y, 0, 0, 0, 0);
    const uint32_t w0 = j < 2 ? scl0 : sch0, w1 = j < 2 ? scl1 : sch1;
    const uint32_t k0 = 2 * (j & 1);
    const int sl0 = ubyte(w0, k0), sl1 = ubyte(w1, k0);
    Il[0] += sl0 * D[0];
    Il[1] += sl0 * D[1];
    Il[2] += sl1 * D[2];
    Il[3] += sl1 * D[3];
    mma_u8s8(D, q.x & ~M4, q.z & ~M4, q.y & ~M4, q.w & ~M4, bh[j].x, bh[j].y, 0, 0, 0, 0);
    const int sh0 = ubyte(w0, k0 + 1), sh1 = ubyte(w1, k0 + 1);
    Ih[0] += sh0 * D[0];
    Ih[1] += sh0 * D[1];
    Ih[2] += sh1 * D[2];
    Ih[3] += sh1 * D[3];
  }
  // block result: d * X_b / 16 * (16 * sum_lo + sum_hi); high nibbles were 16x
  const float dx0 = ref_half(h0.x & 0xFFFFu) * (xbv * 0.0625f);
  const float dx1 = ref_half(h1.x & 0xFFFFu) * (xbv * 0.0625f);
  acc.F[0] = fmaf(dx0, (float)(16 * Il[0] + Ih[0]), acc.F[0]);
  acc.F[1] = fmaf(dx0, (float)(16 * Il[1] + Ih[1]), acc.F[1]);
  acc.F[2] = fmaf(dx1, (float)(16 * Il[2] + Ih[2]), acc.F[2]);
  acc.F[3] = fmaf(dx1, (float)(16 * Il[3] + Ih[3]), acc.F[3]);
  // min term, sub-blocks 2t and 2t+1 of this lane: dmin * (m_2t xs_2t + m_2t+1 xs_2t+1)
  const uint32_t mw0 = t < 2 ? (h0.z & 0x3F3F3F3Fu) : (((h0.w >> 4) & M4) | ((h0.z >> 2) & 0x30303030u));
  const uint32_t mw1 = t < 2 ? (h1.z & 0x3F3F3F3Fu) : (((h1.w >> 4) & M4) | ((h1.z >> 2) & 0x30303030u));
  const uint32_t km = 2 * (t & 1);
  const float m00 = (float)ubyte(mw0, km), m01 = (float)ubyte(mw0, km + 1);
  const float m10 = (float)ubyte(mw1, km), m11 = (float)ubyte(mw1, km + 1);
  acc.M[0] = fmaf(ref_half(h0.x >> 16), fmaf(m00, xsp.x, m01 * xsp.y), acc.M[0]);
  acc.M[1] = fmaf(ref_half(h1.x >> 16), fmaf(m10, xsp.x, m11 * xsp.y), acc.M[1]);
}

// One Q6_K tile: [0, 3072) quants, [half n][lane][48 B] = row g: ql bytes
// 64n+8t..+7, ql 64n+32+8t..+7, qh 32n+8t..+7, then row g+8 the same;
// [3072, 3328) int8 scales[16] per row; [3328, 3360) fp16 d per row.
// b[4n+g4] / c[4n+g4]: B operand and C input of range (n, g4).
__device__ __forceinline__ uint32_t q6_word(uint32_t ql0, uint32_t ql1, uint32_t hm, uint32_t hn, int g4) {
  const uint32_t M4 = 0x0F0F0F0Fu;
  switch (g4) {
    case 0: return lop_sel(ql0, hm << 4, M4);
    case 1: return lop_sel(ql1, hn << 2, M4);
    case 2: return lop_sel(ql0 >> 4, hm, M4);
    default: return lop_sel(ql1 >> 4, hn >> 2, M4);
  }
}
// sel[q][c]: PRMT selectors of the scale byte 2q + (column c's group) in a
// word of four scales (column 2t uses the second 16-element group when t >= 2,
// column 2t+1 when t >= 1).
__device__ __forceinline__ void q6_scale_sels(int t, uint32_t (&sel)[2][2]) {
  const uint32_t o0 = t >= 2 ? 1u : 0u, o1 = t >= 1 ? 1u : 0u;
  sel[0][0] = sx_sel(o0);
  sel[0][1] = sx_sel(o1);
  sel[1][0] = sx_sel(2u + o0);
  sel[1][1] = sx_sel(2u + o1);
}
__device__ __forceinline__ void q6_tile(uint32_t T, const uint2 (&b)[8], const uint2 (&c)[8],
                                        float xbv, const uint32_t (&sel)[2][2], int lane, int g, Acc& acc) {
  const uint4 S0 = lds128(T + 3072 + 16 * g), S1 = lds128(T + 3072 + 16 * (g + 8));
  const uint32_t s0w[4] = {S0.x, S0.y, S0.z, S0.w}, s1w[4] = {S1.x, S1.y, S1.z, S1.w};
  int I[4] = {0, 0, 0, 0};
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    const uint32_t Q = T + 1536 * n + 48 * lane;
    const uint4 v0 = lds128(Q), v1 = lds128(Q + 16), v2 = lds128(Q + 32);
    // row g: ql0 = (v0.x, v0.y), ql1 = (v0.z, v0.w), qh = (v1.x, v1.y)
    // row h: ql0 = (v1.z, v1.w), ql1 = (v2.x, v2.y), qh = (v2.z, v2.w)
    const uint32_t gm0 = v1.x & 0x33333333u, gn0 = v1.x & 0xCCCCCCCCu;
    const uint32_t gm1 = v1.y & 0x33333333u, gn1 = v1.y & 0xCCCCCCCCu;
    const uint32_t hm0 = v2.z & 0x33333333u, hn0 = v2.z & 0xCCCCCCCCu;
    const uint32_t hm1 = v2.w & 0x33333333u, hn1 = v2.w & 0xCCCCCCCCu;
#pragma unroll
    for (int g4 = 0; g4 < 4; ++g4) {
      const int r = 4 * n + g4;
      const uint32_t a0 = q6_word(v0.x, v0.z, gm0, gn0, g4);  // row g, elements 8t..8t+3
      const uint32_t a2 = q6_word(v0.y, v0.w, gm1, gn1, g4);  // row g, 8t+4..8t+7
      const uint32_t a1 = q6_word(v1.z, v2.x, hm0, hn0, g4);  // row g+8
      const uint32_t a3 = q6_word(v1.w, v2.y, hm1, hn1, g4);
      int D[4];
      mma_u8s8(D, a0, a1, a2, a3, b[r].x, b[r].y, (int)c[r].x, (int)c[r].y, (int)c[r].x, (int)c[r].y);
      // scale index 8n + 2 g4 (+1 for the second group): word 2n + (g4 >> 1), byte 2 (g4 & 1) (+1)
      const uint32_t wi = 2 * n + (g4 >> 1), q = g4 & 1;
      I[0] += sbyte_sel(s0w[wi], sel[q][0]) * D[0];
      I[1] += sbyte_sel(s0w[wi], sel[q][1]) * D[1];
      I[2] += sbyte_sel(s1w[wi], sel[q][0]) * D[2];
      I[3] += sbyte_sel(s1w[wi], sel[q][1]) * D[3];
    }
  }
  const float dx0 = ref_half(lds16(T + 3328 + 2 * g)) * xbv, dx1 = ref_half(lds16(T + 3328 + 2 * (g + 8))) * xbv;
  acc.F[0] = fmaf(dx0, (float)I[0], acc.F[0]);
  acc.F[1] = fmaf(dx0, (float)I[1], acc.F[1]);
  acc.F[2] = fmaf(dx1, (float)I[2], acc.F[2]);
  acc.F[3] = fmaf(dx1, (float)I[3], acc.F[3]);
}

// Row values of an item's matrix in lanes t == 0 (rows g, g+8), summed over
// the four lanes of a row group: sum_c 256^limb(c) F_c - M.
__device__ __forceinline__ void acc_rows(const Acc& acc, bool q4, int t, float& vg, float& vh) {
  // column 2t and 2t+1 weights: Q4_K limbs 0..2 (columns 3..7 are zero),
  // Q6_K limb c % 3 for c < 6
  const int c0 = 2 * t, c1 = 2 * t + 1;
  const float w0 = q4 ? (c0 == 0 ? 1.f : c0 == 2 ? 65536.f : 0.f)
                      : (c0 == 0 ? 1.f : c0 == 2 ? 65536.f : c0 == 4 ? 256.f : 0.f);
  const float w1 = q4 ? (c1 == 1 ? 256.f : 0.f) : (c1 == 1 ? 256.f : c1 == 3 ? 1.f : c1 == 5 ? 65536.f : 0.f);
  vg = fmaf(acc.F[0], w0, acc.F[1] * w1);
  vh = fmaf(acc.F[2], w0, acc.F[3] * w1);
  if (q4) {
    vg -= acc.M[0];
    vh -= acc.M[1];
  }
  vg += __shfl_xor_sync(0xffffffffu, vg, 1);
  vh += __shfl_xor_sync(0xffffffffu, vh, 1);
  vg += __shfl_xor_sync(0xffffffffu, vg, 2);
  vh += __shfl_xor_sync(0xffffffffu, vh, 2);
}

// The blocks [it.b0, it.b0 + nbs) of an item (one or two matrices) whose
// tiles are at S (gate) and S + nbs * tile bytes (up).
template <int NM>
__device__ __forceinline__ void item_q4(uint32_t S0, uint32_t S1, const Item& it, const XRegion& X,
                                        uint32_t boff_q4, int g, int t, int lane, Acc (&acc)[2]) {
#pragma unroll 1
  for (uint32_t bi = 0; bi < it.nbs; ++bi) {
    const uint32_t b = it.b0 + bi;
    uint2 bl[4], bh[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t xr = X.a_xl + (8 * b + 2 * j) * 96;
      bl[j] = lds64(boff_q4 == 0xFFFFFFFFu ? X.a_zero : xr + boff_q4);
      bh[j] = lds64(boff_q4 == 0xFFFFFFFFu ? X.a_zero : xr + 96 + boff_q4);
    }
    const uint2 xs2 = lds64(X.a_xs + 4 * (8 * b + 2 * t));
    const float2 xsp = make_float2(__uint_as_float(xs2.x), __uint_as_float(xs2.y));
    const float xbv = __uint_as_float(lds32(X.a_xb + 4 * b));
#pragma unroll
    for (int mi = 0; mi < NM; ++mi)
      q4_tile((mi == 0 ? S0 : S1) + bi * Q4T_BYTES, bl, bh, xsp, xbv, g, t, lane, acc[mi]);
  }
}
template <int NM>
__device__ __forceinline__ void item_q6(uint32_t S0, uint32_t S1, const Item& it, const XRegion& X,
                                        uint32_t boff_q6, const uint32_t (&sel)[2][2], int g, int t, int lane,
                                        Acc (&acc)[2]) {
#pragma unroll 1
  for (uint32_t bi = 0; bi < it.nbs; ++bi) {
    const uint32_t b = it.b0 + bi;
    uint2 bb[8], cc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint32_t kr = 8 * b + r;
      bb[r] = lds64(boff_q6 == 0xFFFFFFFFu ? X.a_zero : X.a_xl + kr * 96 + boff_q6);
      cc[r] = lds64(X.a_xc + kr * 32 + 8 * t);
    }
    const float xbv = __uint_as_float(lds32(X.a_xb + 4 * b));
#pragma unroll
    for (int mi = 0; mi < NM; ++mi)
      q6_tile((mi == 0 ? S0 : S1) + bi * Q6T_BYTES, bb, cc, xbv, sel, lane, g, acc[mi]);
  }
}

// --------------------------- reduction + epilogue -------------------------------
// K-slice partials: a.red_slots item slots of a.red_stride floats (16 rows,
// then for a dual plan the 16 up rows: 32) in MMV_RED_FLOATS floats of shared
// memory, and as many row-tile counters.  An item's slot is its global index %
// red_slots, a row tile's counter the global index of its first item %
// red_slots.  While a row tile waits for its reduction, the items that may
// run are bounded by the ring (the reducing warp has not released its next
// item), so slices + stages + warps < red_slots (checked by the planner) keeps
// every slot in use unique.
constexpr int MMV_RED_FLOATS = 4096;
constexpr int MMV_RED_MAX_SLOTS = 256;

__device__ __forceinline__ void epilogue(const MmvArgs& a, const MmvSeg& g, uint32_t row0, int lane, float v,
                                         float osc) {
  // lanes 0..15: row row0 + lane (value v); lanes 16..31: the up row (dual)
  const uint32_t r = (uint32_t)(lane & 15);
  const uint32_t row = row0 + r;
  v *= osc;
  if (g.dual) {
    const float u = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < 16 && row < g.m) {
      const float sig = 1.0f / (1.0f + expf(-v));  // SwiGLU (engine/src/ops.c:491-496)
      g.y[row] = (v * sig) * u;
    }
    return;
  }
  if (g.epi == EPI_ROPE) {
    // (2i, 2i+1) pairs are lanes r, r+1 (row0 is a multiple of 16)
    const float o1 = __shfl_down_sync(0xffffffffu, v, 1);
    if (lane < 16 && (r & 1) == 0 && row + 1 < g.m) {
      const float p = (float)__ldcg(a.pos);
      const uint32_t i = row % g.rope_hd;
      // angle = pos * freq in fp32 as engine/src/ops.c:227-228
      const float ang = p * a.rope_freq[i >> 1];
      const float c = cosf(ang), sn = sinf(ang);
      g.y[row] = v * c - o1 * sn;
      g.y[row + 1] = v * sn + o1 * c;
    }
    return;
  }
  if (lane < 16 && row < g.m) {
    if (g.epi == EPI_ADD)
      g.y[row] = __ldcg(&g.y[row]) + v;
    else
      g.y[row] = v;
  }
}

// Consumers: warp `warp` takes this CTA's local items warp, warp + MMV_WARPS,
// ... of [i0, i1); cbase: the ring position (chunks) of item i0.  False if a
// bounded wait ran out.
template <bool HAS4, bool HAS6>
__device__ __forceinline__ bool mmv_consume(const MmvArgs& a, const MRing& R, uint32_t i0, uint32_t i1,
                                            uint32_t cbase, const XRegion& X, float osc, float* part, int* cnt,
                                            int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  // B operand offsets inside a 96-byte range (0xFFFFFFFF: no column, zeros)
  const uint32_t boff_q4 = g < 3 ? (uint32_t)(32 * g + 8 * t) : 0xFFFFFFFFu;
  const uint32_t boff_q6 = (g < 3 && t < 2) ? (uint32_t)(32 * g + 8 * t)
                           : (g >= 3 && g < 6 && t >= 2) ? (uint32_t)(32 * (g - 3) + 8 * t)
                                                         : 0xFFFFFFFFu;
  uint32_t sel6[2][2];
  q6_scale_sels(t, sel6);
  // ring position of this warp's current chunk (chunk index c, its stage st,
  // the stage's use count) and its current item, advanced without division
  uint32_t c = cbase, st = cbase % R.ns, use = cbase / R.ns;
  Item it = item_of(a, min(i0 + warp, i1 > 0 ? i1 - 1 : 0));
  for (uint32_t i = i0 + warp; i < i1; i += MMV_WARPS) {
    // local item j: chunk cbase + j / chunk, slot k = j % chunk
    const uint32_t j = i - i0, k = j & (R.chunk - 1);
    for (const uint32_t cn = cbase + (j >> R.lg_chunk); c < cn; ++c)
      if (++st == R.ns) {
        st = 0;
        ++use;
      }
    if (!mbar_wait_spin(&R.full[st], use & 1u, a.err, DERR_TIMEOUT_FULL)) return false;
    if (i != i0 + warp) item_skip(a, it, MMV_WARPS);
    const MmvSeg& sg = a.seg[it.s];
    const uint32_t base = smem_u32(R.stages) + st * R.chunk * R.slot_bytes;
    const uint32_t S0 = base + (a.nseg == 1 ? k * item_bytes(sg) : chunk_off(a, i - k, i));
    const uint32_t S1 = base + R.chunk * item_bytes(sg) + k * item_bytes(sg);
    Acc acc[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) acc[m] = Acc{{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f}};
    const bool q4 = sg.qt == T_Q4K;
    if (HAS4 && (!HAS6 || q4)) {
      if (sg.dual)
        item_q4<2>(S0, S1, it, X, boff_q4, g, t, lane, acc);
      else
        item_q4<1>(S0, S1, it, X, boff_q4, g, t, lane, acc);
    } else if (HAS6) {
      if (sg.dual)
        item_q6<2>(S0, S1, it, X, boff_q6, sel6, g, t, lane, acc);
      else
        item_q6<1>(S0, S1, it, X, boff_q6, sel6, g, t, lane, acc);
    }
    __syncwarp();
    if (lane == 0) {
      // the stage's bytes are no longer read; the CTA's last item of a plan
      // also stands in for the empty slots of a partial last chunk
      const uint32_t extra = (i + 1 == i1) ? R.chunk - 1 - k : 0u;
      mbar_arrive_cnt(&R.empty[st], 1u + extra);
    }
    float vg0, vh0, vg1 = 0.f, vh1 = 0.f;
    acc_rows(acc[0], q4, t, vg0, vh0);
    if (sg.dual) acc_rows(acc[1], q4, t, vg1, vh1);
    const uint32_t nsl = a.red_slots, srd = a.red_stride;
    float* pp = part + (i % nsl) * srd;
    if (t == 0) {
      pp[g] = vg0;
      pp[g + 8] = vh0;
      if (sg.dual) {
        pp[16 + g] = vg1;
        pp[24 + g] = vh1;
      }
    }
    // this CTA's slices of the row tile: [lo_s, hi_s) of its [first, first + ks)
    const uint32_t first = i - it.sl;
    const uint32_t lo_s = max(first, i0), hi_s = min(first + (uint32_t)sg.ks, i1);
    const int nloc = (int)(hi_s - lo_s);
    int last = 1;
    __syncwarp();
    if (nloc > 1) {
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&cnt[first % nsl], 1) == nloc - 1;
        if (last) {
          cnt[first % nsl] = 0;
          __threadfence_block();
        }
      }
      last = __shfl_sync(0xffffffffu, last, 0);
    }
    if (!last) continue;
    // the row tile's slices in slice order
    const volatile float* vp = part;
    float v = 0.f;
    if ((uint32_t)lane < srd)
      for (uint32_t q = lo_s; q < hi_s; ++q) v += vp[(q % nsl) * srd + lane];
    if (nloc < (int)sg.ks) {
      // the other slices are in the neighbouring CTA: combine through global
      // memory, lower part + upper part, by whichever CTA comes second
      const bool upper = first < i0;
      const uint32_t b = upper ? blockIdx.x : blockIdx.x + 1;
      float* xp = a.xpart + (size_t)b * 64;
      xp[(upper ? 32 : 0) + lane] = v;
      __syncwarp();
      int second = 0;
      if (lane == 0) {
        __threadfence();
        second = atomicAdd(&a.xcnt[b], 1) == 1;
        if (second) {
          a.xcnt[b] = 0;
          __threadfence();
        }
      }
      second = __shfl_sync(0xffffffffu, second, 0);
      if (!second) continue;
      const float other = __ldcg(xp + (upper ? 0 : 32) + lane);
      v = upper ? other + v : v + other;
    }
    epilogue(a, sg, 16 * it.t, lane, v, osc);
  }
  return true;
}

}  // namespace mdev
}  // namespace shk
