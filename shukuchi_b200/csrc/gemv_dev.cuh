// gemv_dev.cuh -- device side of the batch-1 Q4_K / Q6_K dequantise-matvec:
// task math, the shared-memory stage ring, producer / prologue / consumer
// bodies.  Used by the stand-alone GEMV kernel (gemv.cu) and the persistent
// decode kernel (decode.cu).
//
// Reference semantics: op_matmul_q4_k / op_matmul_q6_k (engine/src/ops.c:266-314,
// 361-404): y[r] = sum_k dequant(W[r, k]) * x[k] over 256-element super-blocks
// laid out row-major as in GGUF.  Summation order differs from the reference's
// sequential fp32 sum; results agree to fp32 rounding.
//
// Kernel shape (one CTA per SM, persistent over a byte-balanced row range):
//  * warp GEMV_WARPS (15) is the producer: one lane streams whole-row chunks
//    of the weight matrix into a shared-memory ring with cp.async.bulk (TMA,
//    1-D, no tensor map, one destination CTA), completion tracked by mbarrier
//    tx-counts; a per-stage generation tag orders consumers that skip ahead;
//  * warps 0-14 are consumers: they load x (bulk copies, RMSNorm fused) and
//    turn it into the fixed-point form below while the first chunks are in
//    flight, then decode blocks from the ring.  The last warp to finish a chunk's tasks releases
//    its stage.
//
// Arithmetic: the weights' integer quants are multiplied with integer limbs of
// x by dp4a, exactly, in int32.  Each 256-element block of x is written as
// X_b * x_int with X_b a power of two and |x_int| <= 2^22 (24-bit fixed point,
// relative step 2^-22 of the block maximum, i.e. fp32-level precision for the
// dot product), and x_int = l0 + 256*l1 + 65536*l2 where l0, l1 are its two low
// bytes (unsigned) and l2 its third byte read as signed: two's complement makes
// the bytes of x_int exactly its limbs.  Per
// sub-block the three limb sums are scaled by the 6-bit (Q4_K) or int8 (Q6_K)
// sub-block scale with IMAD, then per block converted to float and multiplied by
// d * X_b.  The Q4_K min term uses fp32 sums of x; the Q6_K -32 offset comes
// from -32 * limb sums carried in the unused fourth words of the x vectors.  Integer packing keeps the
// per-weight work on the dp4a/IMAD path instead of the half-rate logic pipe.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"

// Unroll factors of the per-block inner loops (1: rolled, compact code).
#ifndef SHK_Q4_JU
#define SHK_Q4_JU 1
#endif
#ifndef SHK_Q6_ISU
#define SHK_Q6_ISU 1
#endif
#ifndef SHK_Q6_NU
#define SHK_Q6_NU 1
#endif
#define SHK_PRAGMA(x) _Pragma(#x)
#define SHK_UNROLL(n) SHK_PRAGMA(unroll n)

namespace shk {
namespace gdev {

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// x limbs live in shared memory as int4 vectors {l0 word, l1 word, l2 word, 0}
// (4 elements each).  A 256-element block b takes 65 slots from 65b: its first
// 32 vectors, one pad slot, then the last 32 (vector w of the block at
// 65b + w + (w >= 32)).  Lanes reading the same offset of consecutive blocks
// (Q4_K: a lane per block) and lanes reading half n of every second block
// (Q6_K: 65*2s + 33n) then fall in distinct 16-byte bank groups.
__device__ __forceinline__ uint32_t xpad(uint32_t v) { return v + (v >> 6) + ((v >> 5) & 1u); }

// Limbs 0 and 1 of x are unsigned bytes, limb 2 is a signed byte (see the
// prologue); quants are unsigned and below 64, so limb 2 may use the signed form.
__device__ __forceinline__ int dp4a_u(uint32_t a, int b, int c) {
  return (int)__dp4a(a, (uint32_t)b, (uint32_t)c);
}
// a: four unsigned bytes, b: four signed bytes
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ float limbs_to_float(int a0, int a1, int a2) {
  return fmaf(65536.0f, (float)a2, fmaf(256.0f, (float)a1, (float)a0));
}

// Code size matters here: the hot loops below are written so that one
// compact body per quant type serves every segment kind (single, dual,
// RoPE) -- a kernel whose instruction footprint overflows the SM's
// instruction caches stalls on fetch rather than on memory.

// ------------------------------- Q4_K ---------------------------------------
// Two rows (r0, r1: consecutive rows, or the gate and up rows of a dual
// segment) of one 256-element block against x block xblk.  The four
// 64-element groups j (low nibbles = sub-block 2j, high nibbles = 2j+1,
// engine/src/ops.c:117-142) run in a rolled loop.  High nibbles are used in
// place (q << 4, masked, no shift): their dp4a sums are 16x, so the low
// sub-block's scale is taken 16x as well and the block result is divided by 16
// (exact).  Per group: |16 sc_lo S_lo + sc_hi S_hi| <= 2 * 63 * 32 * 240 * 255,
// four groups stay below 2^31.
__device__ __forceinline__ void q4k_block2(const uint8_t* __restrict__ r0, const uint8_t* __restrict__ r1,
                                           const int4* __restrict__ xblk, float xb,
                                           const float* __restrict__ xs, float& acc0, float& acc1) {
  const uint8_t* rp[2] = {r0, r1};
  uint32_t scl[2], sch[2], ml[2], mh[2];
  float dx[2], dm[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4 h = *reinterpret_cast<const uint4*>(rp[r]);
    // 6-bit scales/mins of sub-blocks 0-3 and 4-7, packed four per word
    // (engine/src/ops.c:107-115 get_scale_min_k4)
    scl[r] = h.y & 0x3F3F3F3Fu;
    ml[r] = h.z & 0x3F3F3F3Fu;
    sch[r] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    mh[r] = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    dx[r] = ref_half(h.x & 0xFFFFu) * xb;
    dm[r] = ref_half(h.x >> 16);
  }
  int A[2][3] = {{0, 0, 0}, {0, 0, 0}};
  float M[2] = {0.f, 0.f};
SHK_UNROLL(SHK_Q4_JU)
  for (int j = 0; j < 4; ++j) {
    int S[2][2][3] = {{{0, 0, 0}, {0, 0, 0}}, {{0, 0, 0}, {0, 0, 0}}};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint4 w[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) w[r] = *reinterpret_cast<const uint4*>(rp[r] + 16 + 32 * j + 16 * half);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int4* xj = xblk + 16 * j + (j >> 1);  // groups 2, 3 follow the pad slot
        const int4 xl = xj[4 * half + i];
        const int4 xh = xj[8 + 4 * half + i];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint32_t q = i == 0 ? w[r].x : i == 1 ? w[r].y : i == 2 ? w[r].z : w[r].w;
          const uint32_t lo = q & 0x0F0F0F0Fu, hi = q & 0xF0F0F0F0u;
          S[r][0][0] = dp4a_u(lo, xl.x, S[r][0][0]);
          S[r][0][1] = dp4a_u(lo, xl.y, S[r][0][1]);
          S[r][0][2] = dp4a_us(lo, xl.z, S[r][0][2]);
          S[r][1][0] = dp4a_u(hi, xh.x, S[r][1][0]);
          S[r][1][1] = dp4a_u(hi, xh.y, S[r][1][1]);
          S[r][1][2] = dp4a_us(hi, xh.z, S[r][1][2]);
        }
      }
    }
    const float2 xsum = *reinterpret_cast<const float2*>(xs + 2 * j);
    const uint32_t sel = 0x4440u + 2u * (uint32_t)(j & 1);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t scw = j < 2 ? scl[r] : sch[r], mw = j < 2 ? ml[r] : mh[r];
      const int sc0 = (int)__byte_perm(scw, 0u, sel) << 4;  // x16: see above
      const int sc1 = (int)__byte_perm(scw, 0u, sel + 1);
      const int m0 = (int)__byte_perm(mw, 0u, sel);
      const int m1 = (int)__byte_perm(mw, 0u, sel + 1);
#pragma unroll
      for (int l = 0; l < 3; ++l) A[r][l] += sc0 * S[r][0][l] + sc1 * S[r][1][l];
      M[r] = fmaf((float)m0, xsum.x, fmaf((float)m1, xsum.y, M[r]));
    }
  }
  acc0 += fmaf(dx[0], limbs_to_float(A[0][0], A[0][1], A[0][2]) * 0.0625f, -(dm[0] * M[0]));
  acc1 += fmaf(dx[1], limbs_to_float(A[1][0], A[1][1], A[1][2]) * 0.0625f, -(dm[1] * M[1]));
}

// ------------------------------- Q6_K ---------------------------------------
// Rows are in the planar layout of repack.cu: block b's ql chunk c (16 bytes)
// at 128 b + 16 ((c + b) & 7), qh chunk c at 128 nb + 64 b + 16 ((c + (b >> 1))
// & 3), scales at 192 nb + 16 b, d at 208 nb + 2 b -- every load is an aligned
// vector load, and lanes on consecutive blocks hit distinct bank groups.
__device__ __forceinline__ uint32_t w4(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// One Q6_K block (both 128-element halves n) of NR rows (engine/src/ops.c:
// 167-193 dequantize_row_q6_k).  For each 32-bit word i of ql/qh, four words
// of exact 6-bit quants are formed (element groups +0, +32, +64, +96) and fed
// to dp4a; each 16-element scale group's three limb sums start at -32 * (sum
// of x limbs), which applies the -32 offset.  |T| < 16 groups * 2^19 * 128 <
// 2^31.  NR = 2 rows (r0, r1) or NR = 1 (r0 only).
template <int NR>
__device__ __forceinline__ void q6k_block(const uint8_t* __restrict__ r0, const uint8_t* __restrict__ r1,
                                          uint32_t nb, uint32_t b, const int4* __restrict__ xblk,
                                          float xb, float& acc0, float& acc1) {
  const uint32_t MK = 0x0F0F0F0Fu;
  const uint8_t* rp[2] = {r0, r1};
  const uint32_t qlb = 128u * b, qhb = 128u * nb + 64u * b, scb = 192u * nb + 16u * b;
  const uint32_t rq = b & 7u, rh = (b >> 1) & 3u;
  float dd[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) dd[r] = ref_half(*reinterpret_cast<const uint16_t*>(rp[r] + 208u * nb + 2u * b)) * xb;
  int T[NR][3];
#pragma unroll
  for (int r = 0; r < NR; ++r) T[r][0] = T[r][1] = T[r][2] = 0;
SHK_UNROLL(SHK_Q6_NU)
  for (int n = 0; n < 2; ++n) {
    uint2 SC[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) SC[r] = *reinterpret_cast<const uint2*>(rp[r] + scb + 8u * n);
    const int4* xh = xblk + 33 * n;
SHK_UNROLL(SHK_Q6_ISU)
    for (int is = 0; is < 2; ++is) {
      uint4 A[NR], B[NR], H[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        A[r] = *reinterpret_cast<const uint4*>(rp[r] + qlb + 16u * ((4u * n + is + rq) & 7u));
        B[r] = *reinterpret_cast<const uint4*>(rp[r] + qlb + 16u * ((4u * n + 2u + is + rq) & 7u));
        H[r] = *reinterpret_cast<const uint4*>(rp[r] + qhb + 16u * ((2u * n + is + rh) & 3u));
      }
      int S[NR][4][3];
#pragma unroll
      for (int g = 0; g < 4; ++g)
#pragma unroll
        for (int r = 0; r < NR; ++r) S[r][g][0] = S[r][g][1] = S[r][g][2] = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int4 xv[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) xv[g] = xh[8 * g + 4 * is + i];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          const uint32_t h = w4(H[r], i), a = w4(A[r], i), bq = w4(B[r], i);
          const uint32_t hm = h & 0x33333333u, hn = h & 0xCCCCCCCCu;
          const uint32_t Q[4] = {lop_sel(a, hm << 4, MK), lop_sel(bq, hn << 2, MK), lop_sel(a >> 4, hm, MK),
                                 lop_sel(bq >> 4, hn >> 2, MK)};
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            // the -32 offset: vector i < 3 of a 16-group carries -32 * (sum of
            // the group's limb i) in its fourth word
            if (i < 3) S[r][g][i] += xv[g].w;
            S[r][g][0] = dp4a_u(Q[g], xv[g].x, S[r][g][0]);
            S[r][g][1] = dp4a_u(Q[g], xv[g].y, S[r][g][1]);
            S[r][g][2] = dp4a_us(Q[g], xv[g].z, S[r][g][2]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t si = (uint32_t)is + 2u * g;  // scale index within this half
          const int sc = (int)(int8_t)__byte_perm(g < 2 ? SC[r].x : SC[r].y, 0u, 0x4440u + (si & 3u));
          T[r][0] += sc * S[r][g][0];
          T[r][1] += sc * S[r][g][1];
          T[r][2] += sc * S[r][g][2];
        }
    }
  }
  acc0 = fmaf(dd[0], limbs_to_float(T[0][0], T[0][1], T[0][2]), acc0);
  if (NR == 2) acc1 = fmaf(dd[NR - 1], limbs_to_float(T[NR - 1][0], T[NR - 1][1], T[NR - 1][2]), acc1);
}

// ------------------------------ chunk walk ----------------------------------
struct Range {
  uint32_t ub, ue;
};
// Task units (rg*rl rows) of segment s whose starting cost lies in [lo, hi).
__device__ __forceinline__ Range seg_units(const GemvArgs& a, int s, uint64_t seg_off, uint64_t lo,
                                           uint64_t hi) {
  const GemvSeg& g = a.seg[s];
  const uint32_t ur = (uint32_t)g.rg * g.rl;
  const uint64_t units = (g.m + ur - 1) / ur;
  auto first_at_or_after = [&](uint64_t c) -> uint64_t {
    if (c <= seg_off) return 0;
    const uint64_t u = (c - seg_off + g.unit_cost - 1) / g.unit_cost;
    return u < units ? u : units;
  };
  return Range{(uint32_t)first_at_or_after(lo), (uint32_t)first_at_or_after(hi)};
}

// Epilogue of one lane group: rl = 2 gives rows row, row+1 (o0, o1); rl = 1
// one row (o0), or for a dual segment the gate (o0) and up (o1) of one row.
__device__ __forceinline__ void store2(const GemvArgs& a, const GemvSeg& g, uint32_t row, int nvalid,
                                       float o0, float o1) {
  if (g.dual) {  // EPI_SWIGLU: silu(gate) * up (engine/src/ops.c:491-496)
    const float sig = 1.0f / (1.0f + expf(-o0));
    g.y[row] = (o0 * sig) * o1;
    return;
  }
  const bool two = g.rl == 2 && nvalid > 1;
  if (g.epi == EPI_TP) {  // peer stores over NVLink; the last CTA raises the flags
    const GemvTp& t = a.tp;
    const size_t base = (size_t)t.rank * t.d + t.row_off + row;
    for (uint32_t p = 0; p < t.world; ++p) {
      t.parts_out[p][base] = o0;
      if (two) t.parts_out[p][base + 1] = o1;
    }
    return;
  }
  if (g.epi == EPI_ROPE) {
    // (2i, 2i+1) pairs are the two rows of this lane (rl = 2, row even)
    if (!two) return;
    const float p = (float)__ldcg(a.pos);
    const uint32_t i = row % g.rope_hd;
    // angle = pos * freq in fp32 as engine/src/ops.c:227-228; freq comes from
    // a table built with the host libm powf, so the angle matches bit for bit
    const float ang = p * a.rope_freq[i >> 1];
    const float c = cosf(ang), sn = sinf(ang);
    g.y[row] = o0 * c - o1 * sn;
    g.y[row + 1] = o0 * sn + o1 * c;
  } else if (g.epi == EPI_ADD) {
    g.y[row] = __ldcg(&g.y[row]) + o0;
    if (two) g.y[row + 1] = __ldcg(&g.y[row + 1]) + o1;
  } else {
    g.y[row] = o0;
    if (two) g.y[row + 1] = o1;
  }
}

struct XView {
  const int4* xq;     // padded limb vectors, K/4 (+ one pad vector per 256-block)
  const float* xbs;   // per-256-block scale X_b, K/256
  const float* xs32;  // Q4_K: fp32 sums of x per 32-element sub-block, K/32
  float oscale;       // output scale: the RMSNorm factor inv_rms, or 1
};

// One task of a chunk: rg lane groups, each owning rl output rows (two row
// pointers r0, r1 per lane: consecutive rows, gate/up rows, or r1 = r0 when a
// single row is wanted).  Rows past rows_valid read stale (in-bounds) stage
// bytes; their results are never stored.
//  32/rg lanes per group, a lane takes blocks s, s + 32/rg, ... (Q4_K and
//  planar Q6_K alike).
// K split (g.ks > 1, then rg = 1): this task covers slice `sl` of the blocks;
// each slice's warp leaves its two row sums in kp[sl] and the last slice to
// finish (counter kc) adds the slices in slice order and stores.
template <bool HAS4, bool HAS6>
__device__ __forceinline__ void run_task(const GemvArgs& a, const GemvSeg& g, const uint8_t* rows,
                                         uint32_t row0, int rows_valid, uint32_t dual_off,
                                         const XView& x, int lane, uint32_t sl = 0, float* kp = nullptr,
                                         int* kc = nullptr) {
  const int lg_rg = __ffs(g.rg) - 1;
  const int rl = g.rl;
  const bool q4 = g.qt == T_Q4K;
  const int spr = 32 >> lg_rg;
  const int grp = lane >> (5 - lg_rg);
  const int s = lane & (spr - 1);
  const uint32_t blo = sl * g.sw, bhi = min(g.nb, blo + g.sw);
  float o0 = 0.f, o1 = 0.f;
  if (grp * rl < rows_valid) {
    const uint8_t* r0 = rows + (size_t)(grp * rl) * g.row_stride;
    const uint8_t* r1 = g.dual ? r0 + dual_off : ((rl == 2 && grp * 2 + 1 < rows_valid) ? r0 + g.row_stride : r0);
    if (HAS4 && (!HAS6 || q4)) {
      for (uint32_t b = blo + s; b < bhi; b += spr)
        q4k_block2(r0 + (size_t)b * Q4K_BYTES, r1 + (size_t)b * Q4K_BYTES, x.xq + 65 * b, x.xbs[b],
                   x.xs32 + 8 * b, o0, o1);
    } else if (HAS6) {
      if (rl == 1 && !g.dual) {  // single row
        for (uint32_t b = blo + s; b < bhi; b += spr)
          q6k_block<1>(r0, r1, g.nb, b, x.xq + 65 * b, x.xbs[b], o0, o1);
      } else {
        for (uint32_t b = blo + s; b < bhi; b += spr)
          q6k_block<2>(r0, r1, g.nb, b, x.xq + 65 * b, x.xbs[b], o0, o1);
      }
    }
  }
  for (int o = 16 >> lg_rg; o > 0; o >>= 1) {
    o0 += __shfl_xor_sync(0xffffffffu, o0, o);
    o1 += __shfl_xor_sync(0xffffffffu, o1, o);
  }
  const int lpg = 32 >> lg_rg;  // lanes per group
  if (g.ks > 1) {
    if (lane == 0) {
      kp[2 * sl] = o0;
      kp[2 * sl + 1] = o1;
      __threadfence_block();
      if (atomicAdd(kc, 1) == (int)g.ks - 1) {  // the last slice of this row task
        __threadfence_block();
        const volatile float* vp = kp;
        float s0 = 0.f, s1 = 0.f;
        for (uint32_t k = 0; k < g.ks; ++k) {
          s0 += vp[2 * k];
          s1 += vp[2 * k + 1];
        }
        *kc = 0;
        if (rows_valid > 0) store2(a, g, row0, rows_valid, s0 * x.oscale, s1 * x.oscale);
      }
    }
    return;
  }
  if ((lane & (lpg - 1)) == 0 && grp * rl < rows_valid)
    store2(a, g, row0 + grp * rl, rows_valid - grp * rl, o0 * x.oscale, o1 * x.oscale);
}

// Shared-memory map: [full | empty | xbar barriers][done][gen][red]
// [K-split partials and counts][x-copy barriers, one per consumer warp]
// [x raw / limb vectors (K*4)][X_b (K/256)][xs32 (K/32, Q4_K)][stage ring].
// Each consumer warp bulk-copies its blocks of x into the limb-vector slots
// and turns them into limbs in place.
// K split of long rows (more than 32 blocks, e.g. the down projection): a row
// task's blocks are cut into ks <= GEMV_KS_MAX slices processed by different
// warps; a chunk then holds at most GEMV_KS_ROWT row tasks.
constexpr int GEMV_KS_MAX = 8;
constexpr int GEMV_KS_ROWT = 4;
constexpr int SMEM_KPART = (8 * (2 * GEMV_MAX_STAGES + 1) + 8 * GEMV_MAX_STAGES + 4 * 32 + 15) & ~15;
constexpr int SMEM_KCNT = SMEM_KPART + GEMV_MAX_STAGES * GEMV_KS_ROWT * GEMV_KS_MAX * 2 * 4;
constexpr int SMEM_XBARS = SMEM_KCNT + GEMV_MAX_STAGES * GEMV_KS_ROWT * 4;  // x copies: one mbarrier per warp
constexpr int SMEM_HDR = SMEM_XBARS + 16 * 8;

// Bounded spin until the producer has claimed stage `st` for chunk `it`.  A
// consumer may run several ring cycles ahead of a stage (it skips chunks with
// no task for it), so the mbarrier parity alone could name a stale phase; the
// tag makes the following parity wait refer to chunk `it` exactly.
__device__ __forceinline__ bool wait_gen(const volatile uint32_t* gen, uint32_t st, uint32_t it,
                                         int* err) {
  if (gen[st] == it) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1; gen[st] != it; ++n) {
    __nanosleep(32);
    if ((n & 31) == 0 && globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
      set_error(err, DERR_TIMEOUT_FULL);
      return false;
    }
  }
  return true;
}

// X_b array padded to a 16-byte multiple so xs32 (float2 loads) stays
// aligned for every K.
__host__ __device__ __forceinline__ uint32_t xbs_floats(uint32_t K) { return ((K / 256) + 3) & ~3u; }

__host__ __device__ __forceinline__ size_t xq_bytes(uint32_t K) {
  return (size_t)(K / 4 + K / 256) * 16;  // one pad vector per 64
}

__host__ __device__ __forceinline__ size_t x_region_bytes(uint32_t K, bool has4, bool /*has6*/) {
  size_t b = xq_bytes(K) + (size_t)xbs_floats(K) * 4;
  if (has4) b += (size_t)(K / 32) * 4;
  return b;
}


// ------------------------------ the ring ------------------------------------
// Shared-memory stage ring: `full[s]` completes when stage s holds its chunk
// (tx-count of the bulk copies), `empty[s]` when every task of that chunk is
// done; gen[s] tags the chunk a stage holds.  The producer and the consumers
// walk the same chunk sequence, so their positions (it, st, ph) agree.
struct Ring {
  uint64_t* full;
  uint64_t* empty;
  int* done;
  volatile uint32_t* gen;
  uint8_t* stages;
  uint32_t ns;           // stages
  uint32_t stage_bytes;  // bytes per stage (>= every chunk of every plan on this ring)
  float* kpart;          // K-split partial sums: [stage][row task][slice][2]
  int* kcnt;             // K-split slices done: [stage][row task]
};
struct RingPos {
  uint32_t it = 0, st = 0, ph = 0;  // chunk index, its stage, stage use parity
  __device__ __forceinline__ void advance(uint32_t ns) {
    ++it;
    if (++st == ns) {
      st = 0;
      ph ^= 1u;
    }
  }
};

#ifndef GEMV_PRE_STAGES
#define GEMV_PRE_STAGES 5
#endif
// Where the consumers release the rest of the ring fill: 0 once their x loads
// have landed, 1 after the limb conversion.
#ifndef GEMV_XREADY_AT
#define GEMV_XREADY_AT 0
#endif
// Producer (one lane): streams this CTA's chunks of plan `a` (cost range
// [lo, hi)) into the ring.  If xready is given, only GEMV_PRE_STAGES chunks
// are issued before the consumers signal that their loads of x have landed:
// a full ring of bulk copies queued ahead of those loads (about 30 MB over
// all SMs) would delay them by several microseconds.  False if a bounded wait
// ran out.
__device__ __forceinline__ bool gemv_produce(const GemvArgs& a, const Ring& R, RingPos& p,
                                             uint64_t lo, uint64_t hi, uint64_t* xready = nullptr) {
  uint32_t issued = 0;
  uint64_t seg_off = 0;
  for (uint32_t s = 0; s < a.nseg; ++s) {
    const GemvSeg& g = a.seg[s];
    const Range rr = seg_units(a, s, seg_off, lo, hi);
    const uint32_t lg_ur = __ffs((uint32_t)g.rg * g.rl) - 1, cu = g.chunk_rows >> lg_ur;
    for (uint32_t u = rr.ub; u < rr.ue; u += cu) {
      const uint32_t r0 = u << lg_ur;
      const uint32_t r1 = min(min(u + cu, rr.ue) << lg_ur, g.m);
      const uint32_t bytes = (r1 - r0) * g.row_stride;
      if (xready && issued == GEMV_PRE_STAGES &&
          !mbar_wait_bounded(xready, 0, a.err, DERR_TIMEOUT_FULL))
        return false;
      ++issued;
      if (p.it >= R.ns && !mbar_wait_bounded(&R.empty[p.st], p.ph ^ 1u, a.err, DERR_TIMEOUT_EMPTY))
        return false;
      uint8_t* dst = R.stages + (size_t)p.st * R.stage_bytes;
      R.gen[p.st] = p.it;
      mbar_arrive_expect_tx(&R.full[p.st], g.dual ? 2 * bytes : bytes);
      bulk_g2s(dst, g.w + (size_t)r0 * g.row_stride, bytes, &R.full[p.st]);
      if (g.dual) bulk_g2s(dst + bytes, g.w2 + (size_t)r0 * g.row_stride, bytes, &R.full[p.st]);
      p.advance(R.ns);
    }
    seg_off += (uint64_t)((g.m + (1u << lg_ur) - 1) >> lg_ur) * g.unit_cost;
  }
  return true;
}

// Before the CTA exits: wait (bounded) for the last issued stages to land, so
// no bulk copy is in flight into shared memory that is being released.
__device__ __forceinline__ void ring_drain(const Ring& R, const RingPos& p, int* err) {
  const uint32_t n_tail = p.it < R.ns ? p.it : R.ns;
  for (uint32_t t = p.it - n_tail; t < p.it; ++t)
    mbar_wait_bounded(&R.full[t % R.ns], (t / R.ns) & 1, err, DERR_TIMEOUT_FULL);
}

// Activations (x, the residual read by EPI_ADD, the position) may have been
// written earlier in the same launch by other CTAs (persistent decode kernel),
// so they are read with ld.global.cg (L2), never through the non-coherent
// or L1 paths.  Weights and norm vectors are read-only for the whole launch.
struct XBuf {
  int4* xq;
  float* xbs;
  float* xs32;
  __device__ __forceinline__ XView view(float oscale = 1.0f) const { return XView{xq, xbs, xs32, oscale}; }
};

// Consumers (warps 0..GEMV_WARPS-1): x (optionally RMSNorm'ed) -> fixed-point
// limb vectors in shared memory.  Ends with a consumer-only barrier.
// Profiling hook: a build may define GEMV_STAMP(i) to record a timestamp at
// point i of the prologue; empty by default.
#ifndef GEMV_STAMP
#define GEMV_STAMP(i)
#endif

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Consumers (warps 0..GEMV_WARPS-1): x (optionally RMSNorm'ed) -> fixed-point
// limb vectors in shared memory.  Warp w owns 256-blocks w, w+15, ...; lane l
// holds elements 8l..8l+7 of a block (limb vectors 2l, 2l+1), so a block's
// maximum is a warp reduction.  Raw x is first copied (bulk copies on the
// warp's barrier, or cp.async by every lane) into the very slots the lane
// later overwrites with limbs; xready (nullable) is arrived on by each warp at
// the point GEMV_XREADY_AT names.
// Rolled loops: this runs once per launch, compact code matters more.
// Ends with a consumer-only barrier.
// Step 1 of the prologue: start the copies of raw x into this lane's slots.
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Tensor-parallel consumer: wait (bounded) for every rank's partial of this
// step, then x = residual + partials in rank order, into the raw-x slots.
__device__ __forceinline__ bool gemv_x_tp(const GemvArgs& a, const XBuf& xb_, int warp, int lane) {
  const GemvTp& t = a.tp;
  const uint32_t NB = a.k / 256;
  float4* xr = reinterpret_cast<float4*>(xb_.xq);
  const uint32_t ep = __ldcg(t.epoch);
  bool ok = true;
  if (lane == 0) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t r = 0; r < t.world && ok; ++r) {
      for (uint32_t n = 0; (int)(ld_relaxed_sys(t.flags_in + r) - ep) < 0; ++n) {
        __nanosleep(64);
        if ((n & 31) == 31 && globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
          set_error(a.err, DERR_TIMEOUT_GRID);
          ok = false;
          break;
        }
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // acquire: the partials are read below
  }
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  __syncwarp();
#pragma unroll 1
  for (uint32_t kb = warp; kb < NB; kb += GEMV_WARPS) {
    const uint32_t e0 = 256 * kb + 8 * lane;
    float4 v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) v[h] = __ldcg(reinterpret_cast<const float4*>(a.x + e0) + h);
    for (uint32_t r = 0; r < t.world && ok; ++r) {
      if (e0 < t.cov_lo[r] || e0 >= t.cov_hi[r]) continue;  // ranges are multiples of 8 elements
      const float4* pr = reinterpret_cast<const float4*>(t.parts_in + (size_t)r * t.d + e0);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float4 q = __ldcg(pr + h);
        v[h].x += q.x;
        v[h].y += q.y;
        v[h].z += q.z;
        v[h].w += q.w;
      }
    }
    const uint32_t v0 = 64 * kb + 2 * lane;
    xr[xpad(v0)] = v[0];
    xr[xpad(v0 + 1)] = v[1];
    if (blockIdx.x == 0) {
      reinterpret_cast<float4*>(t.res_out + e0)[0] = v[0];
      reinterpret_cast<float4*>(t.res_out + e0)[1] = v[1];
    }
  }
  return ok;
}

// Tensor-parallel producer, after this warp's last task: once every consumer
// warp of every CTA is done, the last one raises this rank's flag on every
// rank.  `done` counts this CTA's finished warps (shared memory).
__device__ __forceinline__ void gemv_tp_signal(const GemvArgs& a, int* done, int lane) {
  const GemvTp& t = a.tp;
  __syncwarp();
  if (lane != 0) return;
  __threadfence_block();  // release (CTA scope): this warp's stores before its count
  if (atomicAdd(done, 1) != GEMV_WARPS - 1) return;
  // the CTA's last warp: one system-scope fence orders every warp's peer
  // stores (they happen before it through the counts) before the count below
  __threadfence_system();
  if (atomicAdd(t.counter, 1u) != gridDim.x - 1) return;
  __threadfence_system();
  const uint32_t ep = __ldcg(t.epoch);
  for (uint32_t p = 0; p < t.world; ++p)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(t.flags_out[p] + t.rank), "r"(ep) : "memory");
  *t.counter = 0;
}

// x by 1-D bulk copies (two 512-byte runs per 256-element block, around the
// block's pad slot) on the warp's mbarrier, when the caller provides them,
// x comes from an earlier launch (not the tensor-parallel exchange) and is
// 16-byte aligned; else cp.async by every lane.
__device__ __forceinline__ bool gemv_x_bulk(const GemvArgs& a, const uint64_t* xbars) {
  return xbars && !a.tp.in && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
}
__device__ __forceinline__ void gemv_x_issue(const GemvArgs& a, const XBuf& xb_, int warp, int lane,
                                             uint64_t* xbars = nullptr) {
  const uint32_t NB = a.k / 256;
  float4* xr = reinterpret_cast<float4*>(xb_.xq);  // raw x staged in the limb slots
  if (a.tp.in) {
    gemv_x_tp(a, xb_, warp, lane);
    return;
  }
  if (gemv_x_bulk(a, xbars)) {
    if (lane == 0) {
      const uint32_t nblk = NB > (uint32_t)warp ? (NB - (uint32_t)warp + GEMV_WARPS - 1) / GEMV_WARPS : 0u;
      mbar_arrive_expect_tx(&xbars[warp], nblk * 1024u);
      for (uint32_t kb = warp; kb < NB; kb += GEMV_WARPS) {
        bulk_g2s(&xr[65 * kb], a.x + 256 * (size_t)kb, 512, &xbars[warp]);
        bulk_g2s(&xr[65 * kb + 33], a.x + 256 * (size_t)kb + 128, 512, &xbars[warp]);
      }
    }
    GEMV_STAMP(0);
    return;
  }
  const bool xal = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
#pragma unroll 1
  for (uint32_t kb = warp; kb < NB; kb += GEMV_WARPS) {
    const uint32_t v0 = 64 * kb + 2 * lane;
    const float* src = a.x + 256 * (size_t)kb + 8 * lane;
    if (xal) {
      cp_async16(&xr[xpad(v0)], src);
      cp_async16(&xr[xpad(v0 + 1)], src + 4);
    } else {
      xr[xpad(v0)] = make_float4(__ldcg(src), __ldcg(src + 1), __ldcg(src + 2), __ldcg(src + 3));
      xr[xpad(v0 + 1)] = make_float4(__ldcg(src + 4), __ldcg(src + 5), __ldcg(src + 6), __ldcg(src + 7));
    }
  }
  GEMV_STAMP(0);
}

// The rest: wait for the copies, RMSNorm scale, conversion.  x_issued: step 1
// already ran (else it runs here).
// RMSNorm weights of the blocks a consumer lane converts in the prologue's
// first iteration, loaded before the wait for the previous kernel (they do
// not depend on it): their global-memory latency leaves the critical path.
constexpr int GEMV_PU = 4;  // blocks per conversion iteration
struct NormPre {
  float4 w[GEMV_PU][2];
};
__device__ __forceinline__ void gemv_norm_prefetch(const GemvArgs& a, int warp, int lane, NormPre& np) {
  if (!a.norm_w) return;
  const uint32_t NB = a.k / 256;
#pragma unroll
  for (int u = 0; u < GEMV_PU; ++u) {
    const uint32_t kb = warp + u * GEMV_WARPS;
    np.w[u][0] = np.w[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);  // slots past the row: unused
    if (kb < NB) {
      const float4* wn = reinterpret_cast<const float4*>(a.norm_w + 256 * (size_t)kb + 8 * lane);
      np.w[u][0] = __ldg(wn);
      np.w[u][1] = __ldg(wn + 1);
    }
  }
}

template <bool HAS4, bool HAS6>
__device__ __forceinline__ float gemv_prologue(const GemvArgs& a, const XBuf& xb_, float* red,
                                              int warp, int lane, uint64_t* xready = nullptr,
                                              bool x_issued = false, const NormPre* np = nullptr,
                                              uint64_t* xbars = nullptr) {
  constexpr int CT = 32 * GEMV_WARPS;
  const uint32_t K = a.k;
  const uint32_t NB = K / 256;
  int4* xq = xb_.xq;
  float* xbs = xb_.xbs;
  float* xs32 = xb_.xs32;
  float4* xr = reinterpret_cast<float4*>(xq);
  if (!x_issued) gemv_x_issue(a, xb_, warp, lane, xbars);
  if (gemv_x_bulk(a, xbars)) {
    // on a time-out the error is recorded and the prologue still runs to its
    // barrier (every consumer warp must reach it); the launch's result is void
    mbar_wait_bounded(&xbars[warp], 0, a.err, DERR_TIMEOUT_FULL);
  } else {
    cp_async_wait_all();
  }
  __syncwarp();
  GEMV_STAMP(1);
  if (GEMV_XREADY_AT == 0 && xready && lane == 0) mbar_arrive(xready);

  // RMSNorm (engine/src/ops.c:195-214) is applied as a scale on the outputs:
  // W (x * inv_rms * w) = inv_rms * W (x * w), so the limbs are made from
  // x * w right away and the sum of squares is reduced alongside (same
  // per-lane order and fixed warp order as a separate pass: every CTA gets
  // the same scale), without a barrier between the two.
  const float* nw = a.norm_w;
  float ss = 0.f;
  GEMV_STAMP(2);
  // Conversion, PU blocks per iteration: independent dependency chains in
  // flight (a single block's chain -- reductions, shuffles, packing -- is long).
  constexpr int PU = GEMV_PU;
  // every block's norm weights are already in registers when one iteration
  // covers the row (K <= 256 * PU * GEMV_WARPS): no global load at all then
  const bool np_all = np && NB <= (uint32_t)(PU * GEMV_WARPS);
#pragma unroll 1
  for (uint32_t kb0 = warp; kb0 < NB; kb0 += PU * GEMV_WARPS) {
    // slots of this iteration that hold a block (warp-uniform): short rows
    // (K = 4096: one block per warp) skip the work of the empty slots
    const uint32_t nu = min((uint32_t)PU, (NB - kb0 + GEMV_WARPS - 1) / GEMV_WARPS);
    float v[PU][8];
#pragma unroll
    for (int u = 0; u < PU; ++u) {
      if ((uint32_t)u >= nu) break;
      const uint32_t v0 = 64 * (kb0 + u * GEMV_WARPS) + 2 * lane;
      const float4 t0 = xr[xpad(v0)], t1 = xr[xpad(v0 + 1)];
      v[u][0] = t0.x; v[u][1] = t0.y; v[u][2] = t0.z; v[u][3] = t0.w;
      v[u][4] = t1.x; v[u][5] = t1.y; v[u][6] = t1.z; v[u][7] = t1.w;
      if (nw) {
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[u][e], v[u][e], ss);
      }
    }
    if (nw) {
#pragma unroll
      for (int u = 0; u < PU; ++u) {
        if ((uint32_t)u >= nu) break;
        float4 w0, w1;
        if (np_all) {
          w0 = np->w[u][0];
          w1 = np->w[u][1];
        } else {
          const float4* wn = reinterpret_cast<const float4*>(nw + 256 * (size_t)(kb0 + u * GEMV_WARPS) + 8 * lane);
          w0 = __ldg(wn);
          w1 = __ldg(wn + 1);
        }
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[u][e] *= w[e];
      }
    }
    float amax[PU];
    bool finite[PU];
#pragma unroll
    for (int u = 0; u < PU; ++u) {
      if ((uint32_t)u >= nu) break;
      amax[u] = 0.f;
      finite[u] = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        amax[u] = fmaxf(amax[u], fabsf(v[u][e]));
        finite[u] = finite[u] && isfinite(v[u][e]);
      }
      // warp maximum in one step: |x| >= 0, whose bit patterns order as
      // unsigned integers (non-finite blocks are caught by `finite` below)
      amax[u] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax[u])));
    }
#pragma unroll
    for (int u = 0; u < PU; ++u) {
      const uint32_t kb = kb0 + u * GEMV_WARPS;
      if ((uint32_t)u >= nu) break;  // uniform across the warp
      const bool fin = __all_sync(0xffffffffu, finite[u]);
      // X_b = 2^(f-21) with amax in [2^f, 2^(f+1)): |x / X_b| < 2^22.  Blocks
      // whose maximum is below 2^-104 (subnormal maxima included) are scaled as
      // if it were 2^-104.  f from the exponent bits; the powers of two are
      // built from bits (f - 21 and 21 - f stay within the normal range).
      const int e8 = (int)((__float_as_uint(amax[u]) >> 23) & 0xFFu);
      const int f = amax[u] > 0.f ? max(e8 - 127, -104) : 0;
      const float xbv = fin ? __uint_as_float((uint32_t)(f - 21 + 127) << 23) : __int_as_float(0x7fc00000);
      const float inv_xb = __uint_as_float((uint32_t)(21 - f + 127) << 23);
      if (lane == 0) xbs[kb] = xbv;
      int t[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) t[e] = fin ? __float2int_rn(v[u][e] * inv_xb) : 0;
      uint32_t lw[2][3];  // [vector][limb]: limb k of 4 elements = byte k of each
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const uint32_t sel = (uint32_t)k | ((uint32_t)(k + 4) << 4);
          const uint32_t lo = __byte_perm((uint32_t)t[4 * h], (uint32_t)t[4 * h + 1], sel);
          const uint32_t hi = __byte_perm((uint32_t)t[4 * h + 2], (uint32_t)t[4 * h + 3], sel);
          lw[h][k] = __byte_perm(lo, hi, 0x5410);
        }
      // Q6_K: -32 * (sum of limb k over each 16-element group, lanes 2m and
      // 2m+1) rides in the fourth word of the group's vector k (k < 3), where
      // the dot-product loop adds it to its limb-k accumulators
      int w3[2] = {0, 0};
      if (HAS6) {
        int l0 = (int)__dp4a(lw[0][0], 0x01010101u, __dp4a(lw[1][0], 0x01010101u, 0u));
        int l1 = (int)__dp4a(lw[0][1], 0x01010101u, __dp4a(lw[1][1], 0x01010101u, 0u));
        int l2 = __dp4a((int)lw[0][2], 0x01010101, __dp4a((int)lw[1][2], 0x01010101, 0));
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l2 += __shfl_xor_sync(0xffffffffu, l2, 1);
        w3[0] = (lane & 1) ? -32 * l2 : -32 * l0;
        w3[1] = (lane & 1) ? 0 : -32 * l1;
      }
      const uint32_t v0 = 64 * kb + 2 * lane;
      xq[xpad(v0)] = make_int4((int)lw[0][0], (int)lw[0][1], (int)lw[0][2], w3[0]);
      xq[xpad(v0 + 1)] = make_int4((int)lw[1][0], (int)lw[1][1], (int)lw[1][2], w3[1]);
      if (HAS4) {  // fp32 sums of x per 32-element sub-block (4 lanes)
        float sm = ((v[u][0] + v[u][1]) + (v[u][2] + v[u][3])) + ((v[u][4] + v[u][5]) + (v[u][6] + v[u][7]));
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        if ((lane & 3) == 0) xs32[8 * kb + (lane >> 2)] = sm;
      }
    }
  }
  if (nw) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
  }
  GEMV_STAMP(3);
  if (GEMV_XREADY_AT == 1 && xready && lane == 0) mbar_arrive(xready);
  named_sync(1, CT);
  if (!nw) return 1.0f;
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < GEMV_WARPS; ++w) tot += red[w];
  return 1.0f / sqrtf(tot / (float)K + 1e-5f);
}

// Consumers: walk this CTA's chunks of plan `a` in the producer's order; a
// warp waits only for chunks that hold one of its tasks, and the last warp to
// finish a chunk's tasks releases the stage.  False if a bounded wait ran out.
template <bool HAS4, bool HAS6>
__device__ __forceinline__ bool gemv_consume(const GemvArgs& a, const Ring& R, RingPos& p,
                                             uint32_t& gtask, uint64_t lo, uint64_t hi,
                                             const XView& xv, int warp, int lane) {
  uint64_t seg_off = 0;
  for (uint32_t s = 0; s < a.nseg; ++s) {
    const GemvSeg& g = a.seg[s];
    const Range rr = seg_units(a, s, seg_off, lo, hi);
    const uint32_t lg_ur = __ffs((uint32_t)g.rg * g.rl) - 1, ur = 1u << lg_ur;
    const uint32_t cu = g.chunk_rows >> lg_ur;
    for (uint32_t u = rr.ub; u < rr.ue; u += cu) {
      const uint32_t r0 = u << lg_ur;
      const uint32_t r1 = min(min(u + cu, rr.ue) << lg_ur, g.m);
      const uint32_t nrows = r1 - r0;
      const uint32_t ks = g.ks;
      const uint32_t ntasks = ((nrows + ur - 1) >> lg_ur) * ks;
      uint32_t t = (uint32_t)(warp - (int)(gtask % GEMV_WARPS) + GEMV_WARPS) % GEMV_WARPS;
      if (t < ntasks) {
        if (!wait_gen(R.gen, p.st, p.it, a.err)) return false;
        if (!mbar_wait_bounded(&R.full[p.st], p.ph, a.err, DERR_TIMEOUT_FULL)) return false;
        const uint8_t* buf = R.stages + (size_t)p.st * R.stage_bytes;
        const uint32_t dual_off = nrows * g.row_stride;
        uint32_t mine = 0;
        for (; t < ntasks; t += GEMV_WARPS, ++mine) {
          const uint32_t rt = t >> g.lg_ks, sl = t & (ks - 1);
          const int rv = (int)min(ur, nrows - (rt << lg_ur));
          const uint8_t* rows = buf + (size_t)(rt << lg_ur) * g.row_stride;
          const uint32_t ki = p.st * GEMV_KS_ROWT + (rt < GEMV_KS_ROWT ? rt : 0);
          run_task<HAS4, HAS6>(a, g, rows, r0 + (rt << lg_ur), rv, dual_off, xv, lane, sl,
                               R.kpart + ki * (2 * GEMV_KS_MAX), R.kcnt + ki);
        }
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          const int prev = atomicAdd(&R.done[p.st], (int)mine);
          if (prev + (int)mine == (int)ntasks) {
            R.done[p.st] = 0;
            mbar_arrive(&R.empty[p.st]);
          }
        }
      }
      gtask += ntasks;
      p.advance(R.ns);
    }
    seg_off += (uint64_t)((g.m + ur - 1) >> lg_ur) * g.unit_cost;
  }
  return true;
}

}  // namespace gdev
}  // namespace shk
