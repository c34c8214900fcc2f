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
//  * warp 8 is the producer: one lane streams whole-row chunks of the weight
//    matrix into a shared-memory ring with cp.async.bulk (TMA, 1-D, no tensor
//    map, no multicast), completion tracked by mbarrier tx-counts; a per-stage
//    generation tag orders consumers that skip ahead;
//  * warps 0-7 are consumers: they load x (RMSNorm fused) and turn it into the
//    fixed-point form below while the first chunks are in flight, then decode
//    blocks from the ring.  The last warp to finish a chunk's tasks releases
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
// d * X_b.  The Q4_K min term uses fp32 sums of x; the Q6_K -32 offset is folded
// into the dp4a accumulators' initial value.  Integer packing keeps the
// per-weight work on the dp4a/IMAD path instead of the half-rate logic pipe.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"

namespace shk {
namespace gdev {

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// x limbs live in shared memory as int4 vectors {l0 word, l1 word, l2 word, 0}
// (4 elements each).  Vector v is stored at v + v/64: one pad vector after
// every 256-element block.  A block's 64 vectors are then contiguous (lanes use
// constant offsets), and lanes reading the same offset in consecutive blocks
// land in distinct bank groups.
__device__ __forceinline__ uint32_t xpad(uint32_t v) { return v + (v >> 6); }

// Limbs 0 and 1 of x are unsigned bytes, limb 2 is a signed byte (see the
// prologue); quants are unsigned and below 64, so limb 2 may use the signed form.
__device__ __forceinline__ int dp4a_u(uint32_t a, int b, int c) {
  return (int)__dp4a(a, (uint32_t)b, (uint32_t)c);
}
__device__ __forceinline__ int dp4a_s(uint32_t a, int b, int c) { return __dp4a((int)a, b, c); }

__device__ __forceinline__ float limbs_to_float(int a0, int a1, int a2) {
  return fmaf(65536.0f, (float)a2, fmaf(256.0f, (float)a1, (float)a0));
}

// ------------------------------- Q4_K ---------------------------------------
// A lane owns whole blocks b (all 256 elements) for RL rows (and both matrices
// of a dual segment), so each row's scale/min decode and block epilogue is paid
// once per 256 weights.  The four 64-element groups j are walked in a rolled
// loop (compact code); within a group the low nibbles are sub-block 2j and the
// high nibbles sub-block 2j+1 (engine/src/ops.c:117-142).
template <int RL, bool DUAL>
__device__ __forceinline__ void q4k_block_rows(const uint8_t* const (&rp)[RL * (DUAL ? 2 : 1)],
                                               uint32_t boff, const int4* __restrict__ xblk,
                                               float xb, const float* __restrict__ xs,
                                               float (&acc)[RL][2]) {
  constexpr int NR = RL * (DUAL ? 2 : 1);
  uint32_t scl[NR], sch[NR], ml[NR], mh[NR];
  float dx[NR], dm[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const uint4 h = *reinterpret_cast<const uint4*>(rp[r] + boff);
    // 6-bit scales/mins of sub-blocks 0-3 and 4-7, packed four per word
    // (engine/src/ops.c:107-115 get_scale_min_k4)
    scl[r] = h.y & 0x3F3F3F3Fu;
    ml[r] = h.z & 0x3F3F3F3Fu;
    sch[r] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    mh[r] = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    dx[r] = ref_half(h.x & 0xFFFFu) * xb;
    dm[r] = ref_half(h.x >> 16);
  }
  int A[NR][3];
  float M[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    A[r][0] = A[r][1] = A[r][2] = 0;
    M[r] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int S[NR][2][3];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) S[r][hh][0] = S[r][hh][1] = S[r][hh][2] = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // qs words 4*half .. 4*half+3
      uint4 w[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r)
        w[r] = *reinterpret_cast<const uint4*>(rp[r] + boff + 16 + 32 * j + 16 * half);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int4 xl = xblk[16 * j + 4 * half + i];
        const int4 xh = xblk[16 * j + 8 + 4 * half + i];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          const uint32_t q = i == 0 ? w[r].x : i == 1 ? w[r].y : i == 2 ? w[r].z : w[r].w;
          const uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;
          S[r][0][0] = dp4a_u(lo, xl.x, S[r][0][0]);
          S[r][0][1] = dp4a_u(lo, xl.y, S[r][0][1]);
          S[r][0][2] = dp4a_s(lo, xl.z, S[r][0][2]);
          S[r][1][0] = dp4a_u(hi, xh.x, S[r][1][0]);
          S[r][1][1] = dp4a_u(hi, xh.y, S[r][1][1]);
          S[r][1][2] = dp4a_s(hi, xh.z, S[r][1][2]);
        }
      }
    }
    const float2 xsum = *reinterpret_cast<const float2*>(xs + 2 * j);
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const uint32_t scw = j < 2 ? scl[r] : sch[r], mw = j < 2 ? ml[r] : mh[r];
      // bytes 2(j&1), 2(j&1)+1 of the packed words: sub-blocks 2j, 2j+1
      const int sc0 = (int)__byte_perm(scw, 0u, 0x4440 + 2 * (j & 1));
      const int sc1 = (int)__byte_perm(scw, 0u, 0x4441 + 2 * (j & 1));
      const int m0 = (int)__byte_perm(mw, 0u, 0x4440 + 2 * (j & 1));
      const int m1 = (int)__byte_perm(mw, 0u, 0x4441 + 2 * (j & 1));
      A[r][0] += sc0 * S[r][0][0] + sc1 * S[r][1][0];
      A[r][1] += sc0 * S[r][0][1] + sc1 * S[r][1][1];
      A[r][2] += sc0 * S[r][0][2] + sc1 * S[r][1][2];
      M[r] = fmaf((float)m0, xsum.x, fmaf((float)m1, xsum.y, M[r]));
    }
  }
#pragma unroll
  for (int r = 0; r < NR; ++r)
    acc[r % RL][r / RL] += fmaf(dx[r], limbs_to_float(A[r][0], A[r][1], A[r][2]), -(dm[r] * M[r]));
}

template <int RL, bool DUAL>
__device__ __forceinline__ void q4k_task(const uint8_t* __restrict__ rows, uint32_t row_stride,
                                         uint32_t nb, int rows_valid, uint32_t dual_off,
                                         const int4* __restrict__ xq, const float* __restrict__ xbs,
                                         const float* __restrict__ xs32, int lane, int lg_rg,
                                         float (&acc)[RL][2]) {
  constexpr int NR = RL * (DUAL ? 2 : 1);
  const int SPR = 32 >> lg_rg;  // block slots (lanes) per row group
  const int g = lane >> (5 - lg_rg), s = lane & (SPR - 1);
#pragma unroll
  for (int r = 0; r < RL; ++r) acc[r][0] = acc[r][1] = 0.f;
  if (g * RL < rows_valid) {
    // Rows past rows_valid read stale (in-bounds) stage bytes; their results
    // are never stored.
    const uint8_t* rp[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r)
      rp[r] = rows + (size_t)(g * RL + (r % RL)) * row_stride + (r >= RL ? dual_off : 0);
    for (uint32_t b = s; b < nb; b += SPR)
      q4k_block_rows<RL, DUAL>(rp, b * Q4K_BYTES, xq + 65 * b, xbs[b], xs32 + 8 * b, acc);
  }
  for (int o = 16 >> lg_rg; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < RL; ++r) {
      acc[r][0] += __shfl_xor_sync(0xffffffffu, acc[r][0], o);
      if (DUAL) acc[r][1] += __shfl_xor_sync(0xffffffffu, acc[r][1], o);
    }
}

// ------------------------------- Q6_K ---------------------------------------
// Blocks are 210 bytes: inside a 16-byte-aligned row, block b starts at an
// address == 2*b (mod 4).  Lanes of a warp always work on blocks of the same
// parity P, so every field is either word aligned (P = 0) or two bytes past a
// word (P = 1); P is a template constant and fields are read as 32-bit words.
template <int P, int NW>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&o)[NW]) {
  if (P == 0) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
#pragma unroll
    for (int i = 0; i < NW; ++i) o[i] = q[i];
  } else {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - 2);
    uint32_t prev = q[0];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const uint32_t nx = q[i + 1];
      o[i] = __byte_perm(prev, nx, 0x5432);
      prev = nx;
    }
  }
}

// One lane handles half n (128 elements) of a Q6_K block for RL rows
// (engine/src/ops.c:167-193 dequantize_row_q6_k).  For each 32-bit word i of
// ql/qh, four words of exact 6-bit quants are formed (element groups +0, +32,
// +64, +96) and fed to dp4a.  Each 16-element scale group's three limb sums
// start at -32 * (sum of x limbs), which applies the -32 offset.
template <int P, int RL>
__device__ __forceinline__ void q6k_block_rows(const uint8_t* __restrict__ blk, uint32_t row_stride,
                                               int n, const int4* __restrict__ xq, uint32_t b,
                                               const int4* __restrict__ xi, float xb,
                                               float (&acc)[RL]) {
  const uint32_t M = 0x0F0F0F0Fu;
  const int4* xh = xq + 65 * b + 32 * n;  // this half's 32 vectors; group g at +8g
  uint32_t A[RL][8], B[RL][8], H[RL][8], SC[RL][2];
  float dd[RL];
#pragma unroll
  for (int r = 0; r < RL; ++r) {
    const uint8_t* p = blk + (size_t)r * row_stride;
    load_words<P, 8>(p + 64 * n, A[r]);
    load_words<P, 8>(p + 64 * n + 32, B[r]);
    load_words<P, 8>(p + 128 + 32 * n, H[r]);
    load_words<P, 2>(p + 192 + 8 * n, SC[r]);
    dd[r] = ref_half(*reinterpret_cast<const uint16_t*>(p + 208)) * xb;
  }
  int T[RL][3];
#pragma unroll
  for (int r = 0; r < RL; ++r) T[r][0] = T[r][1] = T[r][2] = 0;
#pragma unroll
  for (int is = 0; is < 2; ++is) {
    int S[RL][4][3];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int4 init = xi[2 * g + is];  // -32 * limb sums of this 16-group
#pragma unroll
      for (int r = 0; r < RL; ++r) {
        S[r][g][0] = init.x;
        S[r][g][1] = init.y;
        S[r][g][2] = init.z;
      }
    }
#pragma unroll
    for (int i = 4 * is; i < 4 * is + 4; ++i) {
      int4 xv[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) xv[g] = xh[8 * g + i];
#pragma unroll
      for (int r = 0; r < RL; ++r) {
        const uint32_t h = H[r][i];
        const uint32_t hm = h & 0x33333333u, hn = h & 0xCCCCCCCCu;
        const uint32_t Q[4] = {lop_sel(A[r][i], hm << 4, M), lop_sel(B[r][i], hn << 2, M),
                               lop_sel(A[r][i] >> 4, hm, M), lop_sel(B[r][i] >> 4, hn >> 2, M)};
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          S[r][g][0] = dp4a_u(Q[g], xv[g].x, S[r][g][0]);
          S[r][g][1] = dp4a_u(Q[g], xv[g].y, S[r][g][1]);
          S[r][g][2] = dp4a_s(Q[g], xv[g].z, S[r][g][2]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RL; ++r)
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int si = is + 2 * g;  // scale index within this half
        const int sc = (int)(int8_t)__byte_perm(SC[r][si >> 2], 0u, 0x4440 + (si & 3));
        T[r][0] += sc * S[r][g][0];
        T[r][1] += sc * S[r][g][1];
        T[r][2] += sc * S[r][g][2];
      }
  }
#pragma unroll
  for (int r = 0; r < RL; ++r) acc[r] = fmaf(dd[r], limbs_to_float(T[r][0], T[r][1], T[r][2]), acc[r]);
}

template <int P, int RL>
__device__ __forceinline__ void q6k_class(const uint8_t* __restrict__ row, uint32_t row_stride,
                                          uint32_t nb, int s, int spr, int n,
                                          const int4* __restrict__ xq, const int4* __restrict__ xi16,
                                          const float* __restrict__ xbs, float (&acc)[RL]) {
  if (nb <= (uint32_t)P) return;
  const uint32_t nbc = (nb - P + 1) / 2;
  for (uint32_t t = s; t < nbc; t += spr) {
    const uint32_t b = P + 2 * t;
    q6k_block_rows<P, RL>(row + (size_t)b * Q6K_BYTES, row_stride, n, xq, b, xi16 + b * 16 + 8 * n,
                          xbs[b], acc);
  }
}

template <int RL>
__device__ __forceinline__ void q6k_rows(const uint8_t* __restrict__ row, uint32_t row_stride,
                                         uint32_t nb, int s, int spr, int n, const int4* xq,
                                         const int4* xi16, const float* xbs, float (&acc)[RL]) {
  q6k_class<0, RL>(row, row_stride, nb, s, spr, n, xq, xi16, xbs, acc);
  q6k_class<1, RL>(row, row_stride, nb, s, spr, n, xq, xi16, xbs, acc);
}

template <int RL, bool DUAL>
__device__ __forceinline__ void q6k_task(const uint8_t* __restrict__ rows, uint32_t row_stride,
                                         uint32_t nb, int rows_valid, uint32_t dual_off,
                                         const int4* __restrict__ xq, const float* __restrict__ xbs,
                                         const int4* __restrict__ xi16, int lane, int lg_rg,
                                         float (&acc)[RL][2]) {
  const int SPR = 16 >> lg_rg;
  const int slot = lane >> 1, n = lane & 1;
  const int g = slot >> (4 - lg_rg), s = slot & (SPR - 1);
  float a0[RL], a1[RL];
#pragma unroll
  for (int r = 0; r < RL; ++r) a0[r] = a1[r] = 0.f;
  if (g * RL < rows_valid) {
    const uint8_t* row = rows + (size_t)(g * RL) * row_stride;
    q6k_rows<RL>(row, row_stride, nb, s, SPR, n, xq, xi16, xbs, a0);
    if (DUAL) q6k_rows<RL>(row + dual_off, row_stride, nb, s, SPR, n, xq, xi16, xbs, a1);
  }
  for (int o = 16 >> lg_rg; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < RL; ++r) {
      a0[r] += __shfl_xor_sync(0xffffffffu, a0[r], o);
      if (DUAL) a1[r] += __shfl_xor_sync(0xffffffffu, a1[r], o);
    }
#pragma unroll
  for (int r = 0; r < RL; ++r) {
    acc[r][0] = a0[r];
    acc[r][1] = a1[r];
  }
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

template <int RL>
__device__ __forceinline__ void store_rows(const GemvArgs& a, const GemvSeg& g, uint32_t row0,
                                           int nvalid, const float (&acc)[RL][2]) {
  if (g.epi == EPI_ROPE) {
    // (2i, 2i+1) pairs are adjacent rows of this lane (RL even, row0 even)
    const float p = (float)__ldcg(a.pos);
#pragma unroll
    for (int r = 0; r + 1 < RL; r += 2) {
      if (r + 1 >= nvalid) break;
      const uint32_t row = row0 + r;
      const uint32_t i = row % g.rope_hd;
      // angle = pos * freq in fp32 as engine/src/ops.c:227-228; freq comes from
      // a table built with the host libm powf, so the angle matches bit for bit
      const float ang = p * a.rope_freq[i >> 1];
      const float c = cosf(ang), sn = sinf(ang);
      const float x0 = acc[r][0], x1 = acc[r + 1][0];
      g.y[row] = x0 * c - x1 * sn;
      g.y[row + 1] = x0 * sn + x1 * c;
    }
    return;
  }
#pragma unroll
  for (int r = 0; r < RL; ++r) {
    if (r >= nvalid) break;
    const uint32_t row = row0 + r;
    if (g.epi == EPI_STORE) {
      g.y[row] = acc[r][0];
    } else if (g.epi == EPI_ADD) {
      g.y[row] = __ldcg(&g.y[row]) + acc[r][0];
    } else {  // EPI_SWIGLU: silu(gate) * up
      const float gt = acc[r][0];
      const float sig = 1.0f / (1.0f + expf(-gt));
      g.y[row] = (gt * sig) * acc[r][1];
    }
  }
}

struct XView {
  const int4* xq;     // swizzled limb vectors, K/4
  const float* xbs;   // per-256-block scale X_b, K/256
  const float* xs32;  // Q4_K: fp32 sums of x per 32-element sub-block, K/32
  const int4* xi16;   // Q6_K: -32 * limb sums per 16-element group, K/16
};

template <int QT, int RL, bool DUAL>
__device__ __forceinline__ void task_and_store(const GemvArgs& a, const GemvSeg& g,
                                               const uint8_t* rows, uint32_t row0, int rows_valid,
                                               uint32_t dual_off, const XView& x, int lane) {
  const int lg_rg = __ffs(g.rg) - 1;
  float acc[RL][2];
  if (QT == T_Q4K)
    q4k_task<RL, DUAL>(rows, g.row_stride, g.nb, rows_valid, dual_off, x.xq, x.xbs, x.xs32, lane,
                       lg_rg, acc);
  else
    q6k_task<RL, DUAL>(rows, g.row_stride, g.nb, rows_valid, dual_off, x.xq, x.xbs, x.xi16, lane,
                       lg_rg, acc);
  const int lpg = 32 >> lg_rg;  // lanes per row group
  const int grp = lane >> (5 - lg_rg);
  if ((lane & (lpg - 1)) == 0 && grp * RL < rows_valid)
    store_rows<RL>(a, g, row0 + grp * RL, rows_valid - grp * RL, acc);
}

// (qt, dual, rl) -> instantiation; the planner only picks these.
__device__ __forceinline__ void dispatch_task(const GemvArgs& a, const GemvSeg& g,
                                              const uint8_t* rows, uint32_t row0, int rv,
                                              uint32_t dual_off, const XView& x, int lane) {
#define SHK_TASK(QT, RL, DU)                                            \
  task_and_store<QT, RL, DU>(a, g, rows, row0, rv, dual_off, x, lane); \
  return
  const int key = (g.qt == T_Q4K ? 0 : 100) + (g.dual ? 10 : 0) + g.rl;
  switch (key) {
    case 4: SHK_TASK(T_Q4K, 4, false);
    case 2: SHK_TASK(T_Q4K, 2, false);
    case 1: SHK_TASK(T_Q4K, 1, false);
    case 12: SHK_TASK(T_Q4K, 2, true);
    case 11: SHK_TASK(T_Q4K, 1, true);
    case 102: SHK_TASK(T_Q6K, 2, false);
    case 101: SHK_TASK(T_Q6K, 1, false);
    case 111: SHK_TASK(T_Q6K, 1, true);
    default: return;
  }
#undef SHK_TASK
}

// Shared-memory map: [full | empty | xbar barriers][done][gen][red]
// [x raw / limb vectors (K*4)][X_b (K/256)][xs32 (K/32, Q4_K)][xi16 (K*1, Q6_K)]
// [stage ring].  The producer first bulk-copies x into the limb-vector slot;
// consumers turn it into limbs in place.
constexpr int SMEM_HDR = 8 * (2 * GEMV_MAX_STAGES + 1) + 8 * GEMV_MAX_STAGES + 4 * 32;

// Bounded spin until the producer has claimed stage `st` for chunk `it`.  A
// consumer may run several ring cycles ahead of a stage (it skips chunks with
// no task for it), so the mbarrier parity alone could name a stale phase; the
// tag makes the following parity wait refer to chunk `it` exactly.
__device__ __forceinline__ bool wait_gen(const volatile uint32_t* gen, uint32_t st, uint32_t it,
                                         int* err) {
  if (gen[st] == it) return true;
  const uint64_t t0 = globaltimer_ns();
  while (gen[st] != it) {
    if (globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
      set_error(err, DERR_TIMEOUT_FULL);
      return false;
    }
  }
  return true;
}

// X_b array padded to a 16-byte multiple so xs32 (float2 loads) and xi16
// (int4 loads) stay aligned for every K.
__host__ __device__ __forceinline__ uint32_t xbs_floats(uint32_t K) { return ((K / 256) + 3) & ~3u; }

__host__ __device__ __forceinline__ size_t xq_bytes(uint32_t K) {
  return (size_t)(K / 4 + K / 256) * 16;  // one pad vector per 64
}

__host__ __device__ __forceinline__ size_t x_region_bytes(uint32_t K, bool has4, bool has6) {
  size_t b = xq_bytes(K) + (size_t)xbs_floats(K) * 4;
  if (has4) b += (size_t)(K / 32) * 4;
  if (has6) b += (size_t)K;  // int4 per 16 elements
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

// Producer (one lane): streams this CTA's chunks of plan `a` (cost range
// [lo, hi)) into the ring.  False if a bounded wait ran out.
__device__ __forceinline__ bool gemv_produce(const GemvArgs& a, const Ring& R, RingPos& p,
                                             uint64_t lo, uint64_t hi) {
  uint64_t seg_off = 0;
  for (uint32_t s = 0; s < a.nseg; ++s) {
    const GemvSeg& g = a.seg[s];
    const Range rr = seg_units(a, s, seg_off, lo, hi);
    const uint32_t lg_ur = __ffs((uint32_t)g.rg * g.rl) - 1, cu = g.chunk_rows >> lg_ur;
    for (uint32_t u = rr.ub; u < rr.ue; u += cu) {
      const uint32_t r0 = u << lg_ur;
      const uint32_t r1 = min(min(u + cu, rr.ue) << lg_ur, g.m);
      const uint32_t bytes = (r1 - r0) * g.row_stride;
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
  int4* xi16;
  __device__ __forceinline__ XView view() const { return XView{xq, xbs, xs32, xi16}; }
};

// Consumers (warps 0..GEMV_WARPS-1): x (optionally RMSNorm'ed) -> fixed-point
// limb vectors in shared memory.  Ends with a consumer-only barrier.
template <bool HAS4, bool HAS6>
__device__ __forceinline__ void gemv_prologue(const GemvArgs& a, const XBuf& xb_, float* red,
                                              int warp, int lane) {
  constexpr int CT = 32 * GEMV_WARPS;
  constexpr int BPW = 4;  // 256-blocks per warp per pass (32 floats per lane)
  const uint32_t K = a.k;
  const uint32_t NB = K / 256;
  int4* xq = xb_.xq;
  float* xbs = xb_.xbs;
  float* xs32 = xb_.xs32;
  int4* xi16 = xb_.xi16;
  const bool xal = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  const bool wal = a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0;
  // Fixed-point conversion.  Warp w owns 256-blocks w, w+8, ...; lane l holds
  // elements 8l..8l+7 of a block (limb vectors 2l, 2l+1), so the block maximum
  // is a warp reduction.  A pass loads up to BPW blocks per warp before using
  // any of them.
  for (uint32_t pass = 0; pass * GEMV_WARPS * BPW < NB; ++pass) {
    float v[BPW][8];
#pragma unroll
    for (int u = 0; u < BPW; ++u) {
      const uint32_t kb = warp + GEMV_WARPS * (BPW * pass + u);
      const float* src = a.x + 256 * (size_t)(kb < NB ? kb : 0) + 8 * lane;
      if (xal) {
        const float4 t0 = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 t1 = __ldcg(reinterpret_cast<const float4*>(src) + 1);
        v[u][0] = t0.x; v[u][1] = t0.y; v[u][2] = t0.z; v[u][3] = t0.w;
        v[u][4] = t1.x; v[u][5] = t1.y; v[u][6] = t1.z; v[u][7] = t1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[u][e] = __ldcg(src + e);
      }
    }
    if (a.norm_w) {
      // RMSNorm prologue (engine/src/ops.c:195-214); the planner guarantees a
      // single pass, and the fixed-order reduction gives every CTA the same scale.
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < BPW; ++u)
        if (warp + GEMV_WARPS * u < NB)
#pragma unroll
          for (int e = 0; e < 8; ++e) ss = fmaf(v[u][e], v[u][e], ss);
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      named_sync(1, CT);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < GEMV_WARPS; ++w) tot += red[w];
      const float inv_rms = 1.0f / sqrtf(tot / (float)K + 1e-5f);
#pragma unroll
      for (int u = 0; u < BPW; ++u) {
        const uint32_t kb = warp + GEMV_WARPS * u;
        const float* wn = a.norm_w + 256 * (size_t)(kb < NB ? kb : 0) + 8 * lane;
        float w[8];
        if (wal) {
          const float4 t0 = __ldg(reinterpret_cast<const float4*>(wn));
          const float4 t1 = __ldg(reinterpret_cast<const float4*>(wn) + 1);
          w[0] = t0.x; w[1] = t0.y; w[2] = t0.z; w[3] = t0.w;
          w[4] = t1.x; w[5] = t1.y; w[6] = t1.z; w[7] = t1.w;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) w[e] = __ldg(wn + e);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[u][e] = (v[u][e] * inv_rms) * w[e];
      }
    }
#pragma unroll
    for (int u = 0; u < BPW; ++u) {
      const uint32_t kb = warp + GEMV_WARPS * (BPW * pass + u);
      if (kb >= NB) break;  // uniform across the warp
      float amax = 0.f;
      bool finite = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        amax = fmaxf(amax, fabsf(v[u][e]));
        finite = finite && isfinite(v[u][e]);
      }
      amax = warp_max(amax);
      finite = __all_sync(0xffffffffu, finite);
      // X_b = 2^(f-21) with amax in [2^f, 2^(f+1)): |x / X_b| < 2^22.  Blocks
      // whose maximum is below 2^-104 are scaled as if it were 2^-104.
      const int f = amax > 0.f ? max(ilogbf(amax), -104) : 0;
      const float xb = finite ? ldexpf(1.0f, f - 21) : __int_as_float(0x7fc00000);
      const float inv_xb = ldexpf(1.0f, 21 - f);
      if (lane == 0) xbs[kb] = xb;
      int t[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) t[e] = finite ? __float2int_rn(v[u][e] * inv_xb) : 0;
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
      const uint32_t v0 = 64 * kb + 2 * lane;
      xq[xpad(v0)] = make_int4((int)lw[0][0], (int)lw[0][1], (int)lw[0][2], 0);
      xq[xpad(v0 + 1)] = make_int4((int)lw[1][0], (int)lw[1][1], (int)lw[1][2], 0);
      if (HAS4) {  // fp32 sums of x per 32-element sub-block (4 lanes)
        float s = ((v[u][0] + v[u][1]) + (v[u][2] + v[u][3])) + ((v[u][4] + v[u][5]) + (v[u][6] + v[u][7]));
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) xs32[8 * kb + (lane >> 2)] = s;
      }
      if (HAS6) {  // -32 * limb sums per 16-element group (2 lanes)
        int l0 = (int)__dp4a(lw[0][0], 0x01010101u, __dp4a(lw[1][0], 0x01010101u, 0u));
        int l1 = (int)__dp4a(lw[0][1], 0x01010101u, __dp4a(lw[1][1], 0x01010101u, 0u));
        int l2 = __dp4a((int)lw[0][2], 0x01010101, __dp4a((int)lw[1][2], 0x01010101, 0));
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l2 += __shfl_xor_sync(0xffffffffu, l2, 1);
        if ((lane & 1) == 0) xi16[16 * kb + (lane >> 1)] = make_int4(-32 * l0, -32 * l1, -32 * l2, 0);
      }
    }
  }
  named_sync(1, CT);
}

// Consumers: walk this CTA's chunks of plan `a` in the producer's order; a
// warp waits only for chunks that hold one of its tasks, and the last warp to
// finish a chunk's tasks releases the stage.  False if a bounded wait ran out.
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
      const uint32_t ntasks = (nrows + ur - 1) >> lg_ur;
      uint32_t t = (uint32_t)(warp - (int)(gtask % GEMV_WARPS) + GEMV_WARPS) % GEMV_WARPS;
      if (t < ntasks) {
        if (!wait_gen(R.gen, p.st, p.it, a.err)) return false;
        if (!mbar_wait_bounded(&R.full[p.st], p.ph, a.err, DERR_TIMEOUT_FULL)) return false;
        const uint8_t* buf = R.stages + (size_t)p.st * R.stage_bytes;
        const uint32_t dual_off = nrows * g.row_stride;
        uint32_t mine = 0;
        for (; t < ntasks; t += GEMV_WARPS, ++mine) {
          const int rv = (int)min(ur, nrows - (t << lg_ur));
          const uint8_t* rows = buf + (size_t)(t << lg_ur) * g.row_stride;
          dispatch_task(a, g, rows, r0 + (t << lg_ur), rv, dual_off, xv, lane);
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
