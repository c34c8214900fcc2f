// attn_dev.cuh -- device side of the Q8_0 KV cache: bit-exact
// quantise-on-append and one (KV head, position split) item of split-K decode
// attention.  Used by the stand-alone attention kernel (attn.cu) and the
// persistent decode kernel (decode.cu).
//
// Reference semantics:
//  * q8_quantize_vec (engine/src/kv_cache.c:28-55): per 32 floats
//    scale = maxabs / 127 (0 -> 1), q = clamp(lrintf(v / scale), -127, 127).
//    The same IEEE division and round-half-even conversion are used, so
//    blocks are bit-identical for identical fp32 input.
//  * op_attention (engine/src/ops.c:406-461) over kv_cache_read_range output:
//    query head h reads KV head h % n_kv_heads, score = dot(q, k) * scale,
//    max-subtracted softmax, out = sum p * v.  Here the softmax is computed
//    online per position range (split) and merged with a log-sum-exp combine by
//    the last item of each KV head; results agree to fp32 rounding.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "attn.cuh"
#include "common.cuh"

namespace shk {
namespace adev {

// One warp quantises one 32-element block (lane = element).
__device__ __forceinline__ void q8_block_store(float v, int8_t* q_dst, float* s_dst, int lane) {
  // fmaxf with 0 first: a NaN lane counts as 0, as `a > max_abs` skips it in
  // the reference (an all-NaN block then has scale 1, not NaN)
  const float amax = warp_max(fmaxf(0.0f, fabsf(v)));
  float scale = amax / 127.0f;
  if (scale == 0.0f) scale = 1.0f;
  int q = __float2int_rn(v / scale);
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  q_dst[lane] = (int8_t)q;
  if (lane == 0) *s_dst = scale;
}

// Appends k_new/v_new of KV head `kvh` at position pos; called by nw warps.
__device__ __forceinline__ void append_head(const KvLayout& kv, uint32_t layer, uint32_t kvh,
                                            uint32_t pos, const float* k_new, const float* v_new,
                                            int warp, int lane, int nw) {
  const uint32_t nblk = kv.hd / 32;
  int8_t* reg = kv.region(layer, kvh);
  for (uint32_t b = warp; b < 2 * nblk; b += nw) {
    const bool isv = b >= nblk;
    const uint32_t j = isv ? b - nblk : b;
    const float v = __ldcg((isv ? v_new : k_new) + kvh * kv.hd + 32 * j + lane);
    int8_t* qd = reg + (isv ? kv.vq_off : kv.kq_off) + (size_t)pos * kv.hd + 32 * j;
    float* sd = reinterpret_cast<float*>(reg + (isv ? kv.vs_off : kv.ks_off)) + (size_t)pos * nblk + j;
    q8_block_store(v, qd, sd, lane);
  }
}

constexpr int ATT_MAX_SPLITS = 128;  // splits per KV head (the host caps max_splits at this)

// int8 lanes of a 32-bit word -> fp32, exactly: byte b + 128 placed in the
// low mantissa bits of 2^23 (one byte permute), minus 2^23 + 128 (one add) --
// full-rate ALU / FMA work instead of a conversion instruction per value.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;  // x + 128 in every byte
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// The loads of one warp iteration: PPI positions starting at T.
template <int HD>
struct AttnTile {
  static constexpr int LPP = HD / 32, PPI = 32 / LPP, EPL = HD / 32;
  uint4 k0, k1;         // this lane's 32-byte Q8_0 K block
  float ks;             // its scale
  uint32_t vw[PPI];     // V: this lane's EPL columns of each position
  float vs[PPI];        // their block scales
  __device__ __forceinline__ void load(const int8_t* Kq, const float* Ks, const int8_t* Vq,
                                       const float* Vs, uint32_t T, uint32_t p1, int lane) {
    const uint32_t nt = min((uint32_t)PPI, p1 - T);
    const uint32_t tl = lane / LPP, b = lane % LPP;
    const uint32_t t = T + (tl < nt ? tl : 0);  // clamp to a valid position
    const uint4* kp = reinterpret_cast<const uint4*>(Kq + (size_t)t * HD + 32 * b);
    k0 = __ldcg(kp);
    k1 = __ldcg(kp + 1);
    ks = __ldcg(Ks + (size_t)t * (HD / 32) + b);
#pragma unroll
    for (int j = 0; j < PPI; ++j) {
      const uint32_t tj = T + ((uint32_t)j < nt ? j : 0);
      const int8_t* vp = Vq + (size_t)tj * HD + lane * EPL;
      if (EPL == 4)
        vw[j] = __ldcg(reinterpret_cast<const unsigned int*>(vp));
      else
        vw[j] = __ldcg(reinterpret_cast<const unsigned short*>(vp));
      vs[j] = __ldcg(Vs + (size_t)tj * (HD / 32) + (lane * EPL) / 32);
    }
  }
};

// Shared memory of one attention item (floats): q rows padded to 36 so the
// LPP lanes of a position read distinct banks; per-warp partials; split weights.
template <int HD, int G, int NW>
struct AttnSmem {
  static constexpr int LPP = HD / 32;
  static constexpr int QROW = 36;
  static constexpr int Q = 0;
  static constexpr int WM = Q + G * LPP * QROW;
  static constexpr int WL = WM + NW * G;
  static constexpr int WACC = WL + NW * G;
  static constexpr int SW = WACC + NW * G * HD;
  static constexpr int SL = SW + ATT_MAX_SPLITS * G;
  static constexpr int FLAG = SL + G;
  static constexpr int FLOATS = FLAG + 4;
  static constexpr size_t BYTES = (size_t)FLOATS * 4;
  // the long-range loop's per-warp scratch (attn_item<..., LONG = true> only):
  // a transposed V tile of 16 positions, HD x 16 bytes
  static constexpr int PB = FLOATS;
  static constexpr int PB_WARP = HD * 4;
  static constexpr int FLOATS_LONG = PB + NW * PB_WARP;
};

__device__ __forceinline__ void att_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Long position ranges (at least ATT_LONG_MIN per CTA): a warp iteration
// covers 32 positions, one per lane.  QK^T: the lane loads its position's
// whole Q8_0 K row and forms all G scores (no shuffles); softmax: one warp
// maximum per query head per 32 positions, sums kept per lane until the end;
// PV: lane = EPL columns, the weights of the 32 positions broadcast through
// shared memory (pb: this warp's [G][32]), the V words of all 32 positions
// loaded at the start of the iteration.  The new K/V row (position pos) is
// already in the cache, stored by this CTA before the loop.
constexpr uint32_t ATT_LONG_MIN = 512;
// Split kernel: a split of at least this many positions runs the long loop.
#ifndef SHK_ATT_SPLIT_LONG
#define SHK_ATT_SPLIT_LONG 256
#endif
constexpr uint32_t ATT_SPLIT_LONG = SHK_ATT_SPLIT_LONG;

template <int HD, int G, int NW>
__device__ __forceinline__ void attn_long(const AttnArgs& a, const float* qsm, const int8_t* __restrict__ Kq,
                                          const float* __restrict__ Ks, const int8_t* __restrict__ Vq,
                                          const float* __restrict__ Vs, uint32_t p0, uint32_t p1, int warp,
                                          int lane, float* pb, float (&m)[G], float (&l)[G],
                                          float (&acc)[G][HD / 32]) {
  constexpr int NB = HD / 32, EPL = HD / 32, KV4 = HD / 16, QROW = 36;
  float lp[G];
#pragma unroll
  for (int g = 0; g < G; ++g) lp[g] = 0.f;
  for (uint32_t T = p0 + 32u * warp; T < p1; T += 32u * NW) {
    const uint32_t nt = min(32u, p1 - T);
    const bool valid = (uint32_t)lane < nt;
    const uint32_t t = T + (valid ? (uint32_t)lane : 0u);
    // every load of the iteration first
    uint4 kr[KV4];
    const uint4* kp = reinterpret_cast<const uint4*>(Kq + (size_t)t * HD);
#pragma unroll
    for (int i = 0; i < KV4; ++i) kr[i] = kp[i];
    float ksc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) ksc[b] = Ks[(size_t)t * NB + b];
    uint32_t vw[32];
    float vsc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint32_t tj = T + ((uint32_t)j < nt ? (uint32_t)j : 0u);
      const int8_t* vp = Vq + (size_t)tj * HD + lane * EPL;
      vw[j] = EPL == 4 ? *reinterpret_cast<const uint32_t*>(vp) : *reinterpret_cast<const uint16_t*>(vp);
      vsc[j] = Vs[(size_t)tj * NB + (lane * EPL) / 32];
    }
    // scores of this lane's position
    float sc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g] = 0.f;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float kf[32];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint4 w = kr[2 * b + i];
        s8x4_to_f32(w.x, kf + 16 * i);
        s8x4_to_f32(w.y, kf + 16 * i + 4);
        s8x4_to_f32(w.z, kf + 16 * i + 8);
        s8x4_to_f32(w.w, kf + 16 * i + 12);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4* q4 = reinterpret_cast<const float4*>(qsm + (g * NB + b) * QROW);
        float sb = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 qv = q4[u];
          sb = fmaf(qv.x, kf[4 * u], sb);
          sb = fmaf(qv.y, kf[4 * u + 1], sb);
          sb = fmaf(qv.z, kf[4 * u + 2], sb);
          sb = fmaf(qv.w, kf[4 * u + 3], sb);
        }
        sc[g] = fmaf(sb, ksc[b], sc[g]);
      }
    }
    // online softmax over these 32 positions
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sg = valid ? sc[g] * a.scale : -INFINITY;
      const float mn = fmaxf(m[g], warp_max(sg));  // at least position T is valid: finite
      const float corr = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
      const float p = valid ? expf(sg - mn) : 0.f;
      lp[g] = fmaf(lp[g], corr, p);
      m[g] = mn;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] *= corr;
      pb[g * 32 + lane] = p;
    }
    __syncwarp();
    // P.V
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if ((uint32_t)j >= nt) break;  // uniform
      float vf[4];
      s8x4_to_f32(vw[j], vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = pb[g * 32 + j] * vsc[j];
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(pj, vf[e], acc[g][e]);
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int g = 0; g < G; ++g) l[g] = warp_sum(lp[g]);
}


// --------------------- long ranges on the tensor cores -----------------------
// QK^T and PV of a 16-position chunk as mma.sync.m16n8k16 (f16 operands, fp32
// accumulators).  The int8 K and V quants are exact in f16; q is split into
// three f16 parts (high and middle in rows g and g + 8 of one A operand, low
// in rows g of a second: ~33 significant bits, so scores carry fp32-level
// error even when they are huge and the softmax is one-hot) and the softmax
// weights into two (rows g and g + 8: ~22 bits; their error enters the output
// linearly).  q is scaled by a power of two 2^-e (its largest magnitude below 1)
// and each chunk's weights p * v_scale by 1 / (the chunk's largest V scale of
// that block), so no f16 value overflows; both factors are put back in fp32.
//
// Lane layout (g = lane / 4, t = lane % 4): QK^T C-fragment columns 2t, 2t+1 of
// n-tile 0 / 1 are positions 4t, 4t+1 / 4t+2, 4t+3 of the chunk, exactly the
// k index pairs (2t, 2t+1), (2t+8, 2t+9) of the PV A fragment, so the
// softmax weights stay in the registers that computed them.  Head dims are
// permuted inside each 32-element block (k-steps 2j and 2j+1 take dims
// 32j + 8t + 0..3 and 32j + 8t + 4..7 for lane t) so a lane reads 8
// contiguous K bytes per block.  V is transposed into the warp's shared tile
// (4x4 byte transposes) so a lane reads the 4 positions of one dim as a word.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// int8 bytes (sel 0x4140: bytes 0, 1; 0x4342: bytes 2, 3) of u = w ^ 0x80808080
// -> f16x2, exactly: 0x64xx is 1024 + (x + 128), minus 1152.
__device__ __forceinline__ uint32_t s8x2_h2(uint32_t u, uint32_t sel) {
  const uint32_t h = __byte_perm(u, 0x64646464u, sel);
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
  return r;
}
__device__ __forceinline__ uint32_t h2_pack(float lo_col, float hi_col) {
  const __half2 h = __floats2half2_rn(lo_col, hi_col);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// x = hi + lo with hi, lo f16: returns hi, sets lo
__device__ __forceinline__ float split_f16(float x, float& lo) {
  const float hi = __half2float(__float2half_rn(x));
  lo = x - hi;
  return hi;
}

template <int HD, int G, int NW>
__device__ __forceinline__ void attn_long_tc(const AttnArgs& a, const float* qsm, const int8_t* __restrict__ Kq,
                                             const float* __restrict__ Ks, const int8_t* __restrict__ Vq,
                                             const float* __restrict__ Vs, uint32_t p0, uint32_t p1, int warp,
                                             int lane, uint8_t* vt, float* wm_w, float* wl_w, float* wacc_w) {
  constexpr int NB = HD / 32, KS = HD / 16, NT = HD / 8, QROW = 36;
  const int g = lane >> 2, t = lane & 3;
  const bool grow_ = g < G;
  // q -> two f16 parts (dims permuted as above), scaled by 2^-e
  float qmax = 0.f;
  if (grow_)
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) qmax = fmaxf(qmax, fabsf(qsm[(g * NB + j) * QROW + 8 * t + i]));
  qmax = warp_max(qmax);
  const int qe = (qmax > 0.f && isfinite(qmax)) ? ((int)((__float_as_uint(qmax) >> 23) & 0xFFu) - 126) : 0;
  const float qdown = ldexpf(1.0f, -qe), qup = ldexpf(1.0f, qe) * a.scale;
  uint32_t qa[KS][4], qb[KS][2];  // qb: the low part (rows g; rows g + 8 are zero)
#pragma unroll
  for (int j = 0; j < NB; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // k-step 2j + h: dims 32j + 8t + 4h + 0..3
      float v[4], hi[4], mid[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = grow_ ? qsm[(g * NB + j) * QROW + 8 * t + 4 * h + i] * qdown : 0.f;
        float r;
        hi[i] = split_f16(v[i], r);
        mid[i] = split_f16(r, lo[i]);
      }
      qa[2 * j + h][0] = h2_pack(hi[0], hi[1]);
      qa[2 * j + h][1] = h2_pack(mid[0], mid[1]);
      qa[2 * j + h][2] = h2_pack(hi[2], hi[3]);
      qa[2 * j + h][3] = h2_pack(mid[2], mid[3]);
      qb[2 * j + h][0] = h2_pack(lo[0], lo[1]);
      qb[2 * j + h][1] = h2_pack(lo[2], lo[3]);
    }
  float O[NT][2];
#pragma unroll
  for (int n = 0; n < NT; ++n) O[n][0] = O[n][1] = 0.f;
  float m = -INFINITY, lsum = 0.f;
  // the chunk row this lane loads for QK^T n-tile 0 (n-tile 1: +2)
  const uint32_t krow = (uint32_t)(g + 2 * (g >> 1));
  for (uint32_t T = p0 + 16u * warp; T < p1; T += 16u * NW) {
    // ---- loads: K rows (8 bytes of every block), scales, V 4x4 byte blocks
    uint2 kw[2][NB];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const uint32_t pos = T + krow + 2 * n;
      const uint32_t pc = pos < p1 ? pos : T;
#pragma unroll
      for (int j = 0; j < NB; ++j) kw[n][j] = __ldcg(reinterpret_cast<const uint2*>(Kq + (size_t)pc * HD + 32 * j + 8 * t));
    }
    float ksc[4][NB], vsc[4][NB];
    bool valid[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t pos = T + 4 * t + i;
      valid[i] = pos < p1;
      const uint32_t pc = valid[i] ? pos : T;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        ksc[i][j] = __ldcg(Ks + (size_t)pc * NB + j);
        vsc[i][j] = valid[i] ? __ldcg(Vs + (size_t)pc * NB + j) : 0.f;
      }
    }
    uint32_t vw[HD / 32][4];
#pragma unroll
    for (int k = 0; k < HD / 32; ++k) {  // block b = lane + 32k: rows 4(b%4).., cols 4(b/4)..
      const int b = lane + 32 * k, r4 = b & 3, c4 = b >> 2;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t pos = T + 4 * r4 + i;
        vw[k][i] = pos < p1 ? __ldcg(reinterpret_cast<const unsigned int*>(Vq + (size_t)pos * HD + 4 * c4)) : 0x00000000u;
      }
    }
    // ---- V^T into the warp's tile: word (dim d, positions 4r..4r+3) at d*16 + 4r
    __syncwarp();
#pragma unroll
    for (int k = 0; k < HD / 32; ++k) {
      const int b = lane + 32 * k, r4 = b & 3, c4 = b >> 2;
      const uint32_t x0 = __byte_perm(vw[k][0], vw[k][1], 0x5140), x1 = __byte_perm(vw[k][0], vw[k][1], 0x7362);
      const uint32_t y0 = __byte_perm(vw[k][2], vw[k][3], 0x5140), y1 = __byte_perm(vw[k][2], vw[k][3], 0x7362);
      uint32_t* dst = reinterpret_cast<uint32_t*>(vt);
      dst[(4 * c4 + 0) * 4 + r4] = __byte_perm(x0, y0, 0x5410);
      dst[(4 * c4 + 1) * 4 + r4] = __byte_perm(x0, y0, 0x7632);
      dst[(4 * c4 + 2) * 4 + r4] = __byte_perm(x1, y1, 0x5410);
      dst[(4 * c4 + 3) * 4 + r4] = __byte_perm(x1, y1, 0x7632);
    }
    // ---- QK^T: scores of positions 4t..4t+3 for head g
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        float c[4] = {0.f, 0.f, 0.f, 0.f}, d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t ux = kw[n][j].x ^ 0x80808080u, uy = kw[n][j].y ^ 0x80808080u;
        const uint32_t bx0 = s8x2_h2(ux, 0x4140), bx1 = s8x2_h2(ux, 0x4342);
        const uint32_t by0 = s8x2_h2(uy, 0x4140), by1 = s8x2_h2(uy, 0x4342);
        mma16816(c, qa[2 * j], bx0, bx1);
        mma16816(c, qa[2 * j + 1], by0, by1);
        const uint32_t l0[4] = {qb[2 * j][0], 0u, qb[2 * j][1], 0u}, l1[4] = {qb[2 * j + 1][0], 0u, qb[2 * j + 1][1], 0u};
        mma16816(d, l0, bx0, bx1);
        mma16816(d, l1, by0, by1);
        // high + middle (rows g, g + 8), then the low part (rows g)
        s[2 * n] = fmaf(ksc[2 * n][j], (c[0] + c[2]) + d[0], s[2 * n]);
        s[2 * n + 1] = fmaf(ksc[2 * n + 1][j], (c[1] + c[3]) + d[1], s[2 * n + 1]);
      }
    // ---- online softmax over the chunk (the quad holds the head's 16 positions)
    float cmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s[i] = valid[i] ? s[i] * qup : -INFINITY;
      cmax = fmaxf(cmax, s[i]);
    }
    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
    const float mn = fmaxf(m, cmax);  // position T is valid: finite
    const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = valid[i] ? expf(s[i] - mn) : 0.f;
    lsum = fmaf(lsum, corr, (p[0] + p[1]) + (p[2] + p[3]));
    m = mn;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      O[n][0] *= corr;
      O[n][1] *= corr;
    }
    __syncwarp();  // the V^T tile is complete
    // ---- PV, one 32-dim V block (4 n-tiles) at a time
    const uint32_t* vtw = reinterpret_cast<const uint32_t*>(vt);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      float vmax = fmaxf(fmaxf(vsc[0][j], vsc[1][j]), fmaxf(vsc[2][j], vsc[3][j]));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
      const float inv = vmax > 0.f ? 1.0f / vmax : 0.f;
      float hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) hi[i] = split_f16(p[i] * (vsc[i][j] * inv), lo[i]);
      const uint32_t pa[4] = {h2_pack(hi[0], hi[1]), h2_pack(lo[0], lo[1]), h2_pack(hi[2], hi[3]),
                              h2_pack(lo[2], lo[3])};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int n = 4 * j + q;
        const uint32_t u = vtw[(8 * n + g) * 4 + t] ^ 0x80808080u;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(c, pa, s8x2_h2(u, 0x4140), s8x2_h2(u, 0x4342));
        O[n][0] = fmaf(vmax, c[0] + c[2], O[n][0]);
        O[n][1] = fmaf(vmax, c[1] + c[3], O[n][1]);
      }
    }
  }
  __syncwarp();
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
  if (grow_) {
    if (t == 0) {
      wm_w[g] = m;
      wl_w[g] = lsum;
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      wacc_w[g * HD + 8 * n + 2 * t] = O[n][0];
      wacc_w[g * HD + 8 * n + 2 * t + 1] = O[n][1];
    }
  }
}

// q, the new K/V rows, the position and the cache may have been written
// earlier in the same launch by other CTAs (persistent decode kernel): they are
// read with ld.global.cg (L2).
// One (KV head kvh, split) item by NW warps (thread ids 0..32*NW-1, synchronised
// with named barrier 1).  The positions [0, *pos] are cut into at most `nsplit`
// splits of at least min_per_split positions (multiples of PPI); items with
// split >= the active count return at once.  Each warp iteration covers PPI =
// 32/(HD/32) positions (8 at head_dim 128, 16 at 64), with the next
// iteration's loads in flight while the current one computes:
//  QK   HD/32 lanes per position, lane = one 32-element Q8_0 block: 32 FMAs
//       per query head against q in shared memory, block scale, then a
//       shuffle sum over the position's lanes;
//  softmax  online per warp (running max / sum per query head);
//  PV   lane = HD/32 output columns; per position one coalesced row read of V,
//       p broadcast by shuffle with the V block scale folded in.
// Warps merge in shared memory; splits merge through `part` (log-sum-exp),
// the last item of the KV head (atomic ticket) writing the output.
template <int HD, int G, int NW>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, uint32_t kvh, uint32_t split, uint32_t active,
                                            float* sm);

template <int HD, int G, int NW, bool LONG = false>
__device__ __forceinline__ void attn_item(const AttnArgs& a, uint32_t kvh, uint32_t split,
                                          uint32_t nsplit, float* sm) {
  using Tile = AttnTile<HD>;
  using SM = AttnSmem<HD, G, NW>;
  constexpr int LPP = Tile::LPP, PPI = Tile::PPI, EPL = Tile::EPL;
  constexpr int NT = 32 * NW;
  const uint32_t KV = a.kv.n_kv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t pos = __ldcg(a.pos);
  if (pos >= a.kv.max_seq) {
    if (tid == 0) set_error(a.err, DERR_BAD_POS);
    return;
  }
  const uint32_t seq = pos + 1;
  uint32_t n0 = (seq + a.min_per_split - 1) / a.min_per_split;
  n0 = n0 < 1 ? 1 : (n0 > nsplit ? nsplit : n0);
  const uint32_t per = (((seq + n0 - 1) / n0) + PPI - 1) / PPI * PPI;
  const uint32_t active = (seq + per - 1) / per;  // every active split is non-empty
  if (split >= active) return;
  const uint32_t p0 = split * per, p1 = min(seq, p0 + per);

  float (*qs)[LPP][SM::QROW] = reinterpret_cast<float (*)[LPP][SM::QROW]>(sm + SM::Q);
  float (*wm)[G] = reinterpret_cast<float (*)[G]>(sm + SM::WM);
  float (*wl)[G] = reinterpret_cast<float (*)[G]>(sm + SM::WL);
  float (*wacc)[G][HD] = reinterpret_cast<float (*)[G][HD]>(sm + SM::WACC);

  for (int i = tid; i < G * HD; i += NT) {
    const int g = i / HD, d = i % HD;
    qs[g][d / 32][d % 32] = __ldcg(a.q + (kvh + KV * g) * HD + d);  // query head kvh + KV*g (h % KV == kvh)
  }
  if (a.k_new && pos >= p0 && pos < p1)
    append_head(a.kv, a.layer, kvh, pos, a.k_new, a.v_new, warp, lane, NW);
  att_sync(NT);

  const int8_t* reg = a.kv.region(a.layer, kvh);
  const int8_t* Kq = reg + a.kv.kq_off;
  const float* Ks = reinterpret_cast<const float*>(reg + a.kv.ks_off);
  const int8_t* Vq = reg + a.kv.vq_off;
  const float* Vs = reinterpret_cast<const float*>(reg + a.kv.vs_off);
  const int b = lane % LPP;
  const uint32_t tl = lane / LPP;

  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
  }

  constexpr uint32_t STEP = PPI * NW;
  uint32_t T = p0 + PPI * warp;
  Tile cur;
  const bool long_range = LONG && p1 - p0 >= ATT_SPLIT_LONG;
  if (long_range)
    attn_long_tc<HD, G, NW>(a, sm + SM::Q, Kq, Ks, Vq, Vs, p0, p1, warp, lane,
                            reinterpret_cast<uint8_t*>(sm + SM::PB + warp * SM::PB_WARP), &wm[warp][0], &wl[warp][0],
                            &wacc[warp][0][0]);
  else if (T < p1)
    cur.load(Kq, Ks, Vq, Vs, T, p1, lane);
  for (; !long_range && T < p1; T += STEP) {
    Tile nxt;
    if (T + STEP < p1) nxt.load(Kq, Ks, Vq, Vs, T + STEP, p1, lane);
    const bool ok = T + tl < p1;
    // ---- scores ----
    float kf[32];
    s8x4_to_f32(cur.k0.x, kf);
    s8x4_to_f32(cur.k0.y, kf + 4);
    s8x4_to_f32(cur.k0.z, kf + 8);
    s8x4_to_f32(cur.k0.w, kf + 12);
    s8x4_to_f32(cur.k1.x, kf + 16);
    s8x4_to_f32(cur.k1.y, kf + 20);
    s8x4_to_f32(cur.k1.z, kf + 24);
    s8x4_to_f32(cur.k1.w, kf + 28);
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4* qv = reinterpret_cast<const float4*>(&qs[g][b][0]);
      float sb = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 q4 = qv[u];
        sb = fmaf(q4.x, kf[4 * u], sb);
        sb = fmaf(q4.y, kf[4 * u + 1], sb);
        sb = fmaf(q4.z, kf[4 * u + 2], sb);
        sb = fmaf(q4.w, kf[4 * u + 3], sb);
      }
      float sc = sb * cur.ks;
#pragma unroll
      for (int o = 1; o < LPP; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
      p[g] = sc;
    }
    // ---- online softmax (per warp) ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sg = ok ? p[g] * a.scale : -INFINITY;
      const float mn = fmaxf(m[g], warp_max(sg));  // position T is valid: finite
      const float pg = ok ? expf(sg - mn) : 0.f;
      p[g] = pg;
      const float corr = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
      l[g] = fmaf(l[g], corr, warp_sum(b == 0 ? pg : 0.f));
      m[g] = mn;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] *= corr;
    }
    // ---- P.V ----
#pragma unroll
    for (int j = 0; j < PPI; ++j) {
      float vf[4];
      s8x4_to_f32(cur.vw[j], vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = __shfl_sync(0xffffffffu, p[g], j * LPP) * cur.vs[j];
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(pj, vf[e], acc[g][e]);
      }
    }
    cur = nxt;
  }
  // ---- merge the warps (the tensor-core loop stored its own) ----
  if (!long_range) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) wacc[warp][g][lane * EPL + e] = acc[g][e];
      if (lane == 0) {
        wm[warp][g] = m[g];
        wl[warp][g] = l[g];
      }
    }
  }
  attn_finish<HD, G, NW>(a, kvh, split, active, sm);
}


// Split partials in `part`, per KV head: the (max, sum) pairs of every
// (split, query head) first -- [n_kv][max_splits][8][2], so one head's pairs
// are contiguous and 16-byte aligned -- then the unnormalised outputs,
// [n_kv][max_splits][G][HD].
__device__ __forceinline__ float* part_ml(const AttnArgs& a, uint32_t kvh) {
  return a.part + (size_t)kvh * a.max_splits * 16;
}
template <int HD, int G>
__device__ __forceinline__ float* part_o(const AttnArgs& a, uint32_t kvh) {
  return a.part + (size_t)a.kv.n_kv * a.max_splits * 16 + (size_t)kvh * a.max_splits * G * HD;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The end of an item: the NW warps' partial results (wm, wl, wacc of
// AttnSmem, every warp's slots written) merge into this split's result, then
// the splits of the KV head merge through `part` in log-sum-exp form, the last
// item of the head (atomic ticket) writing the output.
template <int HD, int G, int NW>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, uint32_t kvh, uint32_t split, uint32_t active,
                                            float* sm) {
  using SM = AttnSmem<HD, G, NW>;
  constexpr int NT = 32 * NW;
  const uint32_t KV = a.kv.n_kv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float (*wm)[G] = reinterpret_cast<float (*)[G]>(sm + SM::WM);
  float (*wl)[G] = reinterpret_cast<float (*)[G]>(sm + SM::WL);
  float (*wacc)[G][HD] = reinterpret_cast<float (*)[G][HD]>(sm + SM::WACC);
  float (*sw)[G] = reinterpret_cast<float (*)[G]>(sm + SM::SW);
  float* sL = sm + SM::SL;
  int* is_last = reinterpret_cast<int*>(sm + SM::FLAG);
  att_sync(NT);
  // the warps' weights exp(m_w - M), the split's (M, L) per query head, once
  if (tid < G) {
    const int g = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = (wm[w][g] == -INFINITY) ? 0.f : expf(wm[w][g] - M);
      sw[w][g] = f;
      L = fmaf(f, wl[w][g], L);
    }
    sw[NW][g] = M;
    sL[g] = L;
  }
  att_sync(NT);
  float* ml = part_ml(a, kvh) + (size_t)split * 16;
  float* po = part_o<HD, G>(a, kvh) + (size_t)split * G * HD;
  for (int i = tid; i < G * HD; i += NT) {
    const int g = i / HD, d = i % HD;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) O = fmaf(sw[w][g], wacc[w][g][d], O);
    const float L = sL[g];
    if (active == 1) {
      a.out[(kvh + KV * g) * HD + d] = (L == 0.f) ? 0.f : O * (1.0f / L);
    } else {
      po[g * HD + d] = O;
      if (d == 0) {
        ml[2 * g] = sw[NW][g];
        ml[2 * g + 1] = L;
      }
    }
  }
  if (active == 1) {
    att_sync(NT);  // shared memory is reused by the caller's next item
    return;
  }
  // ---- merge the splits: the last item of this KV head ----
  __threadfence();
  att_sync(NT);
  if (tid == 0) {
    const int prev = atomicAdd(&a.counters[kvh], 1);
    *is_last = (prev == (int)active - 1);
  }
  att_sync(NT);
  const bool last = *is_last != 0;
  if (!last) {
    att_sync(NT);  // shared memory is reused by the caller's next item
    return;
  }
  __threadfence();
  {
    const float* mlh = part_ml(a, kvh);
    const float* oh = part_o<HD, G>(a, kvh);
    // split weights exp(m_s - M) per query head, then the weighted sums
#pragma unroll 4
    for (uint32_t i = tid; i < active * G; i += NT) sw[i / G][i % G] = __ldcg(&mlh[((i / G) * 8 + i % G) * 2]);
    att_sync(NT);
    for (int g = warp; g < G; g += NW) {
      float M = -INFINITY;
      for (uint32_t sp = lane; sp < active; sp += 32) M = fmaxf(M, sw[sp][g]);
      M = warp_max(M);
      float L = 0.f;
      for (uint32_t sp = lane; sp < active; sp += 32) {
        const float ms = sw[sp][g];
        const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
        sw[sp][g] = w;
        L = fmaf(w, __ldcg(&mlh[(sp * 8 + g) * 2 + 1]), L);
      }
      L = warp_sum(L);
      if (lane == 0) sL[g] = L;
    }
    att_sync(NT);
    for (int i = tid; i < G * HD; i += NT) {
      const int g = i / HD, d = i % HD;
      float O = 0.f;
#pragma unroll 8
      for (uint32_t sp = 0; sp < active; ++sp) O = fmaf(sw[sp][g], __ldcg(&oh[((size_t)sp * G + g) * HD + d]), O);
      const float L = sL[g];
      a.out[(kvh + KV * g) * HD + d] = (L == 0.f) ? 0.f : O * (1.0f / L);
    }
  }
  if (tid == 0) a.counters[kvh] = 0;
  att_sync(NT);  // shared memory is reused by the caller's next item
}


// ------------------------- cluster attention --------------------------------
// One thread-block cluster per KV head; CTA rank r of the cluster is split r of
// the positions [0, pos].  Splits merge through distributed shared memory:
// each CTA stores its (max, sum, output) into its slot in the leader CTA's
// shared memory with st.async, whose bytes complete on the leader's mbarrier
// (no fence, no arrive), so no partials go through global memory and only the
// leader waits.  The new token's K/V row
// (position pos) is quantised in registers and used directly -- the same
// bytes the append stores -- so the cache loads of the older positions can be
// issued before the previous kernel's outputs (q, new K/V) are waited for.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}
// Shared-memory address of `p` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}

constexpr int ATT_CLUSTER_MAX = 16;  // largest cluster the launcher picks

// Cluster-scope helpers for the split merge: peers store their partial result
// into the leader CTA's shared memory with transaction-counted async stores.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Asynchronous store into a peer CTA's shared memory whose completion counts
// 4 bytes on that CTA's mbarrier (no fence, no arrive: the receiver's barrier
// expects the bytes).
__device__ __forceinline__ void dsmem_st_async(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded (WAIT_BUDGET_NS) wait for the peers' partials; false on time-out.
__device__ __forceinline__ bool wait_peers(uint64_t* bar) {
  if (mbar_try_wait_cluster(bar, 0)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait_cluster(bar, 0)) return true;
    __nanosleep(32);
    if ((n & 31) == 0 && globaltimer_ns() - t0 > WAIT_BUDGET_NS) return false;
  }
}

// Q8_0 of one 32-element block already in registers (q8_quantize_vec,
// engine/src/kv_cache.c:28-55): same maximum, IEEE division and rounding as
// the append kernels, so the bytes are identical.
__device__ __forceinline__ float q8_regs(const float4 (&v4)[8], uint4 (&q)[2]) {
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u)
    amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v4[u].x), fabsf(v4[u].y))), fmaxf(fabsf(v4[u].z), fabsf(v4[u].w)));
  float scale = amax / 127.0f;
  if (scale == 0.0f) scale = 1.0f;
  uint32_t w[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float e4[4] = {v4[u].x, v4[u].y, v4[u].z, v4[u].w};
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int t = __float2int_rn(e4[e] / scale);
      t = t > 127 ? 127 : (t < -127 ? -127 : t);
      word |= ((uint32_t)t & 0xFFu) << (8 * e);
    }
    w[u] = word;
  }
  q[0] = make_uint4(w[0], w[1], w[2], w[3]);
  q[1] = make_uint4(w[4], w[5], w[6], w[7]);
  return scale;
}

template <int HD, int G, int NW>
struct AttnCSmem {  // offsets in floats
  static constexpr int LPP = HD / 32;
  static constexpr int QROW = 36;
  static constexpr int Q = 0;
  static constexpr int WM = Q + G * LPP * QROW;
  static constexpr int WL = WM + NW * G;
  static constexpr int WACC = WL + NW * G;
  static constexpr int SLOT = 2 * G + G * HD;  // one CTA's partial: m[G], l[G], o[G][HD]
  static constexpr int PB = WACC + NW * G * HD;   // long contexts: per-warp p[G][32]
  static constexpr int SLOTS = PB + NW * G * 32;  // leader: one slot per cluster rank
  static_assert(NW * 32 >= ATT_CLUSTER_MAX + 1 && NW * 32 >= NW + 2,
                "merge weights fit in the long loop's scratch");
  static constexpr int BAR = (SLOTS + ATT_CLUSTER_MAX * SLOT + 1) & ~1;  // leader's mbarrier
  static constexpr int FLOATS = BAR + 2;
  static constexpr size_t BYTES = (size_t)FLOATS * 4;
};

// Cluster attention for KV head blockIdx.y by NW warps; see above.  Each CTA
// reduces its positions to a partial (max, sum of exponentials, unnormalised
// output) per query head and stores it into its slot in the leader CTA's
// shared memory; the leader (rank 0) waits for its peers on an mbarrier
// (bounded), merges the slots in rank order and writes the output.  Peers
// leave as soon as their async stores are issued.
template <int HD, int G, int NW, bool LONG>
__device__ __forceinline__ void attn_cluster(const AttnArgs& a, float* sm) {
  using Tile = AttnTile<HD>;
  using SM = AttnCSmem<HD, G, NW>;
  constexpr int LPP = Tile::LPP, PPI = Tile::PPI, EPL = Tile::EPL;
  constexpr int NT = 32 * NW;
  constexpr int LPB = 32 / EPL;  // lanes sharing one V block in the PV layout
  constexpr int QPT = (G * HD + NT - 1) / NT;  // q elements per thread
  const uint32_t KV = a.kv.n_kv, kvh = blockIdx.y;
  const uint32_t rank = cluster_rank(), CS = cluster_size();
  const bool leader = rank == 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The position and the cache rows before it were written by earlier graph
  // launches or stream work, never by the kernel this one may overlap.
  const uint32_t pos = __ldcg(a.pos);
  if (pos >= a.kv.max_seq) {
    if (tid == 0 && rank == 0) set_error(a.err, DERR_BAD_POS);
    return;  // the whole cluster leaves before any cluster barrier
  }
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + SM::BAR);
  if (CS > 1) {
    if (leader && tid == 0) {
      mbar_init(bar, 1);  // the leader's own arrive; the peers' bytes are transactions
      fence_mbar_init();
    }
    cluster_arrive();  // paired with cluster_wait before the first remote store
  }
  const uint32_t seq = pos + 1;
  uint32_t n0 = (seq + a.min_per_split - 1) / a.min_per_split;
  n0 = n0 < 1 ? 1 : (n0 > CS ? CS : n0);
  const uint32_t per = (((seq + n0 - 1) / n0) + PPI - 1) / PPI * PPI;
  const uint32_t active = (seq + per - 1) / per;
  const uint32_t p0 = rank * per, p1 = min(seq, p0 + per);
  const bool mine = rank < active;
  if (CS > 1 && leader && tid == 0)  // every active peer sends one slot
    mbar_arrive_expect_tx(bar, (active - 1) * (uint32_t)SM::SLOT * 4u);
  const bool own_new = a.k_new != nullptr && mine && pos >= p0 && pos < p1;

  float (*qs)[LPP][SM::QROW] = reinterpret_cast<float (*)[LPP][SM::QROW]>(sm + SM::Q);
  float (*wm)[G] = reinterpret_cast<float (*)[G]>(sm + SM::WM);
  float (*wl)[G] = reinterpret_cast<float (*)[G]>(sm + SM::WL);
  float (*wacc)[G][HD] = reinterpret_cast<float (*)[G][HD]>(sm + SM::WACC);

  int8_t* reg = const_cast<int8_t*>(a.kv.region(a.layer, kvh));
  const int8_t* Kq = reg + a.kv.kq_off;
  const float* Ks = reinterpret_cast<const float*>(reg + a.kv.ks_off);
  const int8_t* Vq = reg + a.kv.vq_off;
  const float* Vs = reinterpret_cast<const float*>(reg + a.kv.vs_off);
  const int b = lane % LPP;
  const uint32_t tl = lane / LPP;

  constexpr uint32_t STEP = PPI * NW;
  uint32_t T = p0 + PPI * warp;
  Tile cur;
  if (mine && T < p1) cur.load(Kq, Ks, Vq, Vs, T, p1, lane);  // in flight across the wait

  pdl_wait();  // q and the new K/V row come from the previous kernel
  // every load that depends on it is issued before any is used
  float4 kn4[8];
  float vv[EPL];
  if (own_new) {
    const float4* ks4 = reinterpret_cast<const float4*>(a.k_new + kvh * HD + 32 * b);
#pragma unroll
    for (int u = 0; u < 8; ++u) kn4[u] = __ldcg(ks4 + u);
#pragma unroll
    for (int e = 0; e < EPL; ++e) vv[e] = __ldcg(a.v_new + kvh * HD + lane * EPL + e);
  }
  float qv[QPT];
#pragma unroll
  for (int j = 0; j < QPT; ++j) {
    const int i = tid + j * NT;
    if (i < G * HD) qv[j] = __ldcg(a.q + (kvh + KV * (i / HD)) * HD + i % HD);  // query head kvh + KV*g
  }
#pragma unroll
  for (int j = 0; j < QPT; ++j) {
    const int i = tid + j * NT;
    if (i < G * HD) qs[i / HD][(i % HD) / 32][i % 32] = qv[j];
  }
  // The new K/V row: K in the QK layout (lane = 32-element block b), V in the
  // PV layout (EPL columns per lane, LPB lanes per block); warp 0 appends both.
  uint4 kq_new[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  float ks_new = 1.f;
  uint32_t vw_new = 0;
  float vs_new = 1.f;
  if (own_new) {
    ks_new = q8_regs(kn4, kq_new);
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) amax = fmaxf(amax, fabsf(vv[e]));
#pragma unroll
    for (int o = 1; o < LPB; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    vs_new = amax / 127.0f;
    if (vs_new == 0.0f) vs_new = 1.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      int t = __float2int_rn(vv[e] / vs_new);
      t = t > 127 ? 127 : (t < -127 ? -127 : t);
      vw_new |= ((uint32_t)t & 0xFFu) << (8 * e);
    }
    if (warp == 0) {
      int8_t* vq = reg + a.kv.vq_off + (size_t)pos * HD + lane * EPL;
      if (EPL == 4)
        *reinterpret_cast<uint32_t*>(vq) = vw_new;
      else
        *reinterpret_cast<uint16_t*>(vq) = (uint16_t)vw_new;
      if (lane % LPB == 0)
        reinterpret_cast<float*>(reg + a.kv.vs_off)[(size_t)pos * (HD / 32) + lane / LPB] = vs_new;
      if (tl == 0) {
        uint4* dst = reinterpret_cast<uint4*>(reg + a.kv.kq_off + (size_t)pos * HD + 32 * b);
        dst[0] = kq_new[0];
        dst[1] = kq_new[1];
        reinterpret_cast<float*>(reg + a.kv.ks_off)[(size_t)pos * (HD / 32) + b] = ks_new;
      }
    }
  }
  att_sync(NT);

  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
  }
  if (LONG && mine && p1 - p0 >= ATT_LONG_MIN)
    attn_long<HD, G, NW>(a, sm + SM::Q, Kq, Ks, Vq, Vs, p0, p1, warp, lane, sm + SM::PB + warp * G * 32, m, l, acc);
  else
  for (; mine && T < p1; T += STEP) {
    Tile nxt;
    if (T + STEP < p1) nxt.load(Kq, Ks, Vq, Vs, T + STEP, p1, lane);
    const uint32_t nt = min((uint32_t)PPI, p1 - T);
    const bool ok = tl < nt;
    const uint32_t t = T + (ok ? tl : 0);
    // ---- scores ----
    float kf[32];
    float ksc = cur.ks;
    uint4 k0 = cur.k0, k1 = cur.k1;
    if (own_new && t == pos) {  // the new row, quantised above
      k0 = kq_new[0];
      k1 = kq_new[1];
      ksc = ks_new;
    }
    s8x4_to_f32(k0.x, kf);
    s8x4_to_f32(k0.y, kf + 4);
    s8x4_to_f32(k0.z, kf + 8);
    s8x4_to_f32(k0.w, kf + 12);
    s8x4_to_f32(k1.x, kf + 16);
    s8x4_to_f32(k1.y, kf + 20);
    s8x4_to_f32(k1.z, kf + 24);
    s8x4_to_f32(k1.w, kf + 28);
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4* qv4 = reinterpret_cast<const float4*>(&qs[g][b][0]);
      float sb = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 q4 = qv4[u];
        sb = fmaf(q4.x, kf[4 * u], sb);
        sb = fmaf(q4.y, kf[4 * u + 1], sb);
        sb = fmaf(q4.z, kf[4 * u + 2], sb);
        sb = fmaf(q4.w, kf[4 * u + 3], sb);
      }
      float sc = sb * ksc;
#pragma unroll
      for (int o = 1; o < LPP; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
      p[g] = sc;
    }
    // ---- online softmax (per warp) ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sg = ok ? p[g] * a.scale : -INFINITY;
      const float mn = fmaxf(m[g], warp_max(sg));  // position T is valid: finite
      const float pg = ok ? expf(sg - mn) : 0.f;
      p[g] = pg;
      const float corr = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
      l[g] = fmaf(l[g], corr, warp_sum(b == 0 ? pg : 0.f));
      m[g] = mn;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] *= corr;
    }
    // ---- P.V ----
#pragma unroll
    for (int j = 0; j < PPI; ++j) {
      const uint32_t tj = T + ((uint32_t)j < nt ? j : 0);
      const bool nw_ = own_new && tj == pos;
      float vf[4];
      s8x4_to_f32(nw_ ? vw_new : cur.vw[j], vf);
      const float vsj = nw_ ? vs_new : cur.vs[j];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = __shfl_sync(0xffffffffu, p[g], j * LPP) * vsj;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(pj, vf[e], acc[g][e]);
      }
    }
    cur = nxt;
  }
  // ---- merge the warps into this CTA's partial, stored into its slot in the
  //      leader's shared memory ----
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) wacc[warp][g][lane * EPL + e] = acc[g][e];
    if (lane == 0) {
      wm[warp][g] = m[g];
      wl[warp][g] = l[g];
    }
  }
  att_sync(NT);
  if (CS > 1) cluster_wait();  // the leader runs (its barrier is initialised)
  float* slot = sm + SM::SLOTS + rank * SM::SLOT;
  const uint32_t slot_r = dsmem_addr(slot, 0);  // the same offset in the leader
  const uint32_t bar_r = dsmem_addr(bar, 0);
  // The warps' weights exp(m_w - M) per query head, once (G threads, into
  // the long loop's scratch), then each output is a short FMA chain.
  float* wf = sm + SM::PB;  // [NW][G] weights, then [G] M, then [G] L
  if (mine && tid < G) {
    const int g = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = (wm[w][g] == -INFINITY) ? 0.f : expf(wm[w][g] - M);
      wf[w * G + g] = f;
      L = fmaf(f, wl[w][g], L);
    }
    wf[NW * G + g] = M;
    wf[NW * G + G + g] = L;
  }
  att_sync(NT);
  if (mine) {
    for (int i = tid; i < G * HD; i += NT) {
      const int g = i / HD, d = i % HD;
      const float M = wf[NW * G + g], L = wf[NW * G + G + g];
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) O = fmaf(wf[w * G + g], wacc[w][g][d], O);
      if (leader) {
        slot[2 * G + i] = O;
        if (d == 0) {
          slot[g] = M;
          slot[G + g] = L;
        }
      } else {
        dsmem_st_async(slot_r + 4u * (uint32_t)(2 * G + i), O, bar_r);
        if (d == 0) {
          dsmem_st_async(slot_r + 4u * (uint32_t)g, M, bar_r);
          dsmem_st_async(slot_r + 4u * (uint32_t)(G + g), L, bar_r);
        }
      }
    }
  }
  if (!leader) return;  // the async stores complete on the leader's barrier
  att_sync(NT);         // the leader's own slot
  // ---- leader: merge the splits in rank order ----
  if (CS > 1) {  // one waiter; the others sleep in the CTA barrier
    int* flag = reinterpret_cast<int*>(sm + SM::WM);  // the warp maxima are merged already
    if (tid == 0) *flag = wait_peers(bar) ? 1 : 0;
    att_sync(NT);
    if (*flag == 0) {
      if (tid == 0) set_error(a.err, DERR_TIMEOUT_GRID);
      return;
    }
  }
  // The slot weights exp(m_r - M) and 1/L of each query head, once (G
  // threads), into the long loop's scratch (free by now); then every output
  // is a short fixed-order FMA chain over the slots.
  const float* sl0 = sm + SM::SLOTS;
  float* wsc = sm + SM::PB;  // [ATT_CLUSTER_MAX][G] weights, then [G] 1/L
  // Branch-free over ATT_CLUSTER_MAX slots (loads clamped to the last active
  // slot, inactive slots weighted 0) so the loads and exponentials overlap.
  if (tid < G) {
    const int g = tid;
    float mr[ATT_CLUSTER_MAX], lr[ATT_CLUSTER_MAX];
#pragma unroll
    for (int r = 0; r < ATT_CLUSTER_MAX; ++r) {
      const int rr = r < (int)active ? r : (int)active - 1;
      mr[r] = sl0[rr * SM::SLOT + g];
      lr[r] = sl0[rr * SM::SLOT + G + g];
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < ATT_CLUSTER_MAX; ++r) M = fmaxf(M, mr[r]);
    float L = 0.f;
#pragma unroll
    for (int r = 0; r < ATT_CLUSTER_MAX; ++r) {
      const float e = expf(mr[r] - M);
      const float w = (r < (int)active && mr[r] != -INFINITY) ? e : 0.f;
      wsc[r * G + g] = w;
      L = fmaf(w, lr[r], L);
    }
    wsc[ATT_CLUSTER_MAX * G + g] = (L == 0.f) ? 0.f : 1.0f / L;
  }
  att_sync(NT);
  for (int i = tid; i < G * HD; i += NT) {
    const int g = i / HD;
    float O = 0.f;
#pragma unroll
    for (int r = 0; r < ATT_CLUSTER_MAX; ++r) {
      const int rr = r < (int)active ? r : (int)active - 1;
      O = fmaf(wsc[r * G + g], sl0[rr * SM::SLOT + 2 * G + i], O);
    }
    a.out[(kvh + KV * g) * HD + i % HD] = O * wsc[ATT_CLUSTER_MAX * G + g];
  }
}

}  // namespace adev
}  // namespace shk
