// attn_split.cuh -- decode attention over long caches (device code).
//
// One CTA per (KV head, split) of the positions [0, pos]; the split's Q8_0 K
// and V rows and their block scales stream through shared memory in
// 16-position chunks (cp.async, 16-byte pieces, 128-byte-swizzled rows so the
// tensor-core fragment loads below are conflict-free): warp w takes chunks
// w, w + 4, w + 8, ... of the split, each through its own ring of
// SPL_NSTAGE slots, so the warps never wait for one another.  Per chunk:
//
//   QK^T  exact integer products on the tensor cores (mma.sync m16n8k32,
//         s8 x s8 -> s32): the K bytes are the B operand as stored (ldmatrix
//         of the staged rows); each query head's q is a 32-bit fixed-point
//         integer F = rn(q * c_h) (c_h = 126 * 2^24 / max|q_h|, so every
//         element keeps fp32's relative precision) split into four balanced
//         s8 limbs -- limbs 0/1 in rows h / h+8 of one A operand, limbs 2/3 of
//         a second -- so two MMAs give every Q8_0 block's dot product exactly;
//         the limbs combine in fp32 and the block scale is applied as the
//         reference's dequantised K would (engine/src/kv_cache.c:175-199);
//   softmax  online, in base 2 (scores * scale * log2(e) / c_h), per query
//         head over the 4 lanes of a quad (16 positions);
//   PV    O^T = V^T P on f16 tensor cores (mma.sync m16n8k16, fp32
//         accumulators): V^T fragments by ldmatrix.trans of the staged rows
//         (int8 -> f16 exactly by a byte permute and one f16x2 subtract), the
//         weights p * v_scale as the B operand in two f16 parts (high: the top
//         11 bits, low: the rest, rounded; ~24 bits), both accumulated into
//         the same fp32 registers.  v_scale is taken relative to a running
//         power of two 2^E >= every V scale seen (O rescaled when it grows),
//         so the weights stay <= 1 and in f16's normal range.
//
// The lane mapping (g = lane / 4, t = lane % 4) closes on itself: the QK^T
// accumulator of lane (g, t) holds head g's scores at chunk positions
// 2t, 2t+1 (n-tile 0) and 8+2t, 9+2t (n-tile 1), exactly the k indices
// (2t, 2t+1), (2t+8, 2t+9) of the PV B operand, so the weights never leave
// the registers that computed them.  The PV accumulator of lane (g, t) holds
// heads 2t, 2t+1 at dims 2g, 2g+1 of each 16-dim tile.
//
// Splits merge in two levels: the CTAs of a thread-block cluster (CL
// consecutive splits) over distributed shared memory, then the clusters'
// records through `part` (a ticket per output slice: the last cluster to
// write a slice merges it over every record).  Every wait is a hardware one
// (cp.async.wait_group, bar.sync, barrier.cluster).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "attn_dev.cuh"

namespace shk {
namespace adev {

constexpr int SPL_WARPS = 4;
constexpr int SPL_THREADS = 32 * SPL_WARPS;
constexpr int SPL_CHUNK = 16;                      // positions per warp per stage
constexpr int SPL_NSTAGE = 3;                      // ring depth (chunks per warp)
// Splits: of SPL_MIN_PER_SPLIT positions or more, at most CL of them (one
// cluster: no merge through global memory) while splits of SPL_LONG_SPLIT
// positions would fit one cluster, else of SPL_LONG_SPLIT positions or more
// (as many as the grid holds).
constexpr uint32_t SPL_MIN_PER_SPLIT = 64;
constexpr uint32_t SPL_LONG_SPLIT = 256;  // 128: 8k positions 17.2 us, 256: 15.3, 512: 19.2

// Each warp streams its own 16-position chunks through SPL_NSTAGE slots of
// the ring (no CTA-wide barrier in the loop): slot = [K rows][V rows][K
// scales][V scales] of one chunk.
template <int HD>
struct SplitRing {
  static constexpr int NB = HD / 32;
  static constexpr int KB = SPL_CHUNK * HD;      // K (and V) bytes of a chunk
  static constexpr int SB = SPL_CHUNK * NB * 4;  // K (and V) scale bytes of a chunk
  static constexpr int K = 0, V = KB, KS = 2 * KB, VS = 2 * KB + SB;
  static constexpr int CHUNK = 2 * KB + 2 * SB;
  static constexpr int BYTES = SPL_WARPS * SPL_NSTAGE * CHUNK;
};

// Byte offset of 16-byte piece c of row r of a staged K or V block: rows of
// HD bytes, pieces permuted so any 8 consecutive rows put one piece index in
// 8 distinct bank groups.
template <int HD>
__device__ __forceinline__ uint32_t spl_swz(uint32_t r, uint32_t c) {
  if constexpr (HD == 128)
    return r * 128u + ((c ^ (r & 7u)) << 4);
  else
    return r * 64u + ((c ^ ((r >> 1) & 3u)) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// limbs (weights 2^24, 2^16, 2^8, 1) of one position's block product, in fp32
__device__ __forceinline__ float limb_sum(int c0, int c1, int d0, int d1) {
  return fmaf((float)(c0 * 256 + c1), 65536.0f, (float)(d0 * 256 + d1));
}
// x = hi + lo with hi the top 11 significant bits of x (exact in f16 for
// |x| in f16's normal range) and lo the rest
__device__ __forceinline__ void split_hi_lo(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

// The NB block scales of one staged position (16- or 8-byte aligned).
template <int NB>
__device__ __forceinline__ void lds_scales(const float* p, float (&o)[NB]) {
  if constexpr (NB == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x;
    o[1] = v.y;
    o[2] = v.z;
    o[3] = v.w;
  } else {
    const float2 v = *reinterpret_cast<const float2*>(p);
    o[0] = v.x;
    o[1] = v.y;
  }
}

// Positions `b`..`e` (e - b <= SPL_CHUNK) into the ring slot at shared
// address `slot`, by the 32 lanes of one warp: K and V rows swizzled, scales
// linear.
template <int HD>
__device__ __forceinline__ void spl_issue(uint32_t slot, uint8_t* slot_p, const int8_t* Kq, const float* Ks,
                                          const int8_t* Vq, const float* Vs, uint32_t b, uint32_t e, int lane) {
  using R = SplitRing<HD>;
  constexpr uint32_t CPR = HD / 16;
  const uint32_t n = e - b;
  for (uint32_t i = lane; i < n * CPR; i += 32) {
    const uint32_t r = i / CPR, c = i % CPR;
    const uint32_t o = spl_swz<HD>(r, c);
    cp_async16(slot + R::K + o, Kq + (size_t)(b + r) * HD + 16 * c);
    cp_async16(slot + R::V + o, Vq + (size_t)(b + r) * HD + 16 * c);
  }
  // b is a multiple of 16 positions: the scale rows start 16-byte aligned
  const uint32_t nf = n * R::NB, n16 = nf / 4;
  for (uint32_t i = lane; i < n16; i += 32) {
    cp_async16(slot + R::KS + 16 * i, Ks + (size_t)b * R::NB + 4 * i);
    cp_async16(slot + R::VS + 16 * i, Vs + (size_t)b * R::NB + 4 * i);
  }
  // head_dim 64 with an odd row count: the last row's two scales, by plain
  // loads (published to the warp by the same __syncwarp as the copies)
  for (uint32_t i = 4 * n16 + lane; i < nf; i += 32) {
    reinterpret_cast<float*>(slot_p + R::KS)[i] = __ldcg(Ks + (size_t)b * R::NB + i);
    reinterpret_cast<float*>(slot_p + R::VS)[i] = __ldcg(Vs + (size_t)b * R::NB + i);
  }
}

// The split's attention on one CTA (SPL_THREADS threads): append the new
// row when it falls in [p0, p1), stream the split through the ring, and leave
// every warp's partial result -- (max, sum) per query head in natural-log
// units and the unnormalised outputs -- in AttnSmem's wm / wl / wacc at the
// start of `sm` (the ring is consumed by then).
template <int HD, int G>
__device__ __forceinline__ void spl_compute(const AttnArgs& a, uint32_t kvh, uint32_t pos, uint32_t p0, uint32_t p1,
                                            const float (&qv)[HD / 32][8], uint8_t* sm) {
  using R = SplitRing<HD>;
  using SM = AttnSmem<HD, G, SPL_WARPS>;
  static_assert(SM::BYTES <= (size_t)R::BYTES, "merge area exceeds the ring");
  constexpr int NB = HD / 32, MT = HD / 16;
  constexpr float L2E = 1.4426950408889634f, LN2 = 0.6931471805599453f;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  int8_t* reg = a.kv.region(a.layer, kvh);
  const int8_t* Kq = reg + a.kv.kq_off;
  const float* Ks = reinterpret_cast<const float*>(reg + a.kv.ks_off);
  const int8_t* Vq = reg + a.kv.vq_off;
  const float* Vs = reinterpret_cast<const float*>(reg + a.kv.vs_off);
  if (a.k_new && pos >= p0 && pos < p1)
    append_head(a.kv, a.layer, kvh, pos, a.k_new, a.v_new, warp, lane, SPL_WARPS);
  __syncthreads();  // the new row is in the cache before any stage copies it

  // this warp's chunks: positions p0 + 16 (warp + 4k), k < nk, each through
  // the warp's own slots
  const uint32_t nchunks = (p1 - p0 + SPL_CHUNK - 1) / SPL_CHUNK;
  const uint32_t nk = nchunks > (uint32_t)warp ? (nchunks - warp + SPL_WARPS - 1) / SPL_WARPS : 0;
  const uint32_t wring = smem_u32(sm) + warp * SPL_NSTAGE * R::CHUNK;
  uint8_t* wring_p = sm + warp * SPL_NSTAGE * R::CHUNK;
#pragma unroll
  for (int s = 0; s < SPL_NSTAGE - 1; ++s) {
    if ((uint32_t)s < nk) {
      const uint32_t b = p0 + SPL_CHUNK * (warp + SPL_WARPS * s);
      spl_issue<HD>(wring + s * R::CHUNK, wring_p + s * R::CHUNK, Kq, Ks, Vq, Vs, b, min(p1, b + SPL_CHUNK), lane);
    }
    cp_async_commit();
  }

  // q as 32-bit fixed point in four s8 limbs; lane (g, t) holds dims
  // 32j + 4t..4t+3 and 32j + 16 + 4t..+3
  uint32_t qa[NB][4], qb[NB][4];
  float qk_mul;
  {
    float qmax = 0.f;
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) qmax = fmaxf(qmax, fabsf(qv[j][i]));
    qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
    qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 2));
    const float c = (qmax > 0.f && qmax <= 3.0e38f) ? 2113929216.0f / qmax : 0.f;  // 126 * 2^24
    qk_mul = c > 0.f ? a.scale * L2E / c : 0.f;
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          int F = __float2int_rn(qv[j][4 * h + i] * c);
          const int l3 = (int)(int8_t)(F & 0xFF);
          F = (F - l3) >> 8;
          const int l2 = (int)(int8_t)(F & 0xFF);
          F = (F - l2) >> 8;
          const int l1 = (int)(int8_t)(F & 0xFF);
          const int l0 = (F - l1) >> 8;
          w0 |= (uint32_t)(l0 & 0xFF) << (8 * i);
          w1 |= (uint32_t)(l1 & 0xFF) << (8 * i);
          w2 |= (uint32_t)(l2 & 0xFF) << (8 * i);
          w3 |= (uint32_t)(l3 & 0xFF) << (8 * i);
        }
        qa[j][2 * h] = w0;      // row g: limb 0
        qa[j][2 * h + 1] = w1;  // row g + 8: limb 1
        qb[j][2 * h] = w2;
        qb[j][2 * h + 1] = w3;
      }
  }

  // per-lane fragment addresses inside a chunk slot (rows 0..15)
  uint32_t koff[NB], voff[NB];
  {
    const int i = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      // K: matrices (rows 0-7, piece 2j), (0-7, 2j+1), (8-15, 2j), (8-15, 2j+1)
      koff[j] = R::K + spl_swz<HD>((i >> 1) * 8 + rr, 2 * j + (i & 1));
      // V: matrices (rows 0-7, piece 2j), (8-15, 2j), (0-7, 2j+1), (8-15, 2j+1)
      voff[j] = R::V + spl_swz<HD>((i & 1) * 8 + rr, 2 * j + (i >> 1));
    }
  }
  const int pr[4] = {2 * t, 2 * t + 1, 8 + 2 * t, 9 + 2 * t};  // this lane's chunk positions

  float O[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) O[mt][0] = O[mt][1] = O[mt][2] = O[mt][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  float vsE = 0.f, vsInv = 0.f;  // 2^E and 2^-E (0, 0 until a nonzero V scale is seen)

  for (uint32_t s = 0; s < nk; ++s) {
    cp_async_wait<SPL_NSTAGE - 2>();
    __syncwarp();  // chunk s is in for every lane; slot (s - 1) % NSTAGE is free
    {
      const uint32_t sn = s + SPL_NSTAGE - 1;
      if (sn < nk) {
        const uint32_t sl = sn % SPL_NSTAGE, b = p0 + SPL_CHUNK * (warp + SPL_WARPS * sn);
        spl_issue<HD>(wring + sl * R::CHUNK, wring_p + sl * R::CHUNK, Kq, Ks, Vq, Vs, b, min(p1, b + SPL_CHUNK),
                      lane);
      }
      cp_async_commit();
    }
    const uint32_t c0 = p0 + SPL_CHUNK * (warp + SPL_WARPS * s);  // this warp's chunk
    const uint32_t nvalid = min((uint32_t)SPL_CHUNK, p1 - c0);
    const uint32_t slot = wring + (s % SPL_NSTAGE) * R::CHUNK;
    const uint8_t* slot_p = wring_p + (s % SPL_NSTAGE) * R::CHUNK;
    bool valid[4];
    float ksc[4][NB], vsc[4][NB];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      valid[i] = (uint32_t)pr[i] < nvalid;
      const float* kr = reinterpret_cast<const float*>(slot_p + R::KS) + pr[i] * NB;
      const float* vr = reinterpret_cast<const float*>(slot_p + R::VS) + pr[i] * NB;
      float kv4[NB], vv4[NB];
      lds_scales<NB>(kr, kv4);
      lds_scales<NB>(vr, vv4);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        ksc[i][j] = valid[i] ? kv4[j] : 0.f;
        vsc[i][j] = valid[i] ? vv4[j] : 0.f;
      }
    }
    // ---- QK^T: exact block products, block scales in fp32
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      uint32_t x0, x1, x2, x3;
      ldsm_x4(slot + koff[j], x0, x1, x2, x3);
      int c[4] = {0, 0, 0, 0}, d[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0}, f[4] = {0, 0, 0, 0};
      mma_s8(c, qa[j], x0, x1);
      mma_s8(d, qb[j], x0, x1);
      mma_s8(e, qa[j], x2, x3);
      mma_s8(f, qb[j], x2, x3);
      sc[0] = fmaf(limb_sum(c[0], c[2], d[0], d[2]), ksc[0][j], sc[0]);
      sc[1] = fmaf(limb_sum(c[1], c[3], d[1], d[3]), ksc[1][j], sc[1]);
      sc[2] = fmaf(limb_sum(e[0], e[2], f[0], f[2]), ksc[2][j], sc[2]);
      sc[3] = fmaf(limb_sum(e[1], e[3], f[1], f[3]), ksc[3][j], sc[3]);
    }
    // ---- online softmax, base 2, per head over the quad's 16 positions
    float x[4], cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[i] = valid[i] ? sc[i] * qk_mul : -INFINITY;
      cm = fmaxf(cm, x[i]);
    }
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
    const float mn = fmaxf(m, cm);  // chunk position 0 is valid: finite
    const float corr = ex2(m - mn);  // m = -inf: 0
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = ex2(x[i] - mn);  // -inf: 0
    l = fmaf(l, corr, (p[0] + p[1]) + (p[2] + p[3]));
    m = mn;
    // ---- the V scale exponent: 2^E above every V scale of the range so far
    float vm = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < NB; ++j) vm = fmaxf(vm, vsc[i][j]);
    vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 1));
    vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 2));  // the same in every quad
    float r = 1.f;
    if (vm >= vsE && vm > 0.f) {  // warp-uniform
      const int e = (int)((__float_as_uint(vm) >> 23) & 0xFFu) - 126;  // 2^e > vm
      const float nE = __uint_as_float((uint32_t)(127 + e) << 23);
      r = vsE / nE;  // exact (0 before the first)
      vsE = nE;
      vsInv = __uint_as_float((uint32_t)(127 - e) << 23);
    }
    if (__any_sync(0xffffffffu, corr != 1.f) || r != 1.f) {
      const float ca = __shfl_sync(0xffffffffu, corr, 8 * t) * r;      // head 2t
      const float cb = __shfl_sync(0xffffffffu, corr, 8 * t + 4) * r;  // head 2t + 1
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        O[mt][0] *= ca;
        O[mt][1] *= cb;
        O[mt][2] *= ca;
        O[mt][3] *= cb;
      }
    }
    // ---- PV: O^T += V^T P', per 32-dim block (two 16-dim tiles)
    float pin[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pin[i] = valid[i] ? p[i] * vsInv : 0.f;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      float hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) split_hi_lo(pin[i] * vsc[i][j], hi[i], lo[i]);
      const uint32_t bh0 = h2_pack(hi[0], hi[1]), bh1 = h2_pack(hi[2], hi[3]);
      const uint32_t bl0 = h2_pack(lo[0], lo[1]), bl1 = h2_pack(lo[2], lo[3]);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(slot + voff[j], v0, v1, v2, v3);
      v0 ^= 0x80808080u;
      v1 ^= 0x80808080u;
      v2 ^= 0x80808080u;
      v3 ^= 0x80808080u;
      // word bytes: (pos 2t, dim 2g), (2t, 2g+1), (2t+1, 2g), (2t+1, 2g+1)
      const uint32_t A0[4] = {s8x2_h2(v0, 0x4240), s8x2_h2(v0, 0x4341), s8x2_h2(v1, 0x4240), s8x2_h2(v1, 0x4341)};
      const uint32_t A1[4] = {s8x2_h2(v2, 0x4240), s8x2_h2(v2, 0x4341), s8x2_h2(v3, 0x4240), s8x2_h2(v3, 0x4341)};
      mma16816(O[2 * j], A0, bh0, bh1);
      mma16816(O[2 * j], A0, bl0, bl1);
      mma16816(O[2 * j + 1], A1, bh0, bh1);
      mma16816(O[2 * j + 1], A1, bl0, bl1);
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with the ring: it becomes the merge area

  float* smf = reinterpret_cast<float*>(sm);
  float (*wm)[G] = reinterpret_cast<float (*)[G]>(smf + SM::WM);
  float (*wl)[G] = reinterpret_cast<float (*)[G]>(smf + SM::WL);
  float (*wacc)[G][HD] = reinterpret_cast<float (*)[G][HD]>(smf + SM::WACC);
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if (t == 0 && g < G) {
    wm[warp][g] = m == -INFINITY ? -INFINITY : m * LN2;
    wl[warp][g] = l;
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int d = 16 * mt + 2 * g;
    if (2 * t < G) {
      wacc[warp][2 * t][d] = O[mt][0] * vsE;
      wacc[warp][2 * t][d + 1] = O[mt][2] * vsE;
    }
    if (2 * t + 1 < G) {
      wacc[warp][2 * t + 1][d] = O[mt][1] * vsE;
      wacc[warp][2 * t + 1][d + 1] = O[mt][3] * vsE;
    }
  }
}

// A CTA's merged split result, after AttnSmem in shared memory: per query
// head the max and the sum, then the unnormalised outputs [G][HD].
template <int HD, int G>
struct SplitRes {
  static constexpr int M = (AttnSmem<HD, G, SPL_WARPS>::BYTES + 15) / 16 * 16;
  static constexpr int L = M + 4 * G;
  static constexpr int O = L + 4 * G;
  static constexpr int END = O + 4 * G * HD;
};

__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// One (KV head, split) item of a cluster of CL consecutive splits; `sm` is the
// dynamic shared memory (SplitRing<HD>::BYTES, 128-byte aligned).  Called by
// SPL_THREADS threads after the previous kernel's outputs are visible.
//   1. the split (spl_compute), its warps merged into SplitRes;
//   2. cluster barrier; CTA r of the cluster merges outputs
//      [r * SLICE, (r + 1) * SLICE) of all CL results over distributed shared
//      memory -- the cluster's log-sum-exp merge, written to the output when
//      one cluster holds every split, else as slice r of record `cluster` of
//      `part`;
//   3. per (KV head, r) ticket: the last cluster to write slice r merges
//      slice r of every cluster record (one load per record and output, all
//      in flight at once);
//   4. no CTA leaves before every CTA of its cluster has finished reading
//      its peers (split cluster barrier around steps 2-3).
template <int HD, int G, int CL>
__device__ __forceinline__ void attn_split_item(const AttnArgs& a, uint32_t kvh, uint32_t split, uint32_t nsplit,
                                                uint8_t* sm) {
  using R = SplitRing<HD>;
  using SM = AttnSmem<HD, G, SPL_WARPS>;
  using RS = SplitRes<HD, G>;
  static_assert(RS::END <= R::BYTES, "split result exceeds the ring");
  constexpr int NT = SPL_THREADS;
  constexpr int SLICE = (G * HD + CL - 1) / CL;
  static_assert(SLICE <= NT, "one output per thread in the cluster merge");
  static_assert((G * HD) % CL == 0 && HD % SLICE == 0, "a merge slice lies within one query head");
  constexpr int NB = HD / 32;
  const uint32_t KV = a.kv.n_kv;
  const int tid = threadIdx.x, lane = tid & 31;
  // q of head g = lane / 4 (query head kvh + KV * g), dims 32j + 4t..4t+3 and
  // 32j + 16 + 4t..+3 (t = lane % 4): issued before the position, on which
  // nothing of it depends
  float qv[NB][8];
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
    if ((lane >> 2) < G) {
      const float* qh = a.q + (size_t)(kvh + KV * (lane >> 2)) * HD + 32 * j + 4 * (lane & 3);
      v0 = __ldcg(reinterpret_cast<const float4*>(qh));
      v1 = __ldcg(reinterpret_cast<const float4*>(qh + 16));
    }
    qv[j][0] = v0.x; qv[j][1] = v0.y; qv[j][2] = v0.z; qv[j][3] = v0.w;
    qv[j][4] = v1.x; qv[j][5] = v1.y; qv[j][6] = v1.z; qv[j][7] = v1.w;
  }
  const uint32_t pos = __ldcg(a.pos);
  if (pos >= a.kv.max_seq) {  // the same in every CTA: before any cluster barrier
    if (tid == 0) set_error(a.err, DERR_BAD_POS);
    return;
  }
  const uint32_t seq = pos + 1;
  uint32_t n0 = (seq + a.min_per_split - 1) / a.min_per_split;
  if (n0 > (uint32_t)CL) n0 = max((uint32_t)CL, (seq + SPL_LONG_SPLIT - 1) / SPL_LONG_SPLIT);
  n0 = n0 < 1 ? 1 : (n0 > nsplit ? nsplit : n0);
  const uint32_t per = (((seq + n0 - 1) / n0) + SPL_CHUNK - 1) / SPL_CHUNK * SPL_CHUNK;
  const uint32_t active = (seq + per - 1) / per;  // every active split is non-empty
  const uint32_t ncl = (active + CL - 1) / CL;    // clusters holding active splits
  const uint32_t cl = split / CL;
  if (cl >= ncl) return;  // the whole cluster: no barrier waits on it
  const uint32_t rank = cluster_rank();

  float* smf = reinterpret_cast<float*>(sm);
  float* cM = reinterpret_cast<float*>(sm + RS::M);
  float* cL = reinterpret_cast<float*>(sm + RS::L);
  float* cO = reinterpret_cast<float*>(sm + RS::O);
  if (split < active) {
    const uint32_t p0 = split * per, p1 = min(seq, p0 + per);
    spl_compute<HD, G>(a, kvh, pos, p0, p1, qv, sm);
    float (*wm)[G] = reinterpret_cast<float (*)[G]>(smf + SM::WM);
    float (*wl)[G] = reinterpret_cast<float (*)[G]>(smf + SM::WL);
    float (*wacc)[G][HD] = reinterpret_cast<float (*)[G][HD]>(smf + SM::WACC);
    float (*sw)[G] = reinterpret_cast<float (*)[G]>(smf + SM::SW);
    __syncthreads();
    if (tid < G) {  // the warps' weights exp(m_w - M), the split's (M, L)
      const int g = tid;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < SPL_WARPS; ++w) M = fmaxf(M, wm[w][g]);
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < SPL_WARPS; ++w) {
        const float f = (wm[w][g] == -INFINITY) ? 0.f : expf(wm[w][g] - M);
        sw[w][g] = f;
        L = fmaf(f, wl[w][g], L);
      }
      cM[g] = M;
      cL[g] = L;
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += NT) {
      const int g = i / HD, d = i % HD;
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < SPL_WARPS; ++w) O = fmaf(sw[w][g], wacc[w][g][d], O);
      cO[i] = O;
    }
  } else {
    for (int i = tid; i < G; i += NT) {
      cM[i] = -INFINITY;
      cL[i] = 0.f;
    }
    for (int i = tid; i < G * HD; i += NT) cO[i] = 0.f;
  }
  cluster_arrive();
  cluster_wait();  // every CTA's result is in its shared memory
  // CTA `rank` merges outputs [rank * SLICE, (rank + 1) * SLICE): within one
  // query head g (SLICE divides HD)
  const int i = (int)rank * SLICE + tid;
  const int g = i / HD, d = i % HD;
  float M = -INFINITY, L = 0.f, O = 0.f;
  if (tid < SLICE) {
    float Mq[CL], Lq[CL], Oq[CL];
#pragma unroll
    for (int q = 0; q < CL; ++q) {
      Mq[q] = ld_dsmem(dsmem_addr(cM + g, q));
      Lq[q] = ld_dsmem(dsmem_addr(cL + g, q));
      Oq[q] = ld_dsmem(dsmem_addr(cO + i, q));
    }
#pragma unroll
    for (int q = 0; q < CL; ++q) M = fmaxf(M, Mq[q]);
#pragma unroll
    for (int q = 0; q < CL; ++q) {
      const float w = (Mq[q] == -INFINITY) ? 0.f : expf(Mq[q] - M);
      L = fmaf(w, Lq[q], L);
      O = fmaf(w, Oq[q], O);
    }
  }
  // this CTA's reads of its peers are done; it leaves only after every peer
  // has said the same (the wait below), and works on in between
  cluster_arrive();
  if (ncl == 1) {
    if (tid < SLICE) a.out[(kvh + KV * g) * HD + d] = (L == 0.f) ? 0.f : O * (1.0f / L);
    cluster_wait();
    return;
  }
  // slice `rank` of the cluster's record; the last cluster to finish slice
  // `rank` (ticket per (KV head, rank)) merges that slice over every record
  if (tid < SLICE) {
    part_o<HD, G>(a, kvh)[((size_t)cl * G + g) * HD + d] = O;
    if (tid == 0) {
      float* ml = part_ml(a, kvh) + ((size_t)cl * 8 + rank) * 2;
      ml[0] = M;
      ml[1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  int* flag = reinterpret_cast<int*>(smf + SM::FLAG);
  int* counter = a.counters + kvh * 8 + rank;
  if (tid == 0) *flag = (atomicAdd(counter, 1) == (int)ncl - 1);
  __syncthreads();
  if (*flag) {
    __threadfence();
    constexpr int NCL_MAX = ATT_MAX_SPLITS / CL;
    if (tid < SLICE) {
      const float* ml = part_ml(a, kvh);
      const float* po = part_o<HD, G>(a, kvh);
      float Mc[NCL_MAX], Lc[NCL_MAX], Oc[NCL_MAX];
#pragma unroll
      for (int c = 0; c < NCL_MAX; ++c) {
        const bool in = (uint32_t)c < ncl;
        Mc[c] = in ? __ldcg(ml + ((size_t)c * 8 + rank) * 2) : -INFINITY;
        Lc[c] = in ? __ldcg(ml + ((size_t)c * 8 + rank) * 2 + 1) : 0.f;
        Oc[c] = in ? __ldcg(po + ((size_t)c * G + g) * HD + d) : 0.f;
      }
      float Mf = -INFINITY;
#pragma unroll
      for (int c = 0; c < NCL_MAX; ++c) Mf = fmaxf(Mf, Mc[c]);
      float Lf = 0.f, Of = 0.f;
#pragma unroll
      for (int c = 0; c < NCL_MAX; ++c) {
        const float w = (Mc[c] == -INFINITY) ? 0.f : expf(Mc[c] - Mf);
        Lf = fmaf(w, Lc[c], Lf);
        Of = fmaf(w, Oc[c], Of);
      }
      a.out[(kvh + KV * g) * HD + d] = (Lf == 0.f) ? 0.f : Of * (1.0f / Lf);
    }
    if (tid == 0) *counter = 0;
  }
  cluster_wait();  // no CTA leaves while a peer may still read its memory
}

}  // namespace adev
}  // namespace shk
