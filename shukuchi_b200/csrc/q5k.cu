// q5k.cu -- batch-1 Q5_K dequantise-matvec over GGUF rows (dp4a on fixed-point x).
//
// Reference semantics: op_matmul_q5_k (engine/src/ops.c:316-359) over
// dequantize_row_q5_k (:144-165), element order and block layout as in q5k.cuh.
//
// Design.  Each CTA first turns x (optionally x * RMSNorm weights) into 24-bit
// fixed point per 256-element block, x = X_b * (l0 + 256 l1 + 65536 l2) with
// X_b a power of two and balanced signed-byte limbs, stored in shared memory
// in the order the quants come in: lane l of a warp owns elements 8l..8l+7 of
// a block, whose low 4 bits are the 4 bytes qs[4l..4l+3] (even elements in
// the low nibbles, odd in the high) and whose fifth bits are qh[l].  A warp
// takes a pair of rows ((2i, 2i+1), or row i of gate and up) over one K slice;
// per block and row a lane builds two words of 5-bit quants (even and odd
// elements), takes 6 dp4a against the limb words (Horner in int32: |sum| <
// 2^31 since |q| < 32 and |l2| <= 64) and adds d*sc * X_b * sum - dmin*m *
// (sum of its 8 x) in fp32.  The scale and min of sub-block (lane & 7) of
// block (lane >> 3) are computed once per 4 blocks and fetched by shuffles.
// K slices of a pair are summed in shared memory in slice order, so the
// result does not depend on timing.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "q5k.cuh"

namespace shk {
namespace {

constexpr uint32_t XBLK_BYTES = 912;  // per x block: limbs 0/1 (512), limb 2 (256), sums (128), X_b (16)

__device__ __forceinline__ void q5_limbs(int v, int& l0, int& l1, int& l2) {
  l0 = (int)(int8_t)(v & 0xFF);
  const int r = (v - l0) >> 8;
  l1 = (int)(int8_t)(r & 0xFF);
  l2 = (r - l1) >> 8;
}
__device__ __forceinline__ uint32_t q5_pack(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) |
         ((uint32_t)(d & 0xFF) << 24);
}
// Fifth bits of the even (par 0) or odd (par 1) elements of a lane's eight,
// moved to bit 4 of bytes 0..3: source bits 0, 2, 4, 6 -> 4, 12, 20, 28 (the
// product's other terms land on bits that the mask drops, without carries
// into the kept ones).
__device__ __forceinline__ uint32_t q5_hbits(uint32_t h, int par) {
  return (((h >> par) & 0x55u) * 0x410410u) & 0x10101010u;
}

__device__ __forceinline__ const Q5Seg& q5_seg(const Q5Args& a, uint32_t p) {
  uint32_t si = 0;
  while (si + 1 < a.nseg && p >= a.seg[si + 1].pair0) ++si;
  return a.seg[si];
}

__device__ __forceinline__ void q5_epilogue(const Q5Args& a, uint32_t p, float v0, float v1) {
  const Q5Seg& sg = q5_seg(a, p);
  const uint32_t lp = p - sg.pair0;
  if (sg.w2) {
    const float sig = 1.0f / (1.0f + expf(-v0));  // SwiGLU (engine/src/ops.c:491-496)
    sg.y[lp] = (v0 * sig) * v1;
    return;
  }
  const uint32_t r0 = 2 * lp, r1 = r0 + 1;
  if (sg.epi == EPI_ROPE) {
    if (r1 < sg.m) {
      const float ps = (float)__ldcg(a.pos);
      const uint32_t i = r0 % sg.rope_hd;
      const float ang = ps * a.rope_freq[i >> 1];  // engine/src/ops.c:227-228
      const float c = cosf(ang), sn = sinf(ang);
      sg.y[r0] = v0 * c - v1 * sn;
      sg.y[r1] = v0 * sn + v1 * c;
    }
    return;
  }
  if (sg.epi == EPI_ADD) {
    sg.y[r0] = __ldcg(&sg.y[r0]) + v0;
    if (r1 < sg.m) sg.y[r1] = __ldcg(&sg.y[r1]) + v1;
  } else {
    sg.y[r0] = v0;
    if (r1 < sg.m) sg.y[r1] = v1;
  }
}

template <bool NORM>
__global__ void __launch_bounds__(Q5_THREADS) q5k_kernel(const __grid_constant__ Q5Args a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t NB = a.k / 256, NBP = (NB + Q5_BPI - 1) / Q5_BPI * Q5_BPI;
  uint4* xa = reinterpret_cast<uint4*>(smem);              // [NBP][32]: l0 even, l0 odd, l1 even, l1 odd
  uint2* xc = reinterpret_cast<uint2*>(smem + 512 * NBP);  // [NBP][32]: l2 even, l2 odd
  float* xs = reinterpret_cast<float*>(smem + 768 * NBP);  // [NBP][32]: sum of the lane's 8 x
  float* xb = reinterpret_cast<float*>(smem + 896 * NBP);  // [NBP] X_b (NaN: non-finite block)
  float* part = reinterpret_cast<float*>(smem + XBLK_BYTES * NBP);  // [Q5_WARPS][2]
  float* red = part + 2 * Q5_WARPS;                                  // [Q5_WARPS]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_trigger();
  pdl_wait();  // x (and the residual) come from the previous kernel

  float ss = 0.f;
  for (uint32_t kb = warp; kb < NBP; kb += Q5_WARPS) {
    const size_t slot = (size_t)kb * 32 + lane;
    if (kb >= NB) {  // padding blocks: zero limbs, sums and X_b
      xa[slot] = make_uint4(0u, 0u, 0u, 0u);
      xc[slot] = make_uint2(0u, 0u);
      xs[slot] = 0.f;
      if (lane == 0) xb[kb] = 0.f;
      continue;
    }
    const float4* src = reinterpret_cast<const float4*>(a.x + 256 * (size_t)kb + 8 * lane);
    const float4 t0 = __ldcg(src), t1 = __ldcg(src + 1);
    float v[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
    if (NORM) {
      const float4* wn = reinterpret_cast<const float4*>(a.norm_w + 256 * (size_t)kb + 8 * lane);
      const float4 w0 = __ldg(wn), w1 = __ldg(wn + 1);
      const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss = fmaf(v[e], v[e], ss);
        v[e] *= w[e];
      }
    }
    float amax = 0.f;
    bool fin = true;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      amax = fmaxf(amax, fabsf(v[e]));
      fin = fin && isfinite(v[e]);
    }
    amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
    fin = __all_sync(0xffffffffu, fin);
    // X_b = 2^(f-21) with amax in [2^f, 2^(f+1)): |x / X_b| <= 2^22
    const int e8 = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
    const int f = amax > 0.f ? max(e8 - 127, -104) : 0;
    const float xbv = fin ? __uint_as_float((uint32_t)(f - 21 + 127) << 23) : __int_as_float(0x7fc00000);
    const float inv_xb = __uint_as_float((uint32_t)(21 - f + 127) << 23);
    int L[3][8];
#pragma unroll
    for (int e = 0; e < 8; ++e) q5_limbs(fin ? __float2int_rn(v[e] * inv_xb) : 0, L[0][e], L[1][e], L[2][e]);
    xa[slot] = make_uint4(q5_pack(L[0][0], L[0][2], L[0][4], L[0][6]), q5_pack(L[0][1], L[0][3], L[0][5], L[0][7]),
                          q5_pack(L[1][0], L[1][2], L[1][4], L[1][6]), q5_pack(L[1][1], L[1][3], L[1][5], L[1][7]));
    xc[slot] = make_uint2(q5_pack(L[2][0], L[2][2], L[2][4], L[2][6]), q5_pack(L[2][1], L[2][3], L[2][5], L[2][7]));
    xs[slot] = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    if (lane == 0) xb[kb] = xbv;
  }
  if (NORM) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
  }
  __syncthreads();
  float osc = 1.f;
  if (NORM) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < Q5_WARPS; ++w) tot += red[w];
    osc = 1.0f / sqrtf(tot / (float)a.k + 1e-5f);  // engine/src/ops.c:195-214
  }

  const uint32_t S = a.ks, ppg = Q5_WARPS / S, slice = warp % S;
  const uint32_t groups = (a.total_pairs + ppg - 1) / ppg;
  const size_t rb = (size_t)NB * Q5K_BYTES;
  for (uint32_t g = blockIdx.x; g < groups; g += gridDim.x) {
    const uint32_t p = g * ppg + warp / S;
    float acc0 = 0.f, acc1 = 0.f;
    if (p < a.total_pairs) {
      const Q5Seg& sg = q5_seg(a, p);
      const uint32_t lp = p - sg.pair0;
      const uint8_t* r0;
      const uint8_t* r1;
      if (sg.w2) {
        r0 = sg.w + lp * rb;
        r1 = sg.w2 + lp * rb;
      } else {
        r0 = sg.w + 2 * (size_t)lp * rb;
        r1 = 2 * lp + 1 < sg.m ? r0 + rb : nullptr;
      }
      const uint32_t lo = slice * a.nbs, hi = min(NB, lo + a.nbs);
      const uint32_t sb = lane & 7, sh = 8 * (sb & 3);
#pragma unroll 1
      for (uint32_t b0 = lo; b0 < hi; b0 += Q5_BPI) {
        uint4 hd[2];
        uint32_t W[2][Q5_BPI], H[2][Q5_BPI];
        const uint32_t hb = b0 + (lane >> 3);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint8_t* rp = j ? r1 : r0;
          hd[j] = make_uint4(0u, 0u, 0u, 0u);
          if (rp && hb < hi) hd[j] = __ldcs(reinterpret_cast<const uint4*>(rp + (size_t)hb * Q5K_BYTES));
#pragma unroll
          for (int i = 0; i < Q5_BPI; ++i) {
            W[j][i] = 0u;
            H[j][i] = 0u;
            if (rp && b0 + i < hi) {
              const uint8_t* blk = rp + (size_t)(b0 + i) * Q5K_BYTES;
              W[j][i] = __ldcs(reinterpret_cast<const unsigned int*>(blk + 48 + 4 * lane));
              H[j][i] = __ldcs(blk + 16 + lane);
            }
          }
        }
        // this lane's sub-block (lane & 7) of block hb: d*sc and dmin*m
        // (get_scale_min_k4, engine/src/ops.c:107-115); zero headers give 0
        float fs[2], fm[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint32_t w1 = hd[j].y, w2 = hd[j].z, w3 = hd[j].w;
          uint32_t sc, mn;
          if (sb < 4) {
            sc = (w1 >> sh) & 63u;
            mn = (w2 >> sh) & 63u;
          } else {
            const uint32_t q = (w3 >> sh) & 0xFFu;
            sc = (q & 0xFu) | (((w1 >> sh) >> 6 & 3u) << 4);
            mn = (q >> 4) | (((w2 >> sh) >> 6 & 3u) << 4);
          }
          fs[j] = ref_half(hd[j].x & 0xFFFFu) * (float)sc;
          fm[j] = ref_half(hd[j].x >> 16) * (float)mn;
        }
#pragma unroll
        for (int i = 0; i < Q5_BPI; ++i) {
          const size_t slot = (size_t)(b0 + i) * 32 + lane;
          const uint4 la = xa[slot];
          const uint2 lc = xc[slot];
          const float xsum = xs[slot], xbv = xb[b0 + i];
          const int srcl = i * 8 + (lane >> 2);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float d1 = __shfl_sync(0xffffffffu, fs[j], srcl);
            const float m1 = __shfl_sync(0xffffffffu, fm[j], srcl);
            const int qe = (int)((W[j][i] & 0x0F0F0F0Fu) | q5_hbits(H[j][i], 0));
            const int qo = (int)(((W[j][i] >> 4) & 0x0F0F0F0Fu) | q5_hbits(H[j][i], 1));
            int t = __dp4a(qe, (int)lc.x, 0);
            t = __dp4a(qo, (int)lc.y, t);
            t = __dp4a(qe, (int)la.z, t * 256);
            t = __dp4a(qo, (int)la.w, t);
            t = __dp4a(qe, (int)la.x, t * 256);
            t = __dp4a(qo, (int)la.y, t);
            const float v = d1 * (xbv * (float)t) - m1 * xsum;
            if (j == 0)
              acc0 += v;
            else
              acc1 += v;
          }
        }
      }
    }
    acc0 = warp_sum(acc0);
    acc1 = warp_sum(acc1);
    if (S == 1) {
      if (lane == 0 && p < a.total_pairs) q5_epilogue(a, p, acc0 * osc, acc1 * osc);
    } else {
      if (lane == 0) {
        part[2 * warp] = acc0;
        part[2 * warp + 1] = acc1;
      }
      __syncthreads();
      if (slice == 0 && lane == 0 && p < a.total_pairs) {
        float v0 = 0.f, v1 = 0.f;
        for (uint32_t s = 0; s < S; ++s) {
          v0 += part[2 * (warp + s)];
          v1 += part[2 * (warp + s) + 1];
        }
        q5_epilogue(a, p, v0 * osc, v1 * osc);
      }
      __syncthreads();
    }
  }
}

size_t q5_smem(uint32_t k) {
  const uint32_t nb = k / 256, nbp = (nb + Q5_BPI - 1) / Q5_BPI * Q5_BPI;
  return (size_t)XBLK_BYTES * nbp + 4 * 3 * Q5_WARPS;
}

}  // namespace

cudaError_t q5k_init() {
  const int mx = 227 * 1024;
  cudaError_t e = cudaFuncSetAttribute(q5k_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(q5k_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  return e;
}

int q5k_plan(Q5Plan& p, const Q5Mat* mats, int nmats, uint32_t k, const float* x, const float* norm_w,
             const uint32_t* pos, const float* rope_freq, int* err, int num_sms) {
  if (nmats < 1 || nmats > Q5_MAX_SEGS || k == 0 || k % 256 || !x || !err || num_sms < 1) return -1;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(norm_w) & 15)) return -1;
  const size_t smem = q5_smem(k);
  if (smem > 227u * 1024u) return -2;
  Q5Args& a = p.args;
  a = Q5Args{};
  a.nseg = nmats;
  a.k = k;
  a.x = x;
  a.norm_w = norm_w;
  a.pos = pos;
  a.rope_freq = rope_freq;
  a.err = err;
  uint32_t total = 0;
  for (int i = 0; i < nmats; ++i) {
    const Q5Mat& mt = mats[i];
    Q5Seg& g = a.seg[i];
    if (!mt.w || !mt.y || mt.m == 0 || (reinterpret_cast<uintptr_t>(mt.w) & 15) ||
        (reinterpret_cast<uintptr_t>(mt.w2) & 15))
      return -1;
    if (mt.w2 ? mt.epi != EPI_SWIGLU : (mt.epi > EPI_ROPE)) return -1;
    if (mt.epi == EPI_ROPE && (!pos || !rope_freq || mt.rope_hd == 0 || (mt.rope_hd & 1) || (mt.m & 1))) return -1;
    g.w = static_cast<const uint8_t*>(mt.w);
    g.w2 = static_cast<const uint8_t*>(mt.w2);
    g.y = mt.y;
    g.m = mt.m;
    g.epi = mt.epi;
    g.rope_hd = mt.rope_hd;
    g.pairs = mt.w2 ? mt.m : (mt.m + 1) / 2;
    g.pair0 = total;
    if ((uint64_t)total + g.pairs > 0xFFFFFFFFull) return -1;
    total += g.pairs;
  }
  a.total_pairs = total;
  int bps = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, norm_w ? q5k_kernel<true> : q5k_kernel<false>,
                                                    Q5_THREADS, smem) != cudaSuccess ||
      bps < 1)
    return -2;
  // K slices: enough warps in flight to cover the GPU, each slice >= Q5_BPI blocks
  const uint32_t nb = k / 256;
  const uint64_t target = (uint64_t)num_sms * bps * Q5_WARPS;
  uint32_t ks = 1;
  while (ks < 8 && (uint64_t)total * ks < target && (nb + 2 * ks - 1) / (2 * ks) >= (uint32_t)Q5_BPI) ks *= 2;
  a.ks = ks;
  a.nbs = ((nb + ks - 1) / ks + Q5_BPI - 1) / Q5_BPI * Q5_BPI;
  const uint64_t groups = ((uint64_t)total + (Q5_WARPS / ks) - 1) / (Q5_WARPS / ks);
  p.grid = (int)std::min<uint64_t>(groups, (uint64_t)num_sms * bps);
  p.smem = smem;
  return 0;
}

cudaError_t q5k_launch(const Q5Plan& p, cudaStream_t stream) {
  if (p.args.norm_w)
    return launch_k(q5k_kernel<true>, dim3(p.grid), dim3(Q5_THREADS), p.smem, stream, p.args);
  return launch_k(q5k_kernel<false>, dim3(p.grid), dim3(Q5_THREADS), p.smem, stream, p.args);
}

}  // namespace shk
