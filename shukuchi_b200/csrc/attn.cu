// attn.cu -- Q8_0 KV cache: bit-exact quantise-on-append and split-K decode attention.
//
// Reference semantics:
//  * q8_quantize_vec (engine/src/kv_cache.c:28-55): per 32 floats
//    scale = maxabs / 127 (0 -> 1), q = clamp(lrintf(v / scale), -127, 127).
//    The kernel uses the same IEEE division and round-half-even conversion, so
//    blocks are bit-identical for identical fp32 input.
//  * op_attention (engine/src/ops.c:406-461) over kv_cache_read_range output:
//    query head h reads KV head h % n_kv_heads, score = dot(q, k) * scale,
//    max-subtracted softmax, out = sum p * v.  Here the softmax is computed
//    online per position range (split) and merged with a log-sum-exp combine by
//    the last CTA of each KV head; results agree to fp32 rounding.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "attn.cuh"
#include "common.cuh"

namespace shk {

KvLayout kv_layout_make(uint32_t n_layers, uint32_t n_kv, uint32_t hd, uint32_t max_seq) {
  KvLayout L{};
  L.n_layers = n_layers;
  L.n_kv = n_kv;
  L.hd = hd;
  L.max_seq = max_seq;
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t q = (size_t)max_seq * hd, s = (size_t)max_seq * (hd / 32) * 4;
  L.kq_off = 0;
  L.ks_off = al(q);
  L.vq_off = L.ks_off + al(s);
  L.vs_off = L.vq_off + al(q);
  L.head_bytes = L.vs_off + al(s);
  return L;
}

size_t attn_part_floats(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t max_splits) {
  return (size_t)n_heads * max_splits * (hd + 2);
}

namespace {

// One warp quantises one 32-element block (lane = element).
__device__ __forceinline__ void q8_block_store(float v, int8_t* q_dst, float* s_dst, int lane) {
  const float amax = warp_max(fabsf(v));
  float scale = amax / 127.0f;
  if (scale == 0.0f) scale = 1.0f;
  int q = __float2int_rn(v / scale);
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  q_dst[lane] = (int8_t)q;
  if (lane == 0) *s_dst = scale;
}

// Appends k_new/v_new of KV head `kvh` at position pos; called by a whole CTA.
__device__ __forceinline__ void append_head(const KvLayout& kv, uint32_t layer, uint32_t kvh,
                                            uint32_t pos, const float* k_new, const float* v_new) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const uint32_t nblk = kv.hd / 32;
  int8_t* reg = kv.region(layer, kvh);
  for (uint32_t b = warp; b < 2 * nblk; b += nw) {
    const bool isv = b >= nblk;
    const uint32_t j = isv ? b - nblk : b;
    const float v = (isv ? v_new : k_new)[kvh * kv.hd + 32 * j + lane];
    int8_t* qd = reg + (isv ? kv.vq_off : kv.kq_off) + (size_t)pos * kv.hd + 32 * j;
    float* sd = reinterpret_cast<float*>(reg + (isv ? kv.vs_off : kv.ks_off)) + (size_t)pos * nblk + j;
    q8_block_store(v, qd, sd, lane);
  }
}

__global__ void kv_append_kernel(KvLayout kv, uint32_t layer, const uint32_t* pos_p,
                                 const float* k, const float* v, int* err) {
  const uint32_t pos = *pos_p;
  if (pos >= kv.max_seq) {
    if (threadIdx.x == 0) set_error(err, DERR_BAD_POS);
    return;
  }
  append_head(kv, layer, blockIdx.x, pos, k, v);
}

constexpr int ATT_THREADS = 128;
constexpr int ATT_TILE = 32;

template <int HD, int G>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int EPL = HD / 32;          // elements per lane in the QK phase
  constexpr int TPD = ATT_THREADS / HD; // threads per output column in the PV phase
  const uint32_t kvh = blockIdx.x, split = blockIdx.y;
  const uint32_t KV = a.kv.n_kv;
  const uint32_t pos = *a.pos;
  if (pos >= a.kv.max_seq) {
    if (threadIdx.x == 0) set_error(a.err, DERR_BAD_POS);
    return;
  }
  const uint32_t seq = pos + 1;
  uint32_t active = (seq + a.min_per_split - 1) / a.min_per_split;
  active = active < 1 ? 1 : (active > gridDim.y ? gridDim.y : active);
  if (split >= active) return;
  const uint32_t per = (seq + active - 1) / active;
  const uint32_t p0 = min(seq, split * per), p1 = min(seq, p0 + per);

  __shared__ float qs[G][HD];
  __shared__ float sc[G][ATT_TILE];
  __shared__ float corr[G];
  __shared__ float mrun[G], lrun[G];
  __shared__ float pv_red[TPD > 1 ? G * HD : 1];
  __shared__ int is_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < G * HD; i += ATT_THREADS) {
    const int g = i / HD, d = i % HD;
    qs[g][d] = a.q[(kvh + KV * g) * HD + d];  // query head h = kvh + KV*g (h % KV == kvh)
  }
  if (tid < G) {
    mrun[tid] = -INFINITY;
    lrun[tid] = 0.f;
  }
  if (a.k_new && pos >= p0 && pos < p1) append_head(a.kv, a.layer, kvh, pos, a.k_new, a.v_new);
  __syncthreads();

  const int8_t* reg = a.kv.region(a.layer, kvh);
  const int8_t* Kq = reg + a.kv.kq_off;
  const float* Ks = reinterpret_cast<const float*>(reg + a.kv.ks_off);
  const int8_t* Vq = reg + a.kv.vq_off;
  const float* Vs = reinterpret_cast<const float*>(reg + a.kv.vs_off);

  // per-lane slice of q for the QK phase
  float qr[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < EPL; ++e) qr[g][e] = qs[g][lane * EPL + e];

  const int d_own = tid % HD, tpar = tid / HD;
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.f;

  for (uint32_t T = p0; T < p1; T += ATT_TILE) {
    const uint32_t nt = min((uint32_t)ATT_TILE, p1 - T);
    // ---- scores: warp per position, lanes across head_dim ----
    for (uint32_t tl = warp; tl < nt; tl += ATT_THREADS / 32) {
      const uint32_t t = T + tl;
      const float ksc = Ks[(size_t)t * (HD / 32) + (lane * EPL) / 32];
      float kv_[EPL];
      if (EPL == 4) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(Kq + (size_t)t * HD + lane * 4);
#pragma unroll
        for (int e = 0; e < 4; ++e) kv_[e] = (float)(int8_t)(w >> (8 * e)) * ksc;
      } else {
        const uint32_t w = *reinterpret_cast<const uint16_t*>(Kq + (size_t)t * HD + lane * 2);
#pragma unroll
        for (int e = 0; e < EPL; ++e) kv_[e] = (float)(int8_t)(w >> (8 * e)) * ksc;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float dsum = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dsum = fmaf(qr[g][e], kv_[e], dsum);
        dsum = warp_sum(dsum);
        if (lane == 0) sc[g][tl] = dsum * a.scale;
      }
    }
    __syncthreads();
    // ---- online softmax update: warp per head ----
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
      const float s = (uint32_t)lane < nt ? sc[g][lane] : -INFINITY;
      const float mt = warp_max(s);
      const float mo = mrun[g];
      const float mn = fmaxf(mo, mt);
      const float p = (uint32_t)lane < nt ? expf(s - mn) : 0.f;
      const float ps = warp_sum(p);
      sc[g][lane] = p;
      if (lane == 0) {
        const float c = (mo == -INFINITY) ? 0.f : expf(mo - mn);
        corr[g] = c;
        lrun[g] = lrun[g] * c + ps;
        mrun[g] = mn;
      }
    }
    __syncthreads();
    // ---- P.V: thread owns column d_own for all G heads ----
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] *= corr[g];
    for (uint32_t tl = tpar; tl < nt; tl += TPD) {
      const uint32_t t = T + tl;
      const float vv = (float)Vq[(size_t)t * HD + d_own] * Vs[(size_t)t * (HD / 32) + d_own / 32];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = fmaf(sc[g][tl], vv, acc[g]);
    }
    __syncthreads();
  }
  if (TPD > 1) {
    if (tpar == 1)
#pragma unroll
      for (int g = 0; g < G; ++g) pv_red[g * HD + d_own] = acc[g];
    __syncthreads();
    if (tpar == 0)
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] += pv_red[g * HD + d_own];
  }

  if (active == 1) {
    if (tpar == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float l = lrun[g];
        const float inv = (l == 0.f) ? 0.f : 1.0f / l;
        a.out[(kvh + KV * g) * HD + d_own] = acc[g] * inv;
      }
    }
    return;
  }
  // ---- write partials, last CTA of this KV head merges ----
  const size_t rec = HD + 2;
  float* part = a.part + ((size_t)kvh * a.max_splits * G) * rec;
  if (tpar == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) part[((size_t)split * G + g) * rec + 2 + d_own] = acc[g];
  }
  if (tid < G) {
    part[((size_t)split * G + tid) * rec + 0] = mrun[tid];
    part[((size_t)split * G + tid) * rec + 1] = lrun[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&a.counters[kvh], 1);
    is_last = (prev == (int)active - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int i = tid; i < G * HD; i += ATT_THREADS) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
    for (uint32_t s = 0; s < active; ++s) M = fmaxf(M, __ldcg(&part[((size_t)s * G + g) * rec]));
    float L = 0.f, O = 0.f;
    for (uint32_t s = 0; s < active; ++s) {
      const float* r = part + ((size_t)s * G + g) * rec;
      const float ms = __ldcg(r);
      const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
      L = fmaf(w, __ldcg(r + 1), L);
      O = fmaf(w, __ldcg(r + 2 + d), O);
    }
    const float inv = (L == 0.f) ? 0.f : 1.0f / L;
    a.out[(kvh + KV * g) * HD + d] = O * inv;
  }
  if (tid == 0) a.counters[kvh] = 0;
}

__global__ void kv_read_range_kernel(KvLayout kv, uint32_t layer, uint32_t start, uint32_t end,
                                     float* k_out, float* v_out) {
  const uint32_t p = start + blockIdx.x;
  if (p >= end) return;
  const uint32_t vd = kv.n_kv * kv.hd, nblk = kv.hd / 32;
  for (uint32_t i = threadIdx.x; i < vd; i += blockDim.x) {
    const uint32_t h = i / kv.hd, e = i % kv.hd;
    const int8_t* reg = kv.region(layer, h);
    const float ks = reinterpret_cast<const float*>(reg + kv.ks_off)[(size_t)p * nblk + e / 32];
    const float vs = reinterpret_cast<const float*>(reg + kv.vs_off)[(size_t)p * nblk + e / 32];
    k_out[(size_t)(p - start) * vd + i] = (float)reg[kv.kq_off + (size_t)p * kv.hd + e] * ks;
    v_out[(size_t)(p - start) * vd + i] = (float)reg[kv.vq_off + (size_t)p * kv.hd + e] * vs;
  }
}

__global__ void kv_read_blocks_kernel(KvLayout kv, uint32_t layer, uint32_t start, uint32_t end,
                                      uint8_t* k_out, uint8_t* v_out) {
  const uint32_t p = start + blockIdx.x;
  if (p >= end) return;
  const uint32_t nblk = kv.hd / 32, tot = kv.n_kv * nblk;
  for (uint32_t i = threadIdx.x; i < tot * Q8_BYTES; i += blockDim.x) {
    const uint32_t blk = i / Q8_BYTES, byte = i % Q8_BYTES;
    const uint32_t h = blk / nblk, j = blk % nblk;
    const int8_t* reg = kv.region(layer, h);
    uint8_t kb, vb;
    if (byte < 4) {
      const uint8_t* ks = reinterpret_cast<const uint8_t*>(reg + kv.ks_off) + ((size_t)p * nblk + j) * 4;
      const uint8_t* vs = reinterpret_cast<const uint8_t*>(reg + kv.vs_off) + ((size_t)p * nblk + j) * 4;
      kb = ks[byte];
      vb = vs[byte];
    } else {
      kb = (uint8_t)reg[kv.kq_off + (size_t)p * kv.hd + 32 * j + byte - 4];
      vb = (uint8_t)reg[kv.vq_off + (size_t)p * kv.hd + 32 * j + byte - 4];
    }
    const size_t o = ((size_t)(p - start) * tot) * Q8_BYTES + i;
    k_out[o] = kb;
    v_out[o] = vb;
  }
}

template <int HD>
cudaError_t attn_launch_hd(const AttnArgs& a, uint32_t G, cudaStream_t st) {
  dim3 grid(a.kv.n_kv, a.max_splits);
  switch (G) {
    case 1: attn_decode_kernel<HD, 1><<<grid, ATT_THREADS, 0, st>>>(a); break;
    case 2: attn_decode_kernel<HD, 2><<<grid, ATT_THREADS, 0, st>>>(a); break;
    case 4: attn_decode_kernel<HD, 4><<<grid, ATT_THREADS, 0, st>>>(a); break;
    case 8: attn_decode_kernel<HD, 8><<<grid, ATT_THREADS, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t attn_decode_launch(const AttnArgs& a, cudaStream_t stream) {
  if (a.kv.n_kv == 0 || a.n_heads % a.kv.n_kv) return cudaErrorInvalidValue;
  const uint32_t G = a.n_heads / a.kv.n_kv;
  if (a.kv.hd == 64) return attn_launch_hd<64>(a, G, stream);
  if (a.kv.hd == 128) return attn_launch_hd<128>(a, G, stream);
  return cudaErrorInvalidValue;
}

cudaError_t kv_append_launch(const KvLayout& kv, uint32_t layer, const uint32_t* pos,
                             const float* k, const float* v, int* err, cudaStream_t stream) {
  kv_append_kernel<<<kv.n_kv, 128, 0, stream>>>(kv, layer, pos, k, v, err);
  return cudaGetLastError();
}

cudaError_t kv_read_range_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t end,
                                 float* k_out, float* v_out, cudaStream_t stream) {
  if (end <= start) return cudaSuccess;
  kv_read_range_kernel<<<end - start, 256, 0, stream>>>(kv, layer, start, end, k_out, v_out);
  return cudaGetLastError();
}

cudaError_t kv_read_blocks_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t end,
                                  uint8_t* k_out, uint8_t* v_out, cudaStream_t stream) {
  if (end <= start) return cudaSuccess;
  kv_read_blocks_kernel<<<end - start, 256, 0, stream>>>(kv, layer, start, end, k_out, v_out);
  return cudaGetLastError();
}

}  // namespace shk
