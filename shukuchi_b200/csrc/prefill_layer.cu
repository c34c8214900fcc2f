// prefill_layer.cu -- row-batched glue kernels of the prompt prefill.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "attn_dev.cuh"
#include "common.cuh"
#include "prefill_layer.cuh"

namespace shk {
namespace {

constexpr int PF_ATT_WARPS = 4;

// One row per CTA: the reference's op_rmsnorm expression order per row
// (sum of squares, 1/sqrt(mean + 1e-5), (x * inv) * w).
__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    float* __restrict__ y, uint32_t d) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * d;
  float* yr = y + (size_t)blockIdx.x * d;
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (uint32_t k = 0; k < blockDim.x / 32; ++k) tot += red[k];
  const float inv = 1.0f / sqrtf(tot / (float)d + 1e-5f);
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) yr[i] = (xr[i] * inv) * w[i];
}

// Row blockIdx.y at position pos0 + blockIdx.y; angle pos * freq in fp32 as
// the reference computes it.
__global__ void rope_rows_kernel(float* qk, uint32_t n_heads, uint32_t hd, uint32_t pos0, const float* freq) {
  const uint32_t pairs = n_heads * (hd / 2);
  const float pos = (float)(pos0 + blockIdx.y);
  float* row = qk + (size_t)blockIdx.y * n_heads * hd;
  for (uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) {
    const uint32_t h = p / (hd / 2), i = 2 * (p % (hd / 2));
    const float ang = pos * freq[i >> 1];
    const float c = cosf(ang), s = sinf(ang);
    float* v = row + (size_t)h * hd + i;
    const float a = v[0], b = v[1];
    v[0] = a * c - b * s;
    v[1] = a * s + b * c;
  }
}

// (KV head blockIdx.x, query row blockIdx.y): one split over [0, pos0 + row],
// the decode attention's item (attn_dev.cuh) with this row's q, output and
// position; the long-range loop for ranges of 256+ positions.
template <int HD, int G>
__global__ void __launch_bounds__(32 * PF_ATT_WARPS) attn_prefill_kernel(const __grid_constant__ AttnArgs a,
                                                                         const uint32_t* iota, uint32_t pos0) {
  __shared__ __align__(16) float sm[adev::AttnSmem<HD, G, PF_ATT_WARPS>::FLOATS_LONG];
  AttnArgs b = a;
  const size_t qrow = (size_t)a.n_heads * HD;
  b.pos = iota + pos0 + blockIdx.y;
  b.q = a.q + blockIdx.y * qrow;
  b.out = a.out + blockIdx.y * qrow;
  b.k_new = nullptr;
  b.v_new = nullptr;
  adev::attn_item<HD, G, PF_ATT_WARPS, true>(b, blockIdx.x, 0, 1, sm);
}

template <int HD>
cudaError_t attn_prefill_hd(const AttnArgs& a, uint32_t G, const uint32_t* iota, uint32_t pos0, uint32_t T,
                            cudaStream_t st) {
  const dim3 grid(a.kv.n_kv, T), block(32 * PF_ATT_WARPS);
  switch (G) {
    case 1: attn_prefill_kernel<HD, 1><<<grid, block, 0, st>>>(a, iota, pos0); break;
    case 2: attn_prefill_kernel<HD, 2><<<grid, block, 0, st>>>(a, iota, pos0); break;
    case 4: attn_prefill_kernel<HD, 4><<<grid, block, 0, st>>>(a, iota, pos0); break;
    case 8: attn_prefill_kernel<HD, 8><<<grid, block, 0, st>>>(a, iota, pos0); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t rmsnorm_rows_launch(const float* x, const float* w, float* y, uint32_t d, uint32_t T,
                                cudaStream_t st) {
  if (!T) return cudaSuccess;
  rmsnorm_rows_kernel<<<T, 1024, 0, st>>>(x, w, y, d);
  return cudaGetLastError();
}

cudaError_t rope_rows_launch(float* qk, uint32_t n_heads, uint32_t hd, uint32_t pos0, uint32_t T,
                             const float* freq, cudaStream_t st) {
  if (!T) return cudaSuccess;
  const uint32_t pairs = n_heads * (hd / 2);
  rope_rows_kernel<<<dim3((pairs + 255) / 256, T), 256, 0, st>>>(qk, n_heads, hd, pos0, freq);
  return cudaGetLastError();
}

cudaError_t attn_prefill_launch(const AttnArgs& a, const uint32_t* iota, uint32_t pos0, uint32_t T,
                                cudaStream_t st) {
  if (!T || a.kv.n_kv == 0 || a.n_heads % a.kv.n_kv || T > 65535) return cudaErrorInvalidValue;
  const uint32_t G = a.n_heads / a.kv.n_kv;
  if (a.kv.hd == 64) return attn_prefill_hd<64>(a, G, iota, pos0, T, st);
  if (a.kv.hd == 128) return attn_prefill_hd<128>(a, G, iota, pos0, T, st);
  return cudaErrorInvalidValue;
}

}  // namespace shk
