// glue.cu -- embedding lookup, first-index argmax and stand-alone glue ops.
//
// The decode step fuses RMSNorm, RoPE, SwiGLU and the residual adds into the
// GEMV prologue/epilogues (gemv.cu); the stand-alone kernels here back the
// op-level C entry points (ops.h equivalents) and the token-feedback path.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "glue.cuh"
#include "glue_dev.cuh"

namespace shk {
namespace {
using namespace gldev;

// op_embed (engine/src/ops.c:533-577).  The token id is read from device
// memory so a captured graph can feed back the argmax.
// step (optional): a device step counter advanced once per token (the epoch of
// the tensor-parallel exchange).
__global__ void embed_kernel(const uint8_t* __restrict__ table, uint32_t dtype,
                             const uint32_t* __restrict__ tok_p, uint32_t n_vocab, float* out,
                             uint32_t n_embd, int* err, uint32_t* step) {
  pdl_trigger();
  pdl_wait();
  if (step && blockIdx.x == 0 && threadIdx.x == 0) *step += 1;
  const uint32_t tok = *tok_p;
  if (tok >= n_vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_error(err, DERR_BAD_TOKEN);
    return;
  }
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n_embd; e += gridDim.x * blockDim.x)
    out[e] = embed_elem(table, dtype, tok, n_embd, e);
}

// First index of the maximum (engine/src/engine.c:424-431).  Block partials
// then the last block merges.  Optionally advances the device position counter
// (token feedback in a captured step).
// With idx_off / val_out (a tensor-parallel rank's slice of the vocabulary):
// writes idx_off + local index and the maximum's value, for the merge over
// ranks below.
constexpr int AM_THREADS = 512;
__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const float* __restrict__ x, uint32_t n,
                                                            float* part_v, uint32_t* part_i,
                                                            int* counter, uint32_t* tok_out,
                                                            uint32_t* pos_inc, uint32_t idx_off,
                                                            float* val_out) {
  __shared__ float sv[AM_THREADS / 32];
  __shared__ uint32_t si[AM_THREADS / 32];
  __shared__ int last;
  pdl_trigger();
  pdl_wait();
  // 64-bit: n + gridDim.x and blockIdx.x * per may pass 2^32 for n near it
  const uint64_t per = ((uint64_t)n + gridDim.x - 1) / gridDim.x;
  const uint32_t lo = (uint32_t)min((uint64_t)n, blockIdx.x * per);
  const uint32_t hi = (uint32_t)min((uint64_t)n, (uint64_t)lo + per);
  float bv;
  uint32_t bi;
  am_block<AM_THREADS>(x, lo, hi, sv, si, [] { __syncthreads(); }, bv, bi);
  if (threadIdx.x == 0) {
    part_v[blockIdx.x] = bv;
    part_i[blockIdx.x] = bi;
    __threadfence();
    last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the reference keeps index 0 when x[0] is NaN (only the slice holding the
  // vocabulary's index 0 can see it)
  const bool x0_nan = idx_off == 0 && n > 0 && isnan(__ldcg(x));
  float v;
  const uint32_t ix = am_merge_par<AM_THREADS>(part_v, part_i, gridDim.x, x0_nan, sv, si,
                                               [] { __syncthreads(); }, &v);
  if (threadIdx.x != 0) return;
  *tok_out = idx_off + ix;
  if (val_out) *val_out = v;
  if (pos_inc) *pos_inc += 1;
  *counter = 0;
}

// Merge of the ranks' (value, global index) pairs, rank order, with the same
// first-maximum rule as the blocks above: the vocabulary slices are in rank
// order, so the result is the argmax of the whole logits vector.
__global__ void argmax_ranks_kernel(const uint32_t* __restrict__ pairs, int world, uint32_t* tok_out,
                                    uint32_t* pos_inc) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0) return;
  float v = __uint_as_float(__ldcg(&pairs[0]));
  uint32_t ix = __ldcg(&pairs[1]);
  for (int r = 1; r < world; ++r) {
    const float ov = __uint_as_float(__ldcg(&pairs[2 * r]));
    const uint32_t oi = __ldcg(&pairs[2 * r + 1]);
    if (am_better(v, ix, ov, oi)) {
      v = ov;
      ix = oi;
    }
  }
  *tok_out = ix;
  if (pos_inc) *pos_inc += 1;
}

// op_rmsnorm, n = 1 (engine/src/ops.c:195-214)
__global__ void rmsnorm_kernel(const float* x, const float* w, float* y, uint32_t d) {
  __shared__ float red[32];
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (uint32_t w2 = 0; w2 < blockDim.x / 32; ++w2) tot += red[w2];
  const float inv = 1.0f / sqrtf(tot / (float)d + 1e-5f);
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) y[i] = (x[i] * inv) * w[i];
}

// op_rope (engine/src/ops.c:216-238)
// freq[i/2] = powf(1/theta, i/hd) is computed on the host with the C library,
// so pos * freq matches the reference's fp32 angle exactly.
__global__ void rope_kernel(float* qk, uint32_t n_heads, uint32_t hd, const uint32_t* pos_p,
                            const float* freq) {
  const uint32_t pairs = n_heads * (hd / 2);
  const uint32_t pos = *pos_p;
  for (uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) {
    const uint32_t h = p / (hd / 2), i = 2 * (p % (hd / 2));
    const float ang = (float)pos * freq[i >> 1];
    const float c = cosf(ang), s = sinf(ang);
    float* v = qk + (size_t)h * hd + i;
    const float a = v[0], b = v[1];
    v[0] = a * c - b * s;
    v[1] = a * s + b * c;
  }
}

// SwiGLU (engine/src/ops.c:491-496)
__global__ void swiglu_kernel(const float* g, const float* u, float* h, uint32_t n) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float gt = g[i];
    const float sig = 1.0f / (1.0f + expf(-gt));
    h[i] = (gt * sig) * u[i];
  }
}

// A wait that nothing satisfies: an mbarrier that never completes, waited on
// with the same bounded wait as the GEMV ring (budget_ns instead of 1 s).  It
// must end with DERR_TIMEOUT_FULL in the error word and leave the context
// usable.
__global__ void wait_selftest_kernel(int* err, uint64_t budget_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, err, DERR_TIMEOUT_FULL, budget_ns);
  __syncthreads();
}

__global__ void add_kernel(float* y, const float* x, uint32_t n) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[i] = y[i] + x[i];
}

}  // namespace

cudaError_t embed_launch(const void* table, uint32_t dtype, const uint32_t* tok, uint32_t n_vocab,
                         float* out, uint32_t n_embd, int* err, cudaStream_t st, uint32_t* step) {
  return launch_k(embed_kernel, dim3((n_embd + 255) / 256), dim3(256), 0, st,
                  static_cast<const uint8_t*>(table), dtype, tok, n_vocab, out, n_embd, err, step);
}

int argmax_blocks(uint32_t n) {
  const uint64_t b = ((uint64_t)n + 4095) / 4096;  // 64-bit: n + 4095 may pass 2^32
  return (int)(b < 1 ? 1 : (b > 148 ? 148 : b));
}

cudaError_t argmax_launch(const float* x, uint32_t n, float* part_v, uint32_t* part_i, int* counter,
                          uint32_t* tok_out, uint32_t* pos_inc, cudaStream_t st, uint32_t idx_off,
                          float* val_out) {
  return launch_k(argmax_kernel, dim3(argmax_blocks(n)), dim3(AM_THREADS), 0, st, x, n, part_v, part_i,
                  counter, tok_out, pos_inc, idx_off, val_out);
}

cudaError_t argmax_ranks_launch(const uint32_t* pairs, int world, uint32_t* tok_out, uint32_t* pos_inc,
                                cudaStream_t st) {
  return launch_k(argmax_ranks_kernel, dim3(1), dim3(32), 0, st, pairs, world, tok_out, pos_inc);
}

cudaError_t wait_selftest_launch(int* err, uint64_t budget_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(err, budget_ns);
  return cudaGetLastError();
}

bool& pdl_enabled() {
  static thread_local bool on = false;
  return on;
}

cudaError_t rmsnorm_launch(const float* x, const float* w, float* y, uint32_t d, cudaStream_t st) {
  rmsnorm_kernel<<<1, 1024, 0, st>>>(x, w, y, d);
  return cudaGetLastError();
}

cudaError_t rope_launch(float* qk, uint32_t n_heads, uint32_t hd, const uint32_t* pos,
                        const float* freq, cudaStream_t st) {
  const uint32_t pairs = n_heads * (hd / 2);
  rope_kernel<<<(pairs + 255) / 256, 256, 0, st>>>(qk, n_heads, hd, pos, freq);
  return cudaGetLastError();
}

void rope_freq_table(float theta, uint32_t hd, float* out) {
  const float inv_theta = 1.0f / theta;
  for (uint32_t i = 0; i + 1 < hd; i += 2) out[i / 2] = powf(inv_theta, (float)i / (float)hd);
}

cudaError_t swiglu_launch(const float* g, const float* u, float* h, uint32_t n, cudaStream_t st) {
  swiglu_kernel<<<(n + 255) / 256, 256, 0, st>>>(g, u, h, n);
  return cudaGetLastError();
}

cudaError_t add_launch(float* y, const float* x, uint32_t n, cudaStream_t st) {
  add_kernel<<<(n + 255) / 256, 256, 0, st>>>(y, x, n);
  return cudaGetLastError();
}

}  // namespace shk
