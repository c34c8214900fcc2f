// q5k.cuh -- batch-1 Q5_K dequantise-matvec (host-side plan API).
//
// Reference semantics: op_matmul_q5_k (engine/src/ops.c:316-359) over
// dequantize_row_q5_k (:144-165).  The reference's Q5_K block is 176 bytes,
// {u16 d, u16 dmin, u8 scales[12], u8 qh[32], u8 qs[128]}, and orders the
// elements its own way (not ggml's): element i of a 256-block takes its low
// 4 bits from qs[i/2] (low nibble for even i, high for odd) and its fifth bit
// from bit i%8 of qh[i/8]; value = d*sc*q5 - dmin*m with the 6-bit scale and
// min of sub-block i/32 (get_scale_min_k4, :107-115).
//
// Weights stay in the GGUF row layout (rows of k/256 blocks, contiguous).
// Epilogues as the other matvecs (GemvEpi): store, residual add, RoPE on
// (2i, 2i+1) row pairs, SwiGLU over a gate/up pair; optional RMSNorm of x.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace shk {

constexpr uint32_t Q5K_BYTES = 176;
constexpr int Q5_MAX_SEGS = 4;
constexpr int Q5_WARPS = 8;
constexpr int Q5_THREADS = 32 * Q5_WARPS;
constexpr int Q5_BPI = 4;  // blocks per row per inner iteration

struct Q5Mat {
  const void* w;   // m rows x k/256 Q5_K blocks
  const void* w2;  // non-null: the up matrix of a gate/up pair (SwiGLU)
  float* y;
  uint32_t m;
  uint8_t epi;     // GemvEpi (not EPI_TP)
  uint32_t rope_hd;
};

struct Q5Seg {
  const uint8_t* w;
  const uint8_t* w2;
  float* y;
  uint32_t m;
  uint32_t pairs;    // row pairs (2i, 2i+1), or rows of a gate/up pair
  uint32_t pair0;    // global index of the first pair
  uint32_t rope_hd;
  uint32_t epi;
};

struct Q5Args {
  Q5Seg seg[Q5_MAX_SEGS];
  uint32_t nseg;
  uint32_t k;
  uint32_t total_pairs;
  uint32_t ks;             // K slices per pair (1, 2, 4 or 8): warps of one CTA
  uint32_t nbs;            // blocks per slice (a multiple of Q5_BPI)
  const float* x;
  const float* norm_w;     // optional RMSNorm weights (eps 1e-5), applied as an output scale
  const uint32_t* pos;     // EPI_ROPE position (device)
  const float* rope_freq;  // EPI_ROPE: freq[i/2] = powf(1/theta, i/head_dim)
  int* err;
};

struct Q5Plan {
  Q5Args args;
  int grid = 0;
  size_t smem = 0;
};

// Returns 0, -1 on invalid arguments (alignment: w 16 B, x and norm_w 16 B),
// -2 when k is too large for the shared-memory x region.
int q5k_plan(Q5Plan& p, const Q5Mat* mats, int nmats, uint32_t k, const float* x, const float* norm_w,
             const uint32_t* pos, const float* rope_freq, int* err, int num_sms);
cudaError_t q5k_init();
cudaError_t q5k_launch(const Q5Plan& p, cudaStream_t stream);

}  // namespace shk
