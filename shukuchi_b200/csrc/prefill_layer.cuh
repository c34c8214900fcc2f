// prefill_layer.cuh -- the row-batched glue of a prompt prefill (host API).
//
// A prompt of T tokens runs through each layer as matrices of T rows: the
// projections on the tensor-core prefill matmul (prefill.cu), and between
// them the kernels below, one row (token) per CTA or element range: RMSNorm
// of every row, RoPE of every row at its own position, the causal attention
// of every row over the Q8_0 cache (after the T new K/V rows are appended),
// residual adds and SwiGLU over the whole T x width block.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attn.cuh"

namespace shk {

// y[r] = rmsnorm(x[r]) * w for rows r < T of width d (engine/src/ops.c:195-214).
cudaError_t rmsnorm_rows_launch(const float* x, const float* w, float* y, uint32_t d, uint32_t T,
                                cudaStream_t st);
// RoPE of T rows of n_heads x hd, row r at position pos0 + r (engine/src/ops.c:216-238).
cudaError_t rope_rows_launch(float* qk, uint32_t n_heads, uint32_t hd, uint32_t pos0, uint32_t T,
                             const float* freq, cudaStream_t st);
// Attention of query rows t < T (row t at position pos0 + t) over cache
// positions [0, pos0 + t], one CTA per (KV head, row); a.q / a.out hold T
// rows of n_heads * hd; the K/V rows are already in the cache.  iota: a
// device array with iota[p] == p.
cudaError_t attn_prefill_launch(const AttnArgs& a, const uint32_t* iota, uint32_t pos0, uint32_t T,
                                cudaStream_t st);

}  // namespace shk
