// glue.cuh -- embedding, argmax and stand-alone glue kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace shk {

cudaError_t embed_launch(const void* table, uint32_t dtype, const uint32_t* tok, uint32_t n_vocab,
                         float* out, uint32_t n_embd, int* err, cudaStream_t st);
int argmax_blocks(uint32_t n);
cudaError_t argmax_launch(const float* x, uint32_t n, float* part_v, uint32_t* part_i, int* counter,
                          uint32_t* tok_out, uint32_t* pos_inc, cudaStream_t st);
cudaError_t rmsnorm_launch(const float* x, const float* w, float* y, uint32_t d, cudaStream_t st);
cudaError_t rope_launch(float* qk, uint32_t n_heads, uint32_t hd, const uint32_t* pos, float theta,
                        cudaStream_t st);
cudaError_t swiglu_launch(const float* g, const float* u, float* h, uint32_t n, cudaStream_t st);
cudaError_t add_launch(float* y, const float* x, uint32_t n, cudaStream_t st);

}  // namespace shk
