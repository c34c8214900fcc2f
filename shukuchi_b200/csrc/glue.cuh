// glue.cuh -- embedding, argmax and stand-alone glue kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace shk {

cudaError_t embed_launch(const void* table, uint32_t dtype, const uint32_t* tok, uint32_t n_vocab,
                         float* out, uint32_t n_embd, int* err, cudaStream_t st, uint32_t* step = nullptr);
int argmax_blocks(uint32_t n);
cudaError_t argmax_launch(const float* x, uint32_t n, float* part_v, uint32_t* part_i, int* counter,
                          uint32_t* tok_out, uint32_t* pos_inc, cudaStream_t st, uint32_t idx_off = 0,
                          float* val_out = nullptr);
// pairs: world x {value bits, global index}; writes the first maximum's index.
cudaError_t argmax_ranks_launch(const uint32_t* pairs, int world, uint32_t* tok_out, uint32_t* pos_inc,
                                cudaStream_t st);
cudaError_t rmsnorm_launch(const float* x, const float* w, float* y, uint32_t d, cudaStream_t st);
cudaError_t rope_launch(float* qk, uint32_t n_heads, uint32_t hd, const uint32_t* pos,
                        const float* freq, cudaStream_t st);
// freq[i/2] = powf(1/theta, i/head_dim) for even i (engine/src/ops.c:223-227),
// evaluated with the host C library.
void rope_freq_table(float theta, uint32_t head_dim, float* out);
cudaError_t swiglu_launch(const float* g, const float* u, float* h, uint32_t n, cudaStream_t st);
cudaError_t add_launch(float* y, const float* x, uint32_t n, cudaStream_t st);
// One bounded wait on an mbarrier that never completes (test of the timeout path).
cudaError_t wait_selftest_launch(int* err, uint64_t budget_ns, cudaStream_t st);

}  // namespace shk
