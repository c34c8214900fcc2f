// tp_ll.cuh -- one-shot tensor-parallel all-reduce over NVLink peer memory
// (flags in the data words); host-side API.  See tp_ll.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace shk {

constexpr int LL_MAX_RANKS = 8;

struct LlArgs {
  uint64_t* peer[LL_MAX_RANKS];  // every rank's exchange buffer [slot][rank][d] (own included)
  const uint32_t* epoch;         // device step counter (advanced by the embedding kernel)
  int* err;                      // device error word
  uint32_t rank, world, d;
};

// Bytes of one rank's exchange buffer for `slots` all-reduces per token.
inline size_t ll_buffer_bytes(uint32_t slots, uint32_t world, uint32_t d) {
  return (size_t)slots * world * d * sizeof(uint64_t);
}

// x[0..d) <- sum over ranks (rank order) of every rank's x, in place.
cudaError_t ar_ll_launch(const LlArgs& a, float* x, uint32_t slot, cudaStream_t st);

}  // namespace shk
