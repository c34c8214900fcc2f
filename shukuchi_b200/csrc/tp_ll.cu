// tp_ll.cu -- one-shot all-reduce of the tensor-parallel partial sums over
// NVLink peer memory, with flags carried in the data words.
//
// After the O and the down projection every rank holds a partial sum of the
// residual stream (rank 0's includes the residual itself); the layer's next
// step needs their sum on every rank (engine/src/engine.c:164-166, 218-220
// adds them on one device).  Each element travels as one 8-byte word
// {float bits, epoch}: every rank stores its words into slot `slot`, row
// `rank` of every rank's exchange buffer (plain 8-byte peer stores, single-copy
// atomic), then polls its own buffer until every rank's row carries this
// step's epoch and adds the rows in rank order -- the same order on every
// rank, so all ranks get the same bits.  No fence, flag or collective kernel
// separates the stores from the data: a word whose epoch matches is complete.
//
// A slot is written once per decoded token (2 per layer), and rank R can only
// write slot j of token s+1 after finishing slot j-1 of token s+1, which needs
// every rank's contribution to it, which each rank makes only after reading
// slot j of token s -- so no slot is overwritten before every rank has read it.
// The epoch is the device step counter the embedding kernel advances (1 for
// the first token), so zeroed buffers never match.  Waits are bounded.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "tp_ll.cuh"

namespace shk {
namespace {

__device__ __forceinline__ void st_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) ar_ll_kernel(const __grid_constant__ LlArgs a, float* x, uint32_t slot) {
  pdl_trigger();
  pdl_wait();  // the partial sums and the epoch come from earlier kernels
  const uint32_t e = *a.epoch;
  const uint32_t W = a.world, D = a.d;
  const size_t row = (size_t)D, base = (size_t)slot * W * row;
  // stores: this rank's row of the slot in every rank's buffer
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x) {
    const uint64_t w = (uint64_t)__float_as_uint(x[i]) | ((uint64_t)e << 32);
    for (uint32_t p = 0; p < W; ++p) st_sys_u64(a.peer[p] + base + (size_t)a.rank * row + i, w);
  }
  // loads: every rank's row from this rank's buffer, summed in rank order
  const uint64_t* mine = a.peer[a.rank] + base;
  bool ok = true;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (uint32_t r = 0; r < W; ++r) {
      uint64_t w = ld_sys_u64(mine + (size_t)r * row + i);
      if ((uint32_t)(w >> 32) != e) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t n = 1; ok && (uint32_t)((w = ld_sys_u64(mine + (size_t)r * row + i)) >> 32) != e; ++n)
          if ((n & 255) == 0 && globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
            set_error(a.err, DERR_TIMEOUT_GRID);
            ok = false;
          }
      }
      s += __uint_as_float((uint32_t)w);
    }
    x[i] = s;
    if (!ok) return;
  }
}

}  // namespace

cudaError_t ar_ll_launch(const LlArgs& a, float* x, uint32_t slot, cudaStream_t st) {
  const uint32_t blocks = (a.d + 255) / 256;
  return launch_k(ar_ll_kernel, dim3(blocks < 64 ? blocks : 64), dim3(256), 0, st, a, x, slot);
}

}  // namespace shk
