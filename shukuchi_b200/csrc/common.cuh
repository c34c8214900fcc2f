// common.cuh -- shared device helpers for the sm_100a decode kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace shk {

constexpr int QK = 256;
constexpr int Q4K_BYTES = 144;
constexpr int Q6K_BYTES = 210;
constexpr int Q8_BYTES = 36;  // reference KV block {float scale; int8 q[32]}
constexpr int T_Q4K = 12;
constexpr int T_Q5K = 13;
constexpr int T_Q6K = 14;
constexpr int T_Q6K_PLANAR = 0x10E;  // Q6_K rows in the planar layout of repack.cu

// Device error codes written to the context's error word (first error wins).
constexpr int DERR_TIMEOUT_FULL = 1;   // consumer gave up waiting for a TMA stage
constexpr int DERR_TIMEOUT_EMPTY = 2;  // producer gave up waiting for a free stage
constexpr int DERR_BAD_POS = 3;        // position beyond the cache capacity
constexpr int DERR_BAD_TOKEN = 4;      // token id beyond the vocabulary
constexpr int DERR_TIMEOUT_GRID = 5;   // a CTA gave up waiting at a grid-wide barrier

// Wall-clock budget for any device-side wait (nanoseconds).  Waits in these
// kernels normally finish in microseconds; the budget only turns a broken
// invariant into an error status instead of a hung GPU.
constexpr uint64_t WAIT_BUDGET_NS = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// fp16 -> fp32 as the reference decodes it (engine/src/ops.c:58-91): exact for
// normals, zero, inf and NaN, but subnormals come out at half their IEEE value
// because the reference uses exponent 127-15-shift.  Scaling by 0.5 is exact.
__device__ __forceinline__ float ref_half(uint32_t h16) {
  float f = __half2float(__ushort_as_half((unsigned short)h16));
  return ((h16 & 0x7C00u) == 0u) ? f * 0.5f : f;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier + bulk async copy (TMA, 1-D, no tensor map, this CTA only) ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(n) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase parity.  Returns false (and records `code`) if the
// phase did not complete within WAIT_BUDGET_NS.
// The clock is read once per 32 polls and each unsuccessful poll backs off
// briefly, so waiting warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  int code, uint64_t budget_ns = WAIT_BUDGET_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(32);
    if ((n & 31) == 0 && globaltimer_ns() - t0 > budget_ns) {
      set_error(err, code);
      return false;
    }
  }
}
// Bounded wait without sleeping between polls: mbarrier.try_wait itself
// suspends the warp in hardware until the phase completes or a short time
// limit passes, so a waiter that is about to be released wakes at once.  For
// pipelines whose stages turn over every microsecond or so.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* err, int code,
                                               uint64_t budget_ns = WAIT_BUDGET_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 255) == 0 && globaltimer_ns() - t0 > budget_ns) {
      set_error(err, code);
      return false;
    }
  }
}
// cp.async.bulk global -> shared, completion signalled on `bar` as tx bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- small math helpers ----
__device__ __forceinline__ uint32_t lop_sel(uint32_t a, uint32_t b, uint32_t m) {
  // (a & m) | (b & ~m) in one LOP3
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(r) : "r"(a), "r"(b), "r"(m));
  return r;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float u2f_bits(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel in the
// stream is still running: pdl_trigger() lets the next kernel be scheduled,
// pdl_wait() blocks until every earlier kernel has completed and its memory is
// visible.  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Host: whether launches from this thread carry the attribute (set while a
// decode step is being captured into a graph).
bool& pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  if (pdl_enabled()) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace shk
