// noalloc.cu -- first-index argmax that allocates no device memory.
//
// The context-based shk_cuda_argmax keeps its block partials in buffers that
// shk_cuda_init allocates.  Some callers cannot allocate at all: a sampler that
// runs inside a host runtime which has already reserved the device's memory
// in its own pool (a further cudaMalloc there fails or breaks the runtime's
// accounting), or code that is only handed device pointers and a stream and
// has no shk_ctx.  shk_cuda_argmax_noalloc serves them: its scratch is a
// fixed array in this library's device image, so every GPU that loads the
// library holds SCRATCH_BYTES of it until the process exits.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "glue.cuh"
#include "shk_cuda.h"

namespace {

// One (value, index) partial per argmax block, then the merge ticket.  The
// launch uses at most 148 blocks (argmax_blocks), so 256 slots cover every n.
constexpr uint32_t SLOTS = 256;
constexpr size_t VAL_OFF = 0;
constexpr size_t IDX_OFF = SLOTS * sizeof(float);
constexpr size_t CNT_OFF = IDX_OFF + SLOTS * sizeof(uint32_t);
constexpr size_t SCRATCH_BYTES = CNT_OFF + 256;  // 2304 bytes

// Host code must not pass this name to a kernel: on the host it is a stand-in,
// not a device address.  The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_argmax_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup_mu;
uint8_t* g_scratch_addr[MAX_DEVICES];  // per device ordinal, filled at first use

// Once per device, with that device current: look up the array's device address.
int scratch_for(int dev, uint8_t** out) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p) return SHK_ECUDA;
    g_scratch_addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_addr[dev];
  return SHK_OK;
}

}  // namespace

extern "C" int shk_cuda_argmax_noalloc(const float* x_dev, uint32_t n, uint32_t* out_dev,
                                       void* stream) {
  if (!x_dev || !out_dev || n == 0) return SHK_EINVAL;
  // Index 0xFFFFFFFF marks an empty partial inside the kernel.
  if (n > SHK_ARGMAX_NOALLOC_MAX_N) return SHK_EINVAL;
  if ((uint32_t)shk::argmax_blocks(n) > SLOTS) return SHK_EINVAL;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return SHK_ENODEV;
  if (dev < 0 || dev >= MAX_DEVICES) return SHK_EUNSUPPORTED;
  uint8_t* s = nullptr;
  const int rc = scratch_for(dev, &s);
  if (rc != SHK_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* counter = reinterpret_cast<int*>(s + CNT_OFF);
  // The array keeps the previous call's contents; the merge ticket must start at 0.
  if (cudaMemsetAsync(counter, 0, sizeof(int), st) != cudaSuccess) return SHK_ECUDA;
  if (shk::argmax_launch(x_dev, n, reinterpret_cast<float*>(s + VAL_OFF),
                         reinterpret_cast<uint32_t*>(s + IDX_OFF), counter, out_dev, nullptr,
                         st) != cudaSuccess)
    return SHK_ECUDA;
  return SHK_OK;
}
