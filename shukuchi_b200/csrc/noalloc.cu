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
#include <cuda.h>  // CUcontext (types only: the driver calls come through cudaGetDriverEntryPoint)
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

// A symbol's device address belongs to a CUDA context (the module is loaded
// per context), so the looked-up address is cached per context, keyed by the
// context's process-unique id (cuCtxGetId): a context created after
// cudaDeviceReset, or a caller's own driver context, gets its own look-up even
// if its handle value repeats.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

constexpr int CACHE = 64;
struct Entry {
  unsigned long long ctx_id;
  uint8_t* addr;
};
std::mutex g_setup_mu;
Entry g_cache[CACHE];
int g_cached = 0;
CtxGetCurrentFn g_get_current = nullptr;
CtxGetIdFn g_get_id = nullptr;

// Under the lock: the driver entry points, once per process.
bool driver_fns() {
  if (g_get_current && g_get_id) return true;
  void* f1 = nullptr;
  void* f2 = nullptr;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault) != cudaSuccess || !f1) return false;
  if (cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault) != cudaSuccess || !f2) return false;
  g_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
  g_get_id = reinterpret_cast<CtxGetIdFn>(f2);
  return true;
}

// The array's device address in the current context; looked up (with that
// context current) the first time the context is seen.
int scratch_for_current(uint8_t** out) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  // cudaFree(0) makes the runtime bind the device's primary context to this
  // thread if nothing is current yet (it frees nothing).
  if (cudaFree(nullptr) != cudaSuccess) return SHK_ECUDA;
  if (!driver_fns()) return SHK_ECUDA;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_get_current(&ctx) != CUDA_SUCCESS || !ctx) return SHK_ENODEV;
  if (g_get_id(ctx, &id) != CUDA_SUCCESS) return SHK_ECUDA;
  for (int i = 0; i < g_cached; ++i)
    if (g_cache[i].ctx_id == id) {
      *out = g_cache[i].addr;
      return SHK_OK;
    }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p) return SHK_ECUDA;
  // a full table starts over: entries of contexts long gone are the likely victims
  if (g_cached == CACHE) g_cached = 0;
  g_cache[g_cached++] = Entry{id, static_cast<uint8_t*>(p)};
  *out = static_cast<uint8_t*>(p);
  return SHK_OK;
}

}  // namespace

extern "C" int shk_cuda_argmax_noalloc(const float* x_dev, uint32_t n, uint32_t* out_dev,
                                       void* stream) {
  if (!x_dev || !out_dev || n == 0) return SHK_EINVAL;
  // Index 0xFFFFFFFF marks an empty partial inside the kernel.
  if (n > SHK_ARGMAX_NOALLOC_MAX_N) return SHK_EINVAL;
  if ((uint32_t)shk::argmax_blocks(n) > SLOTS) return SHK_EINVAL;
  uint8_t* s = nullptr;
  const int rc = scratch_for_current(&s);
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
