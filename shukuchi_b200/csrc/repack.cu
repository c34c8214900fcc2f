// repack.cu -- Q6_K rows between the GGUF block layout and the planar layout
// the staged GEMV reads (SHK_DTYPE_Q6_K_PLANAR).
//
// GGUF Q6_K (engine/src/ops.c:51-56): 210-byte blocks {ql[128], qh[64],
// int8 scales[16], fp16 d} back to back, so block b of a row starts at 210 b,
// a 2-byte boundary.  Planar: the same 210 nb bytes of a row regrouped into
// four planes,
//   ql     at 0        : block b's 128 bytes at 128 b,
//   qh     at 128 nb   : block b's  64 bytes at 128 nb + 64 b,
//   scales at 192 nb   : block b's  16 bytes at 192 nb + 16 b,
//   d      at 208 nb   : block b's   2 bytes at 208 nb + 2 b,
// every plane 16-byte aligned when the row is.  Inside a block the 16-byte
// chunks are rotated so that lanes working on consecutive blocks hit distinct
// shared-memory bank groups: ql chunk c of block b sits in slot (c + b) & 7 of
// the block's 128 bytes, qh chunk c in slot (c + (b >> 1)) & 3 of its 64.
// Only byte positions change; the bytes and the dequantisation do not.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"

namespace shk {
namespace {

// Byte offsets (within a row) of 16-byte chunk c (0-12) of block b: c < 8 is
// ql chunk c, 8..11 qh chunk c - 8, 12 the scales.
__device__ __forceinline__ void chunk_offsets(uint32_t nb, uint32_t b, uint32_t c, uint32_t& gguf,
                                              uint32_t& planar) {
  if (c < 8) {
    gguf = 210u * b + 16u * c;
    planar = 128u * b + 16u * ((c + b) & 7u);
  } else if (c < 12) {
    const uint32_t q = c - 8;
    gguf = 210u * b + 128u + 16u * q;
    planar = 128u * nb + 64u * b + 16u * ((q + (b >> 1)) & 3u);
  } else {
    gguf = 210u * b + 192u;
    planar = 192u * nb + 16u * b;
  }
}

// In place: a CTA takes whole rows; each row is read into shared memory, then
// written back in the other layout.  GGUF offsets are 2-byte aligned, so the
// copies move halfwords.
__global__ void q6k_repack_kernel(uint8_t* __restrict__ w, uint32_t rows, uint32_t nb, uint32_t stride,
                                  int to_planar) {
  extern __shared__ __align__(16) uint8_t row_s[];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    uint8_t* row = w + (size_t)r * stride;
    for (uint32_t i = threadIdx.x; i < stride / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(row_s)[i] = reinterpret_cast<const uint4*>(row)[i];
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < nb * 13u * 8u; i += blockDim.x) {
      const uint32_t h = i & 7u, cc = i >> 3, b = cc / 13u, c = cc % 13u;
      uint32_t g, p;
      chunk_offsets(nb, b, c, g, p);
      const uint32_t src = to_planar ? g : p, dst = to_planar ? p : g;
      *reinterpret_cast<uint16_t*>(row + dst + 2 * h) = *reinterpret_cast<const uint16_t*>(row_s + src + 2 * h);
    }
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      const uint32_t g = 210u * b + 208u, p = 208u * nb + 2u * b;
      *reinterpret_cast<uint16_t*>(row + (to_planar ? p : g)) =
          *reinterpret_cast<const uint16_t*>(row_s + (to_planar ? g : p));
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t q6k_repack_launch(void* w, uint32_t rows, uint32_t k, uint32_t stride, bool to_planar,
                              int num_sms, cudaStream_t st) {
  const uint32_t nb = k / QK;
  if (rows == 0) return cudaSuccess;
  if (k % QK || stride % 16 || stride < 210u * nb || stride > 227u * 1024u ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return cudaErrorInvalidValue;
  // per device (tensor-parallel ranks may share a process)
  const cudaError_t e =
      cudaFuncSetAttribute(q6k_repack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return e;
  const uint32_t grid = rows < 4u * (uint32_t)num_sms ? rows : 4u * (uint32_t)num_sms;
  q6k_repack_kernel<<<grid, 256, stride, st>>>(static_cast<uint8_t*>(w), rows, nb, stride, to_planar ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace shk
