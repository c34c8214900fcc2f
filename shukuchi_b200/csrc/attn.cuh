// attn.cuh -- Q8_0 KV cache layout, quantise-on-append and split-K decode attention.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace shk {

// HBM layout of the Q8_0 KV cache.  One region per (layer, kv head) holding, for
// positions 0..max_seq-1: K quants [max_seq][hd] int8, K scales [max_seq][hd/32]
// fp32, then the same for V.  A (scale, 32 quants) pair is exactly one of the
// reference's 36-byte blocks (engine/src/kv_cache.c:7-10); blocks never straddle
// heads because hd is a multiple of 32.
struct KvLayout {
  int8_t* base;        // device allocation
  uint32_t n_layers, n_kv, hd, max_seq;
  size_t head_bytes;   // bytes of one (layer, kv head) region
  size_t kq_off, ks_off, vq_off, vs_off;  // offsets inside a region
  __host__ __device__ int8_t* region(uint32_t layer, uint32_t kvh) const {
    return base + ((size_t)layer * n_kv + kvh) * head_bytes;
  }
};

KvLayout kv_layout_make(uint32_t n_layers, uint32_t n_kv, uint32_t hd, uint32_t max_seq);

struct AttnArgs {
  KvLayout kv;
  uint32_t layer;
  uint32_t n_heads;
  float scale;              // 1/sqrt(hd)
  const float* q;           // n_heads * hd  (after RoPE)
  const float* k_new;       // n_kv * hd     (after RoPE), appended at *pos; null: no append
  const float* v_new;       // n_kv * hd
  const uint32_t* pos;      // device: position of the new token; attention covers [0, pos]
  float* out;               // n_heads * hd
  float* part;              // split partials: attn_part_floats(8 * n_kv, n_kv, hd, max_splits)
  int* counters;            // 8 * n_kv ints, zero between launches (self-resetting)
  uint32_t max_splits;
  uint32_t min_per_split;
  int* err;
  // several sequences in one launch (attn_decode_batch_launch): sequence z
  // attends cache layer `layer + z` with q / out at z * qo_stride floats,
  // k_new / v_new at z * kv_stride, partials at z * part_stride floats and
  // counters at z * 8 * n_kv; the position is shared
  uint32_t n_seq;
  size_t qo_stride, kv_stride, part_stride;
};

// Append + decode attention.  Caches of 4096 positions or more (with part /
// counters / max_splits >= 8 and q 16-byte aligned): the split kernel of
// attn_split.cuh (K/V staged through shared memory, tensor-core QK^T and PV,
// splits merged per thread-block cluster, then across clusters through
// `part`), else the single-level split kernel.  Shorter caches: one cluster
// per KV head (splits merged in distributed shared memory).
cudaError_t attn_decode_launch(const AttnArgs& a, cudaStream_t stream);
// n_seq sequences at the same position in one launch of the staged split
// kernel (a.n_seq and the strides set; q 16-byte aligned; part / counters
// sized for n_seq); cudaErrorNotSupported when that kernel cannot run.
cudaError_t attn_decode_batch_launch(const AttnArgs& a, cudaStream_t stream);
size_t attn_part_floats(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t max_splits);

// Quantise and store one token's K and V (engine/src/kv_cache.c:130-155).
cudaError_t kv_append_launch(const KvLayout& kv, uint32_t layer, const uint32_t* pos,
                             const float* k, const float* v, int* err, cudaStream_t stream);
// Dequantise positions [start, end) to fp32, reference order [pos][n_kv*hd]
// (engine/src/kv_cache.c:175-199).
cudaError_t kv_read_range_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t end,
                                 float* k_out, float* v_out, cudaStream_t stream);
// Export raw 36-byte blocks in the reference order [pos][n_kv*hd/32][36].
cudaError_t kv_append_range_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t n,
                                   const float* k, const float* v, cudaStream_t stream);
cudaError_t kv_read_blocks_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t end,
                                  uint8_t* k_out, uint8_t* v_out, cudaStream_t stream);

}  // namespace shk
