// attn.cu -- Q8_0 KV cache: layout, append / read kernels and the stand-alone
// decode attention kernels (device math in attn_dev.cuh and attn_split.cuh).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

#include "attn.cuh"
#include "attn_dev.cuh"
#include "attn_split.cuh"
#include "common.cuh"

namespace shk {

KvLayout kv_layout_make(uint32_t n_layers, uint32_t n_kv, uint32_t hd, uint32_t max_seq) {
  KvLayout L{};
  L.n_layers = n_layers;
  L.n_kv = n_kv;
  L.hd = hd;
  L.max_seq = max_seq;
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t q = (size_t)max_seq * hd, s = (size_t)max_seq * (hd / 32) * 4;
  L.kq_off = 0;
  L.ks_off = al(q);
  L.vq_off = L.ks_off + al(s);
  L.vs_off = L.vq_off + al(q);
  L.head_bytes = L.vs_off + al(s);
  return L;
}

size_t attn_part_floats(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t max_splits) {
  // [n_kv][max_splits][8][2] (max, sum) pairs, then [n_kv][max_splits][G][hd]
  // outputs: n_heads (= 8 * n_kv at most) * max_splits * (hd + 2) covers both
  return (size_t)n_heads * max_splits * (hd + 2);
}

namespace {
using namespace adev;

__global__ void kv_append_kernel(KvLayout kv, uint32_t layer, const uint32_t* pos_p,
                                 const float* k, const float* v, int* err) {
  const uint32_t pos = *pos_p;
  if (pos >= kv.max_seq) {
    if (threadIdx.x == 0) set_error(err, DERR_BAD_POS);
    return;
  }
  append_head(kv, layer, blockIdx.x, pos, k, v, threadIdx.x >> 5, threadIdx.x & 31, blockDim.x >> 5);
}

// n consecutive positions start.. in one launch: grid (n_kv, n); position i
// reads k/v rows at i * n_kv * hd.
__global__ void kv_append_range_kernel(KvLayout kv, uint32_t layer, uint32_t start,
                                       const float* k, const float* v) {
  const size_t off = (size_t)blockIdx.y * kv.n_kv * kv.hd;
  append_head(kv, layer, blockIdx.x, start + blockIdx.y, k + off, v + off, threadIdx.x >> 5,
              threadIdx.x & 31, blockDim.x >> 5);
}

constexpr int ATT_WARPS = 4;
constexpr int ATT_THREADS = 32 * ATT_WARPS;
// Caches of at least this many positions attend with the split kernel.
constexpr uint32_t ATT_SPLIT_CAPACITY = 4096;

template <int HD, int G>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  __shared__ __align__(16) float sm[AttnSmem<HD, G, ATT_WARPS>::FLOATS_LONG];
  pdl_trigger();
  pdl_wait();
  attn_item<HD, G, ATT_WARPS, true>(a, blockIdx.x, blockIdx.y, gridDim.y, sm);
}

__global__ void kv_read_range_kernel(KvLayout kv, uint32_t layer, uint32_t start, uint32_t end,
                                     float* k_out, float* v_out) {
  const uint32_t p = start + blockIdx.x;
  if (p >= end) return;
  const uint32_t vd = kv.n_kv * kv.hd, nblk = kv.hd / 32;
  for (uint32_t i = threadIdx.x; i < vd; i += blockDim.x) {
    const uint32_t h = i / kv.hd, e = i % kv.hd;
    const int8_t* reg = kv.region(layer, h);
    const float ks = reinterpret_cast<const float*>(reg + kv.ks_off)[(size_t)p * nblk + e / 32];
    const float vs = reinterpret_cast<const float*>(reg + kv.vs_off)[(size_t)p * nblk + e / 32];
    k_out[(size_t)(p - start) * vd + i] = (float)reg[kv.kq_off + (size_t)p * kv.hd + e] * ks;
    v_out[(size_t)(p - start) * vd + i] = (float)reg[kv.vq_off + (size_t)p * kv.hd + e] * vs;
  }
}

__global__ void kv_read_blocks_kernel(KvLayout kv, uint32_t layer, uint32_t start, uint32_t end,
                                      uint8_t* k_out, uint8_t* v_out) {
  const uint32_t p = start + blockIdx.x;
  if (p >= end) return;
  const uint32_t nblk = kv.hd / 32, tot = kv.n_kv * nblk;
  for (uint32_t i = threadIdx.x; i < tot * Q8_BYTES; i += blockDim.x) {
    const uint32_t blk = i / Q8_BYTES, byte = i % Q8_BYTES;
    const uint32_t h = blk / nblk, j = blk % nblk;
    const int8_t* reg = kv.region(layer, h);
    uint8_t kb, vb;
    if (byte < 4) {
      const uint8_t* ks = reinterpret_cast<const uint8_t*>(reg + kv.ks_off) + ((size_t)p * nblk + j) * 4;
      const uint8_t* vs = reinterpret_cast<const uint8_t*>(reg + kv.vs_off) + ((size_t)p * nblk + j) * 4;
      kb = ks[byte];
      vb = vs[byte];
    } else {
      kb = (uint8_t)reg[kv.kq_off + (size_t)p * kv.hd + 32 * j + byte - 4];
      vb = (uint8_t)reg[kv.vq_off + (size_t)p * kv.hd + 32 * j + byte - 4];
    }
    const size_t o = ((size_t)(p - start) * tot) * Q8_BYTES + i;
    k_out[o] = kb;
    v_out[o] = vb;
  }
}

constexpr int ATTC_WARPS = 8;
// Largest cluster the launcher may pick (16, 8 or 4).
#ifndef SHK_ATT_CLUSTER_CAP
#define SHK_ATT_CLUSTER_CAP 16
#endif

// One cluster per KV head (see attn_cluster in attn_dev.cuh).  LONG: the
// variant with the long-context loop (more registers), launched only for
// caches that can hold long contexts.
template <int HD, int G, bool LONG>
__global__ void __launch_bounds__(32 * ATTC_WARPS) attn_cluster_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(16) float smc[];
  pdl_trigger();
  attn_cluster<HD, G, ATTC_WARPS, LONG>(a, smc);
}

// How many clusters of 16, 8 and 4 CTAs of this kernel can be resident at
// once (0 where the size is refused).  Queried once per instantiation.
template <int HD, int G, bool LONG>
const int* cluster_capacity() {
  static int cap[3] = {-1, -1, -1};
  if (cap[0] >= 0) return cap;
  auto k = attn_cluster_kernel<HD, G, LONG>;
  const size_t smem = AttnCSmem<HD, G, ATTC_WARPS>::BYTES;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const bool np = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  const int sizes[3] = {16, 8, 4};
  for (int i = 0; i < 3; ++i) {
    cap[i] = 0;
    if (sizes[i] > 8 && !np) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sizes[i], 1);
    cfg.blockDim = dim3(32 * ATTC_WARPS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = sizes[i];
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess) cap[i] = n;
  }
  cudaGetLastError();  // a refused query leaves no sticky state
  return cap;
}

// The largest cluster with which all n_kv clusters (one per KV head) are
// resident together: a second wave would double the latency.
template <int HD, int G, bool LONG>
int cluster_ctas(uint32_t n_kv) {
  const int* cap = cluster_capacity<HD, G, LONG>();
  if (SHK_ATT_CLUSTER_CAP >= 16 && cap[0] >= (int)n_kv) return 16;
  if (SHK_ATT_CLUSTER_CAP >= 8 && cap[1] >= (int)n_kv) return 8;
  return 4;
}

template <int HD, int G, bool LONG>
cudaError_t attn_cluster_launch(const AttnArgs& a, cudaStream_t st) {
  const int cs = cluster_ctas<HD, G, LONG>(a.kv.n_kv);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, a.kv.n_kv);
  cfg.blockDim = dim3(32 * ATTC_WARPS);
  cfg.dynamicSmemBytes = AttnCSmem<HD, G, ATTC_WARPS>::BYTES;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cs;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  int n = 1;
  if (pdl_enabled()) {
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    n = 2;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, attn_cluster_kernel<HD, G, LONG>, a);
}

template <int HD, bool LONG>
cudaError_t attn_cluster_g(const AttnArgs& a, uint32_t G, cudaStream_t st) {
  switch (G) {
    case 1: return attn_cluster_launch<HD, 1, LONG>(a, st);
    case 2: return attn_cluster_launch<HD, 2, LONG>(a, st);
    case 4: return attn_cluster_launch<HD, 4, LONG>(a, st);
    case 8: return attn_cluster_launch<HD, 8, LONG>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

// The long-context variant whenever the cache can hold enough positions for
// a split of ATT_LONG_MIN positions per CTA (clusters have at least 4 CTAs).
template <int HD>
cudaError_t attn_cluster_hd(const AttnArgs& a, uint32_t G, cudaStream_t st) {
  return a.kv.max_seq >= 4 * ATT_LONG_MIN ? attn_cluster_g<HD, true>(a, G, st) : attn_cluster_g<HD, false>(a, G, st);
}

// Long caches: (KV head, split) CTAs with the split staged through shared
// memory, SPL_CLUSTER consecutive splits per thread-block cluster
// (attn_split.cuh); at most as many clusters as fit the GPU in one wave.
constexpr int SPL_CLUSTER = 8;

template <int HD, int G>
__global__ void __launch_bounds__(SPL_THREADS, 4) attn_split_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(128) uint8_t spl_smem[];
  pdl_trigger();
  pdl_wait();
  if (gridDim.z == 1) {
    attn_split_item<HD, G, SPL_CLUSTER>(a, blockIdx.x, blockIdx.y, gridDim.y, spl_smem);
  } else {  // sequence blockIdx.z of a batch
    AttnArgs b = a;
    const uint32_t z = blockIdx.z;
    b.layer = a.layer + z;
    b.q = a.q + z * a.qo_stride;
    b.out = a.out + z * a.qo_stride;
    if (a.k_new) {
      b.k_new = a.k_new + z * a.kv_stride;
      b.v_new = a.v_new + z * a.kv_stride;
    }
    b.part = a.part + z * a.part_stride;
    b.counters = a.counters + z * 8 * a.kv.n_kv;
    attn_split_item<HD, G, SPL_CLUSTER>(b, blockIdx.x, blockIdx.y, gridDim.y, spl_smem);
  }
}

// cudaErrorNotSupported: fewer than one cluster of splits per KV head fits
// (the caller then takes the single-level split kernel).
template <int HD, int G>
cudaError_t attn_split_go(const AttnArgs& a, cudaStream_t st) {
  auto k = attn_split_kernel<HD, G>;
  const int smem = SplitRing<HD>::BYTES;
  // per device, once: the shared-memory attribute and the co-resident cluster
  // count (a process may drive several GPUs, from several threads)
  static std::atomic<int> co_resident[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int clusters = (dev >= 0 && dev < 64) ? co_resident[dev].load() : 0;
  if (clusters == 0 && (e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
    return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.kv.n_kv, SPL_CLUSTER);
  cfg.blockDim = dim3(SPL_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = SPL_CLUSTER;
  at[0].val.clusterDim.z = 1;
  int n = 1;
  if (pdl_enabled()) {
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    n = 2;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  if (clusters == 0) {
    if ((e = cudaOccupancyMaxActiveClusters(&clusters, k, &cfg)) != cudaSuccess) return e;
    if (clusters > 0 && dev >= 0 && dev < 64) co_resident[dev].store(clusters);
  }
  const uint32_t n_seq = std::max<uint32_t>(1, a.n_seq);
  if (clusters < 1 || a.max_splits < (uint32_t)SPL_CLUSTER) return cudaErrorNotSupported;
  // one wave of clusters over the (KV head, sequence) pairs; with more pairs
  // than clusters, one cluster each (later waves wait for nothing)
  const uint32_t per_head = std::max<uint32_t>(
      1, std::min<uint32_t>(a.max_splits / SPL_CLUSTER, (uint32_t)clusters / (a.kv.n_kv * n_seq)));
  cfg.gridDim = dim3(a.kv.n_kv, per_head * SPL_CLUSTER, n_seq);
  return cudaLaunchKernelEx(&cfg, k, a);
}

template <int HD>
cudaError_t attn_split_hd(const AttnArgs& a, uint32_t G, cudaStream_t st) {
  switch (G) {
    case 1: return attn_split_go<HD, 1>(a, st);
    case 2: return attn_split_go<HD, 2>(a, st);
    case 4: return attn_split_go<HD, 4>(a, st);
    case 8: return attn_split_go<HD, 8>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

template <int HD>
cudaError_t attn_launch_hd(const AttnArgs& a, uint32_t G, cudaStream_t st) {
  dim3 grid(a.kv.n_kv, a.max_splits);
  switch (G) {
    case 1: return launch_k(attn_decode_kernel<HD, 1>, grid, dim3(ATT_THREADS), 0, st, a);
    case 2: return launch_k(attn_decode_kernel<HD, 2>, grid, dim3(ATT_THREADS), 0, st, a);
    case 4: return launch_k(attn_decode_kernel<HD, 4>, grid, dim3(ATT_THREADS), 0, st, a);
    case 8: return launch_k(attn_decode_kernel<HD, 8>, grid, dim3(ATT_THREADS), 0, st, a);
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t attn_decode_launch(const AttnArgs& a, cudaStream_t stream) {
  if (a.kv.n_kv == 0 || a.n_heads % a.kv.n_kv) return cudaErrorInvalidValue;
  if (a.min_per_split == 0) return cudaErrorInvalidValue;
  const uint32_t G = a.n_heads / a.kv.n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return cudaErrorInvalidValue;
  if (a.kv.hd != 64 && a.kv.hd != 128) return cudaErrorInvalidValue;
  AttnArgs b = a;
  if (a.k_new && ((reinterpret_cast<uintptr_t>(a.k_new) & 15) != 0)) {
    // the in-kernel new row reads 16-byte vectors: append first, then attend
    const cudaError_t e = kv_append_launch(a.kv, a.layer, a.pos, a.k_new, a.v_new, a.err, stream);
    if (e != cudaSuccess) return e;
    b.k_new = b.v_new = nullptr;
  }
  if (a.kv.max_seq >= ATT_SPLIT_CAPACITY && a.part && a.counters && a.max_splits > 0 &&
      a.max_splits <= (uint32_t)ATT_MAX_SPLITS) {
    // Long caches: the split kernel with the K/V staged through shared memory
    // and the splits merged per cluster (attn_split.cuh), on every SM.  (Short
    // caches stay on the one-cluster-per-KV-head kernel below: alone the
    // split kernel is faster there too -- 8.1 against 11.4 us at 512
    // positions -- but inside the 8B decode graph the cluster kernel, which
    // starts its cache loads before the dependency wait, gives the faster
    // token: 460 against 452 tok/s.)
    if ((reinterpret_cast<uintptr_t>(a.q) & 15) == 0) {  // q rows are read as 16-byte vectors
      AttnArgs c = b;
      c.min_per_split = std::max(a.min_per_split, SPL_MIN_PER_SPLIT);
      const cudaError_t e = a.kv.hd == 64 ? attn_split_hd<64>(c, G, stream) : attn_split_hd<128>(c, G, stream);
      if (e != cudaErrorNotSupported) return e;  // else not launched: the single-level split kernel
    }
    b.min_per_split = std::max(a.min_per_split, ATT_SPLIT_LONG);
    return a.kv.hd == 64 ? attn_launch_hd<64>(b, G, stream) : attn_launch_hd<128>(b, G, stream);
  }
  return a.kv.hd == 64 ? attn_cluster_hd<64>(b, G, stream) : attn_cluster_hd<128>(b, G, stream);
}

cudaError_t attn_decode_batch_launch(const AttnArgs& a, cudaStream_t stream) {
  if (a.kv.n_kv == 0 || a.n_heads % a.kv.n_kv || a.n_seq == 0) return cudaErrorInvalidValue;
  const uint32_t G = a.n_heads / a.kv.n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return cudaErrorInvalidValue;
  if (a.kv.hd != 64 && a.kv.hd != 128) return cudaErrorInvalidValue;
  if (a.layer + a.n_seq > a.kv.n_layers || !a.part || !a.counters || a.max_splits == 0 ||
      a.max_splits > (uint32_t)ATT_MAX_SPLITS)
    return cudaErrorInvalidValue;
  // 16-byte vectors: q rows and the new K/V rows of every sequence
  const bool al = (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && (a.qo_stride & 3) == 0 &&
                  (!a.k_new || ((reinterpret_cast<uintptr_t>(a.k_new) & 15) == 0 &&
                                (reinterpret_cast<uintptr_t>(a.v_new) & 15) == 0 && (a.kv_stride & 3) == 0));
  if (!al) return cudaErrorNotSupported;
  AttnArgs c = a;
  c.min_per_split = std::max(a.min_per_split, SPL_MIN_PER_SPLIT);
  return a.kv.hd == 64 ? attn_split_hd<64>(c, G, stream) : attn_split_hd<128>(c, G, stream);
}

cudaError_t kv_append_launch(const KvLayout& kv, uint32_t layer, const uint32_t* pos,
                             const float* k, const float* v, int* err, cudaStream_t stream) {
  kv_append_kernel<<<kv.n_kv, 128, 0, stream>>>(kv, layer, pos, k, v, err);
  return cudaGetLastError();
}

cudaError_t kv_append_range_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t n,
                                   const float* k, const float* v, cudaStream_t stream) {
  for (uint32_t done = 0; done < n;) {  // gridDim.y <= 65535
    const uint32_t c = std::min(n - done, 65535u);
    kv_append_range_kernel<<<dim3(kv.n_kv, c), 128, 0, stream>>>(
        kv, layer, start + done, k + (size_t)done * kv.n_kv * kv.hd,
        v + (size_t)done * kv.n_kv * kv.hd);
    done += c;
  }
  return cudaGetLastError();
}

cudaError_t kv_read_range_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t end,
                                 float* k_out, float* v_out, cudaStream_t stream) {
  if (end <= start) return cudaSuccess;
  kv_read_range_kernel<<<end - start, 256, 0, stream>>>(kv, layer, start, end, k_out, v_out);
  return cudaGetLastError();
}

cudaError_t kv_read_blocks_launch(const KvLayout& kv, uint32_t layer, uint32_t start, uint32_t end,
                                  uint8_t* k_out, uint8_t* v_out, cudaStream_t stream) {
  if (end <= start) return cudaSuccess;
  kv_read_blocks_kernel<<<end - start, 256, 0, stream>>>(kv, layer, start, end, k_out, v_out);
  return cudaGetLastError();
}

}  // namespace shk
