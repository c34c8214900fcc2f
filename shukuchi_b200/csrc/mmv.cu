// mmv.cu -- batch-1 Q4_K / Q6_K dequantise-matvec on the tensor cores over
// row-tiled weights: the stand-alone kernel, its planner and the GGUF -> tiled
// repack.  Device-side math, ring and reduction are in mmv_dev.cuh.
//
// Reference semantics: op_matmul_q4_k / op_matmul_q6_k (engine/src/ops.c:266-314,
// 361-404).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "mmv.cuh"
#include "mmv_dev.cuh"

namespace shk {
namespace {
using namespace mdev;

// Shared-memory map of the stand-alone kernel.
constexpr uint32_t SM_FULL = 0;
constexpr uint32_t SM_EMPTY = SM_FULL + 8 * MMV_MAX_STAGES;
constexpr uint32_t SM_XREADY = SM_EMPTY + 8 * MMV_MAX_STAGES;
constexpr uint32_t SM_RED = SM_XREADY + 64;
constexpr uint32_t SM_CNT = SM_RED + 64;
constexpr uint32_t SM_PART = (SM_CNT + 4 * MMV_RED_MAX_SLOTS + 127) & ~127u;
constexpr uint32_t SM_X = (SM_PART + 4 * MMV_RED_FLOATS + 127) & ~127u;
constexpr size_t SMEM_BUDGET = 227 * 1024;
// Blocks per item (K slice of a 16-row tile).
#ifndef SHK_MMV_SW
#define SHK_MMV_SW 2
#endif

template <bool HAS4, bool HAS6>
__global__ void __launch_bounds__(MMV_THREADS, 1) mmv_kernel(const __grid_constant__ MmvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SM_FULL);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + SM_EMPTY);
  uint64_t* xready = reinterpret_cast<uint64_t*>(smem + SM_XREADY);
  float* red = reinterpret_cast<float*>(smem + SM_RED);
  int* cnt = reinterpret_cast<int*>(smem + SM_CNT);
  float* part = reinterpret_cast<float*>(smem + SM_PART);
  const XRegion X = x_region(smem + SM_X, a.k, HAS4, HAS6);
  const size_t ring_off = (SM_X + x_bytes(a.k, HAS4, HAS6) + 127) & ~(size_t)127;
  const MRing R{full, empty, smem + ring_off, a.n_stages, a.stage_bytes, a.chunk, a.lg_chunk};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < (int)a.n_stages) {
    mbar_init(&full[tid], 1);
    mbar_init(&empty[tid], a.chunk);
    fence_mbar_init();
  } else if (tid == MMV_THREADS - 1) {
    mbar_init(xready, MMV_WARPS);
    fence_mbar_init();
  }
  for (int i = tid; i < MMV_RED_MAX_SLOTS; i += MMV_THREADS) cnt[i] = 0;
  __syncthreads();
  pdl_trigger();  // the next kernel may be scheduled; it waits for this one before its reads

  const uint32_t i0 = a.cta_item[blockIdx.x], i1 = a.cta_item[blockIdx.x + 1];
  if (warp == MMV_WARPS) {
    // weights do not depend on the previous kernel: they stream in while it drains
    if (lane == 0) {
      uint32_t nc = 0;  // chunks issued
      mmv_produce(a, R, i0, i1, nc, xready, 0);
      mmv_drain(R, nc, a.err);
    }
    return;
  }
  XPre np;
  x_norm_prefetch(a, warp, lane, np);
  pdl_wait();  // x and the residual come from the previous kernel
  const float osc = mmv_prologue<HAS4, HAS6>(a, X, red, warp, lane, &np);
  if (lane == 0) mbar_arrive(xready);
  mmv_consume<HAS4, HAS6>(a, R, i0, i1, 0, X, osc, part, cnt, warp, lane);
}

// ------------------------------ tiled repack -----------------------------------
// Source byte of tiled offset o (within a tile) for the tile's 16 rows: returns
// the row (0..15) and the byte offset inside that row's GGUF block.
__device__ __forceinline__ void tile_src(uint32_t qt, uint32_t o, uint32_t& r, uint32_t& src) {
  if (qt == T_Q4K) {
    if (o < 256) {
      r = o >> 4;
      src = o & 15u;
      return;
    }
    const uint32_t q = o - 256, j = q >> 9, rem = q & 511u, ln = rem >> 4, w = rem & 15u;
    r = (ln >> 2) + (w >= 8 ? 8u : 0u);
    src = 16u + 32u * j + 8u * (ln & 3u) + (w & 7u);
    return;
  }
  if (o < 3072) {
    const uint32_t n = o / 1536u, rem = o - 1536u * n, ln = rem / 48u, w = rem - 48u * ln;
    r = (ln >> 2) + (w >= 24 ? 8u : 0u);
    const uint32_t w2 = w % 24u, t = ln & 3u;
    src = w2 < 8 ? 64u * n + 8u * t + w2
                 : w2 < 16 ? 64u * n + 32u + 8u * t + (w2 - 8u) : 128u + 32u * n + 8u * t + (w2 - 16u);
  } else if (o < 3328) {
    r = (o - 3072u) >> 4;
    src = 192u + ((o - 3072u) & 15u);
  } else {
    r = (o - 3328u) >> 1;
    src = 208u + ((o - 3328u) & 1u);
  }
}

// One thread per output halfword (every run of the mapping is even-aligned and
// of even length, so a source halfword maps to an output halfword).
__global__ void tile_kernel(uint32_t qt, const uint8_t* __restrict__ src, uint32_t stride, uint32_t m,
                            uint32_t nb, uint8_t* __restrict__ dst, size_t n_half) {
  const uint32_t tb = qt == T_Q4K ? Q4T_BYTES : Q6T_BYTES, bb = qt == T_Q4K ? 144u : 210u;
  for (size_t h = (size_t)blockIdx.x * blockDim.x + threadIdx.x; h < n_half; h += (size_t)gridDim.x * blockDim.x) {
    const size_t o2 = 2 * h;
    const size_t tile = o2 / tb;
    const uint32_t o = (uint32_t)(o2 - tile * tb);
    const uint32_t t = (uint32_t)(tile / nb), b = (uint32_t)(tile - (size_t)t * nb);
    uint32_t r, so;
    tile_src(qt, o, r, so);
    const uint32_t row = 16u * t + r;
    uint16_t v = 0;
    if (row < m) v = *reinterpret_cast<const uint16_t*>(src + (size_t)row * stride + (size_t)b * bb + so);
    *reinterpret_cast<uint16_t*>(dst + o2) = v;
  }
}

}  // namespace

cudaError_t mmv_tile_launch(uint32_t qt, const void* src, uint32_t src_stride, uint32_t m, uint32_t k, void* dst,
                            cudaStream_t stream) {
  if (qt != T_Q4K && qt != T_Q6K) return cudaErrorInvalidValue;
  if (k == 0 || k % 256 || m == 0) return cudaErrorInvalidValue;
  const uint32_t nb = k / 256, bb = qt == T_Q4K ? 144u : 210u;
  const uint32_t stride = src_stride ? src_stride : nb * bb;
  if (stride < nb * bb || (stride & 1) || (reinterpret_cast<uintptr_t>(src) & 1) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return cudaErrorInvalidValue;
  const size_t n_half = mmv_tiled_bytes(qt, m, k) / 2;
  const int threads = 256;
  const size_t want = (n_half + threads - 1) / threads;
  const int grid = (int)std::min<size_t>(want, 148 * 32);
  tile_kernel<<<grid, threads, 0, stream>>>(qt, static_cast<const uint8_t*>(src), stride, m, nb,
                                            static_cast<uint8_t*>(dst), n_half);
  return cudaGetLastError();
}

// Items and ring geometry of a plan whose matrices are validated: K slices of
// sw blocks (sw the largest divisor of nb not above sw_target), item slots,
// chunk size and stage count.  0, or -4 when the ring does not fit `room`.
static int plan_items(MmvArgs& a, const MmvMat* mats, int nmats, uint32_t nb, uint32_t sw_target, size_t room,
                      uint32_t max_item_bytes, uint32_t& item0) {
  uint32_t slot = 0;
  item0 = 0;
  for (int i = 0; i < nmats; ++i) {
    const MmvMat& mt = mats[i];
    MmvSeg& g = a.seg[i];
    const uint32_t nm = mt.w2 ? 2 : 1;
    const uint32_t tb = mt.qt == T_Q4K_TILED ? Q4T_BYTES : Q6T_BYTES;
    // sw: the largest divisor of nb not above sw_target, raised to the
    // smallest divisor that keeps ks <= MMV_MAX_KS (items are whole, equal
    // slices, so an item's tiles start at item index x sw)
    uint32_t sw = 1;
    for (uint32_t d = 1; d <= nb; ++d)
      if (nb % d == 0 && d <= sw_target && (!max_item_bytes || d * tb * nm <= max_item_bytes)) sw = d;
    while (nb / sw > (uint32_t)MMV_MAX_KS) {
      ++sw;
      while (nb % sw) ++sw;
    }
    const uint32_t ks = nb / sw;
    g.w = static_cast<const uint8_t*>(mt.w);
    g.w2 = static_cast<const uint8_t*>(mt.w2);
    g.y = mt.y;
    g.m = mt.m;
    g.nb = nb;
    g.ntiles = (mt.m + 15) / 16;
    g.ks = (uint8_t)ks;
    g.sw = (uint16_t)sw;
    g.items = g.ntiles * ks;
    g.item0 = item0;
    g.qt = (uint8_t)(mt.qt == T_Q4K_TILED ? T_Q4K : T_Q6K);
    g.epi = mt.epi;
    g.dual = mt.w2 ? 1 : 0;
    g.rope_hd = mt.rope_hd;
    item0 += g.items;
    slot = std::max<uint32_t>(slot, sw * tb * nm);
  }
  a.stage_bytes = slot;  // tile bytes are 16-byte multiples
  uint32_t chunk = MMV_MAX_CHUNK, ns = 0;
  for (;; chunk >>= 1) {
    if (chunk == 0) return -4;
    ns = (uint32_t)std::min<size_t>(MMV_MAX_STAGES, room / ((size_t)chunk * slot));
    if (ns >= (MMV_WARPS + chunk - 1) / chunk + 2) break;
  }
  a.chunk = chunk;
  a.lg_chunk = (uint32_t)__builtin_ctz(chunk);
  a.n_stages = ns;
  // partial slots: items in flight never span red_slots indices
  bool any_dual = false;
  for (int i = 0; i < nmats; ++i) any_dual = any_dual || a.seg[i].dual;
  a.red_stride = any_dual ? 32u : 16u;
  a.red_slots = std::min<uint32_t>(MMV_RED_MAX_SLOTS, MMV_RED_FLOATS / a.red_stride);
  for (int i = 0; i < nmats; ++i)
    if (a.seg[i].ks + a.n_stages * chunk + MMV_WARPS + 1 >= a.red_slots) return -4;
  return 0;
}

int mmv_plan(MmvPlan& p, const MmvMat* mats, int nmats, uint32_t k, const float* x, const float* norm_w,
             const uint32_t* pos, const float* rope_freq, int* err, int num_sms, void* scratch,
             uint32_t max_item_bytes) {
  if (nmats < 1 || nmats > MMV_MAX_SEGS || k == 0 || k % 256 || num_sms < 1 || !scratch) return -1;
  // x and the norm weights are read as float4
  if (!x || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(norm_w) & 15)) return -1;
  MmvArgs& a = p.args;
  a = MmvArgs{};
  a.nseg = (uint32_t)nmats;
  a.k = k;
  a.x = x;
  a.norm_w = norm_w;
  a.pos = pos;
  a.rope_freq = rope_freq;
  a.err = err;
  a.xpart = static_cast<float*>(scratch);
  a.xcnt = reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + (size_t)(MMV_MAX_GRID + 1) * 2 * 32 * 4);
  const uint32_t nb = k / 256;
  bool has4 = false, has6 = false;
  for (int i = 0; i < nmats; ++i) {
    const MmvMat& mt = mats[i];
    if (mt.qt != T_Q4K_TILED && mt.qt != T_Q6K_TILED) return -2;
    if (!mt.w || (reinterpret_cast<uintptr_t>(mt.w) & 15) || (mt.w2 && (reinterpret_cast<uintptr_t>(mt.w2) & 15)))
      return -1;
    if ((mt.w2 != nullptr) != (mt.epi == EPI_SWIGLU)) return -1;
    if (mt.epi == EPI_TP) return -2;
    if (mt.epi == EPI_ROPE && (mt.rope_hd == 0 || (mt.rope_hd & 1) || !pos || !rope_freq)) return -1;
    if (mt.m == 0) return -1;
    (mt.qt == T_Q4K_TILED ? has4 : has6) = true;
  }
  a.has4 = has4;
  a.has6 = has6;
  const size_t fixed = ((SM_X + x_bytes(k, has4, has6) + 127) & ~(size_t)127);
  if (fixed >= SMEM_BUDGET) return -4;
  // Items: a row tile's K range cut into ks slices of sw blocks (SHK_MMV_SW,
  // default two; one where the ring has no room for two).  Slots hold the largest item (16-byte multiple; a dual
  // item's gate and up halves); a ring stage is a chunk of up to MMV_MAX_CHUNK
  // slots, and the ring needs ceil(MMV_WARPS / chunk) + 2 stages (parity
  // waits), so smaller chunks are used when x leaves little room.
  const size_t room = SMEM_BUDGET - fixed;
  // items of SHK_MMV_SW blocks where the ring takes them, else of one block
  uint32_t item0 = 0;
  int rc = -4;
  for (uint32_t sw_target : {(uint32_t)SHK_MMV_SW, 1u}) {
    rc = plan_items(a, mats, nmats, nb, sw_target, room, max_item_bytes, item0);
    if (rc == 0) break;
  }
  if (rc) return rc;
  // about 64 KB of weights per SM may go out before x has landed
  a.pre_items = std::max<uint32_t>(1, (64u * 1024u) / a.stage_bytes);
  const uint32_t total = item0;
  int grid = (int)std::min<uint32_t>((uint32_t)std::min(num_sms, MMV_MAX_GRID), total);
  // item start costs (bytes) and the first item of each item's row tile
  std::vector<uint64_t> start(total + 1);
  std::vector<uint32_t> rt_first(total), rt_end(total);
  uint64_t cost = 0;
  for (uint32_t s = 0; s < a.nseg; ++s) {
    const MmvSeg& g = a.seg[s];
    const uint32_t tb = g.qt == T_Q4K ? Q4T_BYTES : Q6T_BYTES;
    for (uint32_t li = 0; li < g.items; ++li) {
      const uint32_t sl = li % g.ks, nbs = std::min<uint32_t>(g.sw, g.nb - sl * g.sw);
      start[g.item0 + li] = cost;
      rt_first[g.item0 + li] = g.item0 + li - sl;
      rt_end[g.item0 + li] = g.item0 + li - sl + g.ks;
      cost += (uint64_t)nbs * tb * (g.dual ? 2 : 1);
    }
  }
  start[total] = cost;
  // CTA c starts at the first item whose start cost is >= cost * c / grid
  auto split_items = [&]() {
    uint32_t it = 0;
    for (int c = 0; c <= grid; ++c) {
      const uint64_t want = cost * (uint64_t)c / (uint64_t)grid;
      while (it < total && start[it] < want) ++it;
      a.cta_item[c] = c == grid ? total : it;
    }
  };
  // every CTA non-empty and no row tile over more than two CTAs
  auto valid = [&]() {
    for (int c = 0; c < grid; ++c) {
      const uint32_t i0 = a.cta_item[c], i1 = a.cta_item[c + 1];
      if (i0 >= i1) return false;
      if (rt_first[i0] < i0 && rt_end[i0] > i1) return false;
    }
    return true;
  };
  split_items();
  if (!valid()) {
    // boundaries only at row-tile starts, by cost
    std::vector<uint32_t> firsts;
    for (uint32_t i = 0; i < total; ++i)
      if (rt_first[i] == i) firsts.push_back(i);
    grid = (int)std::min<size_t>((size_t)grid, firsts.size());
    size_t f = 0;
    a.cta_item[0] = 0;
    for (int c = 1; c < grid; ++c) {
      const uint64_t want = cost * (uint64_t)c / (uint64_t)grid;
      // the first row-tile start at or after `want`, past the previous boundary,
      // leaving a row tile for each CTA still to come
      while (f < firsts.size() && (firsts[f] <= a.cta_item[c - 1] || start[firsts[f]] < want)) ++f;
      const size_t max_f = firsts.size() - (size_t)(grid - c);
      if (f > max_f) f = max_f;
      if (firsts[f] <= a.cta_item[c - 1]) return -4;
      a.cta_item[c] = firsts[f];
    }
    a.cta_item[grid] = total;
    if (!valid()) return -4;
  }
  p.grid = grid;
  a.grid = (uint32_t)grid;
  p.smem = fixed + (size_t)a.n_stages * a.chunk * a.stage_bytes;
  return 0;
}

cudaError_t mmv_init() {
  const int mx = (int)SMEM_BUDGET;
  cudaError_t e = cudaFuncSetAttribute(mmv_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(mmv_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(mmv_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  return e;
}

cudaError_t mmv_launch(const MmvPlan& p, cudaStream_t stream) {
  const MmvArgs& a = p.args;
  if (a.has4 && a.has6)
    return launch_k(mmv_kernel<true, true>, dim3(p.grid), dim3(MMV_THREADS), p.smem, stream, a);
  if (a.has4) return launch_k(mmv_kernel<true, false>, dim3(p.grid), dim3(MMV_THREADS), p.smem, stream, a);
  return launch_k(mmv_kernel<false, true>, dim3(p.grid), dim3(MMV_THREADS), p.smem, stream, a);
}

}  // namespace shk
