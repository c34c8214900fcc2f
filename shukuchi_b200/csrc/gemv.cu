// gemv.cu -- batch-1 Q4_K / Q6_K dequantise-matvec for sm_100a: the stand-alone
// kernel (one launch per fused projection), its planner and the plain-load
// fallback.  The device-side math, ring and work split are in gemv_dev.cuh.
//
// Reference semantics: op_matmul_q4_k / op_matmul_q6_k (engine/src/ops.c:266-314,
// 361-404).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_dev.cuh"

// Largest task (rg row groups x 2 rows) that keeps two rows per lane group.
#ifndef SHK_RL2_MAX_BYTES
#define SHK_RL2_MAX_BYTES 40960
#endif
// Blocks per K slice of a long row.
#ifndef SHK_KS_BLOCKS
#define SHK_KS_BLOCKS 32
#endif

namespace shk {
namespace {
using namespace gdev;

template <bool HAS4, bool HAS6>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + GEMV_MAX_STAGES;
  uint64_t* xbar = empty + GEMV_MAX_STAGES;
  uint64_t* xbars = reinterpret_cast<uint64_t*>(smem + SMEM_XBARS);
  int* done = reinterpret_cast<int*>(xbar + 1);
  volatile uint32_t* gen = reinterpret_cast<volatile uint32_t*>(done + GEMV_MAX_STAGES);
  float* red = reinterpret_cast<float*>(smem + 8 * (2 * GEMV_MAX_STAGES + 1) + 8 * GEMV_MAX_STAGES);
  uint8_t* xreg = smem + ((SMEM_HDR + 127) & ~127);
  const uint32_t K = a.k, NS = a.n_stages;
  XBuf xb;
  xb.xq = reinterpret_cast<int4*>(xreg);  // padded limb vectors, xpad(K/4) of them
  xb.xbs = reinterpret_cast<float*>(xreg + xq_bytes(K));
  xb.xs32 = xb.xbs + xbs_floats(K);
  size_t stage_off = (size_t)(xreg - smem) + x_region_bytes(K, HAS4, HAS6);
  stage_off = (stage_off + 127) & ~(size_t)127;
  const Ring R{full,           empty, done, gen, smem + stage_off, NS, a.stage_bytes,
               reinterpret_cast<float*>(smem + SMEM_KPART), reinterpret_cast<int*>(smem + SMEM_KCNT)};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tid = threadIdx.x;
  if (tid <= NS) {  // one thread per barrier pair, in parallel
    if (tid < NS) {
      mbar_init(&full[tid], 1);
      mbar_init(&empty[tid], 1);
      done[tid] = 0;
      gen[tid] = 0xFFFFFFFFu;
#pragma unroll
      for (int r = 0; r < GEMV_KS_ROWT; ++r) R.kcnt[tid * GEMV_KS_ROWT + r] = 0;
    } else {
      mbar_init(xbar, GEMV_WARPS);
      reinterpret_cast<int*>(red)[31] = 0;  // tensor-parallel producer: finished warps
    }
    fence_mbar_init();
  } else if (tid >= 32 * (GEMV_WARPS - 1) && tid < 32 * (GEMV_WARPS - 1) + GEMV_WARPS) {
    mbar_init(&xbars[tid - 32 * (GEMV_WARPS - 1)], 1);  // x copies of consumer warp tid - 448
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised
  pdl_trigger();    // the next kernel may be scheduled; it waits for this one before its reads

  const uint64_t lo = a.total_cost * blockIdx.x / gridDim.x;
  const uint64_t hi = a.total_cost * (blockIdx.x + 1) / gridDim.x;
  RingPos pos;
  if (warp == GEMV_WARPS) {
    // weights do not depend on the previous kernel: the first chunks stream in
    // while it drains
    if (lane == 0) {
      gemv_produce(a, R, pos, lo, hi, xbar);
      ring_drain(R, pos, a.err);
    }
    return;
  }
  NormPre np;
  gemv_norm_prefetch(a, warp, lane, np);
  pdl_wait();  // x and the residual come from the previous kernel
  gemv_x_issue(a, xb, warp, lane, xbars);
  const float osc = gemv_prologue<HAS4, HAS6>(a, xb, red, warp, lane, xbar, true, &np, xbars);
  uint32_t gtask = 0;
  gemv_consume<HAS4, HAS6>(a, R, pos, gtask, lo, hi, xb.view(osc), warp, lane);
  if (a.tp.out) gemv_tp_signal(a, reinterpret_cast<int*>(red + 31), lane);
}

// Tensor-parallel exchange sum as a kernel of its own (for a consumer that is
// not a staged GEMV): res_out = res_in + partials in rank order.
__global__ void tp_sum_kernel(const __grid_constant__ GemvTp t, const float* __restrict__ res_in, int* err) {
  __shared__ int ok;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    ok = 1;
    const uint32_t ep = __ldcg(t.epoch);
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t r = 0; r < t.world && ok; ++r)
      for (uint32_t n = 0; (int)(ld_acquire_sys(t.flags_in + r) - ep) < 0; ++n) {
        __nanosleep(64);
        if ((n & 31) == 31 && globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
          set_error(err, DERR_TIMEOUT_GRID);
          ok = 0;
          break;
        }
      }
  }
  __syncthreads();
  for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < t.d; k += gridDim.x * blockDim.x) {
    float v = __ldcg(res_in + k);
    for (uint32_t r = 0; r < t.world && ok; ++r)
      if (k >= t.cov_lo[r] && k < t.cov_hi[r]) v += __ldcg(t.parts_in + (size_t)r * t.d + k);
    t.res_out[k] = v;
  }
}

// --------------------------- generic fallback ---------------------------------
// One warp per row; plain byte loads; used only when rows are not 16-byte
// multiples (e.g. a raw Q6_K tensor whose row has an odd number of 8-block
// groups).  Same per-element dequantisation as the reference.
__global__ void gemv_generic_kernel(uint32_t qt, const uint8_t* __restrict__ w,
                                    const float* __restrict__ x, float* __restrict__ y,
                                    uint32_t m, uint32_t k) {
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const uint32_t nb = k / QK;
  float acc = 0.f;
  if (qt == T_Q4K) {
    const uint8_t* rp = w + (size_t)row * nb * Q4K_BYTES;
    for (uint32_t b = 0; b < nb; ++b) {
      const uint8_t* blk = rp + (size_t)b * Q4K_BYTES;
      const float d = ref_half(blk[0] | (blk[1] << 8)), dmin = ref_half(blk[2] | (blk[3] << 8));
      const uint8_t* sc = blk + 4;
      for (int e = lane; e < QK; e += 32) {
        const int g = e / 64, l = e % 64, sub = 2 * g + (l >= 32);
        const uint8_t qb = blk[16 + 32 * g + (l & 31)];
        const int q = (l >= 32) ? (qb >> 4) : (qb & 0xF);
        int s, mn;
        if (sub < 4) {
          s = sc[sub] & 63;
          mn = sc[sub + 4] & 63;
        } else {
          s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
          mn = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
        }
        acc = fmaf((d * s) * q - dmin * mn, x[b * QK + e], acc);
      }
    }
  } else {
    const uint8_t* rp = w + (size_t)row * nb * Q6K_BYTES;
    for (uint32_t b = 0; b < nb; ++b) {
      const uint8_t* blk = rp + (size_t)b * Q6K_BYTES;
      const float d = ref_half(blk[208] | (blk[209] << 8));
      for (int e = lane; e < QK; e += 32) {
        const int n = e / 128, r = e % 128, grp = r / 32, l = r % 32;
        const uint8_t* ql = blk + 64 * n;
        const uint8_t h = blk[128 + 32 * n + l];
        const uint8_t lq = (grp & 1) ? ql[l + 32] : ql[l];
        const int lo = (grp >= 2) ? (lq >> 4) : (lq & 0xF);
        const int q = (lo | (((h >> (2 * grp)) & 3) << 4)) - 32;
        const int s = (int8_t)blk[192 + 8 * n + l / 16 + 2 * grp];
        acc = fmaf((d * (float)s) * (float)q, x[b * QK + e], acc);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

}  // namespace

int gemv_plan(GemvPlan& p, const GemvMat* mats, int nmats, uint32_t k, const float* x,
              const float* norm_w, const uint32_t* pos, const float* rope_freq, int* err,
              int num_sms, uint32_t max_stage_bytes) {
  if (nmats < 1 || nmats > GEMV_MAX_SEGS || k == 0 || k % QK) return -1;
  GemvArgs& a = p.args;
  a = GemvArgs{};
  a.nseg = nmats;
  a.k = k;
  a.x = x;
  a.norm_w = norm_w;
  a.pos = pos;
  a.rope_freq = rope_freq;
  a.err = err;
  p.has4 = p.has6 = 0;
  const uint32_t nb = k / QK;
  const uint32_t target = max_stage_bytes;
  uint32_t stage = 0;
  uint64_t total = 0, units_total = 0;
  for (int i = 0; i < nmats; ++i) {
    const GemvMat& mt = mats[i];
    GemvSeg& g = a.seg[i];
    // the staged kernel reads Q4_K and planar Q6_K (GGUF-layout Q6_K goes
    // through repack.cu or the plain-load kernel)
    if (mt.qt != T_Q4K && mt.qt != T_Q6K_PLANAR) return -2;
    const uint32_t bb = mt.qt == T_Q4K ? Q4K_BYTES : Q6K_BYTES;
    g.w = static_cast<const uint8_t*>(mt.w);
    g.w2 = static_cast<const uint8_t*>(mt.w2);
    g.y = mt.y;
    g.m = mt.m;
    g.nb = nb;
    g.row_stride = mt.row_stride ? mt.row_stride : nb * bb;
    if (g.row_stride % 16 || g.row_stride < nb * bb) return -3;
    if ((reinterpret_cast<uintptr_t>(g.w) & 15) || (g.w2 && (reinterpret_cast<uintptr_t>(g.w2) & 15)))
      return -3;
    g.qt = (uint8_t)(mt.qt == T_Q4K ? T_Q4K : T_Q6K);
    g.epi = mt.epi;
    g.dual = mt.w2 ? 1 : 0;
    if (g.dual != (mt.epi == EPI_SWIGLU)) return -1;
    g.rope_hd = mt.rope_hd;
    if (mt.epi == EPI_ROPE && (mt.rope_hd == 0 || (mt.rope_hd & 1) || !pos || !rope_freq)) return -1;
    // rg: row groups per warp task so that every lane has a block to work on;
    // rl: output rows per lane group (2 rows, or 1 row / one gate-up pair).
    uint32_t rg = 1;
    const uint32_t mats_per_row = g.dual ? 2 : 1;
    // a lane per block: 32 block slots per warp
    if (mt.qt == T_Q4K)
      p.has4 = 1;
    else
      p.has6 = 1;
    while (rg * 2 <= 32 && rg * 2 * nb <= 32) rg *= 2;
    // Rows beyond 40 KB per task pair: one row per lane group (Q6_K has a
    // single-row body; for Q4_K the second row pointer repeats the first).
    uint32_t rl = g.dual ? 1 : 2;
    if (rl == 2 && (uint64_t)rg * 2 * g.row_stride > SHK_RL2_MAX_BYTES) rl = 1;
    if (mt.epi == EPI_ROPE && rl != 2) return -2;
    g.rg = (uint8_t)rg;
    g.rl = (uint8_t)rl;
    // rows of more than 32 blocks: one warp per slice of at most 32 blocks
    uint32_t ks = 1, lg_ks = 0;
    if (rg == 1)
      while (ks < (uint32_t)GEMV_KS_MAX && ks * SHK_KS_BLOCKS < nb) {
        ks *= 2;
        ++lg_ks;
      }
    g.ks = (uint8_t)ks;
    g.lg_ks = (uint8_t)lg_ks;
    g.sw = (uint16_t)((nb + ks - 1) / ks);
    g.unit_cost = rg * rl * g.row_stride * mats_per_row;
    uint32_t cu = std::max<uint32_t>(1, target / g.unit_cost);
    if (ks > 1) cu = std::min<uint32_t>(cu, GEMV_KS_ROWT);
    g.chunk_rows = cu * rg * rl;
    stage = std::max<uint32_t>(stage, cu * g.unit_cost);
    const uint64_t units = (mt.m + rg * rl - 1) / (rg * rl);
    total += units * g.unit_cost;
    units_total += units;
  }
  a.stage_bytes = (stage + 127) & ~127u;
  a.total_cost = total;
  size_t xbytes = (SMEM_HDR + 127) & ~(size_t)127;
  xbytes += x_region_bytes(k, p.has4, p.has6);
  xbytes = (xbytes + 127) & ~(size_t)127;
  const size_t budget = 227 * 1024;
  if (xbytes + 2 * (size_t)a.stage_bytes > budget) return -4;
  a.n_stages = (uint32_t)std::min<size_t>(GEMV_MAX_STAGES, (budget - xbytes) / a.stage_bytes);
  p.smem = xbytes + (size_t)a.n_stages * a.stage_bytes;
  p.grid = (int)std::min<uint64_t>((uint64_t)num_sms, units_total);
  if (p.grid < 1) p.grid = 1;
  return 0;
}

size_t gemv_x_region_bytes(uint32_t K, bool has4, bool has6) { return x_region_bytes(K, has4, has6); }

cudaError_t gemv_init() {
  const int mx = 227 * 1024;
  cudaError_t e = cudaFuncSetAttribute(gemv_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  return e;
}

cudaError_t gemv_launch(const GemvPlan& p, cudaStream_t stream) {
  if (p.args.total_cost == 0) return cudaSuccess;
  if (p.has4 && p.has6)
    return launch_k(gemv_kernel<true, true>, dim3(p.grid), dim3(GEMV_THREADS), p.smem, stream, p.args);
  if (p.has4)
    return launch_k(gemv_kernel<true, false>, dim3(p.grid), dim3(GEMV_THREADS), p.smem, stream, p.args);
  return launch_k(gemv_kernel<false, true>, dim3(p.grid), dim3(GEMV_THREADS), p.smem, stream, p.args);
}

cudaError_t gemv_tp_sum_launch(const GemvArgs& a, cudaStream_t st) {
  return launch_k(tp_sum_kernel, dim3((a.tp.d + 255) / 256), dim3(256), 0, st, a.tp, a.x, a.err);
}

cudaError_t gemv_generic_launch(uint32_t qt, const void* w, const float* x, float* y, uint32_t m,
                                uint32_t k, cudaStream_t stream) {
  if (m == 0) return cudaSuccess;
  const int rows_per_block = 8;
  gemv_generic_kernel<<<(m + rows_per_block - 1) / rows_per_block, 32 * rows_per_block, 0, stream>>>(
      qt, static_cast<const uint8_t*>(w), x, y, m, k);
  return cudaGetLastError();
}

}  // namespace shk
