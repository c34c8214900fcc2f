// prefill.cu -- batched (prefill) dequantise-matmul on the 5th-generation
// tensor cores: Y[t][m] = sum_k W[m][k] * X[t][k] for a batch of T tokens,
// W in Q4_K or planar Q6_K blocks, X fp32, Y fp32.
//
// The reference has no batched path (engine/src/engine.c:306-501 feeds prompt
// tokens one at a time through op_matmul_q4_k / op_matmul_q6_k,
// engine/src/ops.c:266-314, 361-404); this is the dense contraction those
// per-token matvecs add up to, computed in f16 x f16 -> fp32: the weights
// dequantised to f16, each token's activations scaled by a power of two
// (its largest magnitude to [2^14, 2^15)) and rounded to f16, the scale put
// back in the epilogue -- 11 significant bits per operand where bf16 holds 8.
//
// Tile: one CTA per 128 weight rows x 256 tokens (tcgen05.mma M=128, N=256,
// cta_group::1, fp32 accumulator in 256 TMEM columns), optionally a half of K
// (split-K of two: both halves atomically added to a zeroed Y -- two addends,
// so the sum is the same in either order).  Warp roles (10 warps):
//   warp 8, lane 0  TMA: raw weight blocks (one 256-element block = four
//                   K-steps) into a 2-deep ring, and the f16 activation tile
//                   of each K-step (64 elements x 256 tokens, 128-byte swizzle:
//                   the tensor core's canonical K-major layout) into a 3-deep
//                   ring of A/B stages;
//   warps 0-7       dequantise the weight tile of each K-step from shared
//                   memory into f16 (two threads per row, 32 elements each),
//                   written in the same swizzled layout, then arrive;
//   warp 9, lane 0  issues the four K=16 MMAs of a step once both tiles are
//                   in, and commits them to the stage's "empty" barrier;
//   warps 0-3       epilogue: tcgen05.ld of the accumulator (warp w: TMEM
//                   lanes 32w..32w+31 = weight rows), stores coalesced along m.
// Every wait is bounded (1 s); a time-out records the error and sets a
// shared abort flag that ends every role's loop; the MMAs issued so far are
// still waited for (bounded) before the TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "gemv.cuh"

namespace shk {
namespace {

constexpr int PF_M = 128, PF_N = 256, PF_K = 64;
constexpr int PF_DQ_WARPS = 8;                     // dequantising warps (0-7)
constexpr int PF_TMA_WARP = 8, PF_MMA_WARP = 9;
constexpr int PF_THREADS = 32 * 10;
constexpr int PF_S = 3;                            // A/B stages
constexpr int PF_WS = 2;                           // raw weight block stages
constexpr int PF_TILE_A = PF_M * PF_K * 2;         // 16 KB
constexpr int PF_TILE_B = PF_N * PF_K * 2;         // 32 KB
constexpr int PF_WBLK = PF_M * 224;                // raw block of 128 rows (Q6_K planes: 128+64+16+16 B)
constexpr int PF_TMEM_COLS = PF_N;
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + PF_S * PF_TILE_A;
constexpr int OFF_W = OFF_B + PF_S * PF_TILE_B;
constexpr int OFF_BAR = OFF_W + PF_WS * PF_WBLK;
// barriers: a_full[S], b_full[S], ab_empty[S], w_full[WS], w_empty[WS], done
constexpr int PF_NBAR = 3 * PF_S + 2 * PF_WS + 1;
constexpr int OFF_MISC = OFF_BAR + 8 * PF_NBAR;    // TMEM address, abort flag
constexpr int PF_SMEM = 1024 + OFF_MISC + 16;
static_assert(PF_SMEM <= 227 * 1024, "prefill tile exceeds shared memory");

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: start address,
// leading byte offset 16 (unused for swizzled K-major), stride byte offset
// 1024 (8-row groups), descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B f16 (format
// 0 in bits 7-9 and 10-12), both K-major, N, M.
constexpr uint32_t PF_IDESC = (1u << 4) | ((uint32_t)(PF_N >> 3) << 17) | ((uint32_t)(PF_M >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(PF_IDESC), "r"(acc), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2-D tiled TMA load of box {x, y} into this CTA's shared memory only,
// completion as transaction bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Raw weight block in shared memory (128 rows): Q4_K [row][144 B]; planar Q6_K
// [ql: row][128 B] [qh: row][64 B] [scales: row][16 B] [d: row][16 B] (the d
// chunk holds the d of blocks 8*(b/8) .. 8*(b/8)+7).
constexpr int W6_QH = PF_M * 128, W6_SC = W6_QH + PF_M * 64, W6_D = W6_SC + PF_M * 16;

// 32 consecutive elements (half `h` of the 64-element quarter j of block b)
// of one weight row, dequantised with the reference's per-element formulas
// (dequantize_row_q4_k / dequantize_row_q6_k, engine/src/ops.c:117-193), as
// 16 f16 pairs.
template <int QT>
__device__ __forceinline__ void dequant32(const uint8_t* __restrict__ wblk, uint32_t r, uint32_t b, uint32_t j,
                                          uint32_t h, uint32_t (&out)[16]) {
  if (QT == T_Q4K) {
    const uint8_t* blk = wblk + r * Q4K_BYTES;
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
    const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * j);
    // 6-bit scale / min of sub-block `sub` (engine/src/ops.c:107-115)
    auto scb = [&](uint32_t i) -> uint32_t {
      const uint32_t wd = i < 4 ? hd.y : (i < 8 ? hd.z : hd.w);
      return (wd >> (8 * (i & 3))) & 0xFFu;
    };
    const uint32_t sub = 2 * j + h;
    uint32_t s, m;
    if (sub < 4) {
      s = scb(sub) & 63;
      m = scb(sub + 4) & 63;
    } else {
      s = (scb(sub + 4) & 0xF) | ((scb(sub - 4) >> 6) << 4);
      m = (scb(sub + 4) >> 4) | ((scb(sub) >> 6) << 4);
    }
    const float d1 = ref_half(hd.x & 0xFFFFu) * (float)s, m1 = ref_half(hd.x >> 16) * (float)m;
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t q = h ? (w[i] >> 4) : w[i];
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = __fsub_rn(__fmul_rn(d1, (float)((q >> (8 * e)) & 0xF)), m1);
      out[2 * i] = pack_f16(v[0], v[1]);
      out[2 * i + 1] = pack_f16(v[2], v[3]);
    }
  } else {  // planar Q6_K (repack.cu): chunk rotations as in the global layout
    const uint32_t n = j >> 1, g = 2 * (j & 1) + h;  // half, 32-element group
    const uint32_t qlc = 4 * n + 2 * (g & 1), qhc = 2 * n;
    const uint8_t* ql = wblk + r * 128;
    const uint8_t* qhp = wblk + W6_QH + r * 64;
    const uint4 a0 = *reinterpret_cast<const uint4*>(ql + 16 * ((qlc + b) & 7));
    const uint4 a1 = *reinterpret_cast<const uint4*>(ql + 16 * ((qlc + 1 + b) & 7));
    const uint4 h0 = *reinterpret_cast<const uint4*>(qhp + 16 * ((qhc + (b >> 1)) & 3));
    const uint4 h1 = *reinterpret_cast<const uint4*>(qhp + 16 * ((qhc + 1 + (b >> 1)) & 3));
    const int8_t* scp = reinterpret_cast<const int8_t*>(wblk + W6_SC + r * 16 + 8 * n + 2 * g);
    const float d = ref_half(*reinterpret_cast<const uint16_t*>(wblk + W6_D + r * 16 + 2 * (b & 7)));
    const float ds0 = d * (float)scp[0], ds1 = d * (float)scp[1];
    const uint32_t qv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = (g >= 2) ? (qv[i] >> 4) : qv[i];
      const uint32_t hi = hv[i] >> (2 * g);
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = (int)(((lo >> (8 * e)) & 0xF) | (((hi >> (8 * e)) & 3) << 4)) - 32;
        v[e] = (i < 4 ? ds0 : ds1) * (float)q;  // elements 0-15: first scale, 16-31: second
      }
      out[2 * i] = pack_f16(v[0], v[1]);
      out[2 * i + 1] = pack_f16(v[2], v[3]);
    }
  }
}

__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

struct PfMaps {
  CUtensorMap x;     // f16 scaled activations [T][K], box {64, 256}, 128-byte swizzle
  CUtensorMap w0;    // weights as bytes [M][row_stride]: Q4_K box {144, 128}; Q6_K box {128, 128}
  CUtensorMap w1;    // Q6_K box {64, 128}
  CUtensorMap w2;    // Q6_K box {16, 128}
};

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(32);
    if ((n & 31) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
        set_error(err, DERR_TIMEOUT_FULL);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

template <int QT>
__global__ void __launch_bounds__(PF_THREADS, 1)
    prefill_kernel(const __grid_constant__ PfMaps maps, float* __restrict__ y, const float* __restrict__ xs,
                   uint32_t M, uint32_t K, uint32_t T, uint32_t k_split, int* err) {
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* a_full = bars;
  uint64_t* b_full = bars + PF_S;
  uint64_t* ab_empty = bars + 2 * PF_S;
  uint64_t* w_full = bars + 3 * PF_S;
  uint64_t* w_empty = w_full + PF_WS;
  uint64_t* done = w_empty + PF_WS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t m0 = blockIdx.x * PF_M, t0 = blockIdx.y * PF_N;
  const uint32_t kspan = K / k_split, kbase = blockIdx.z * kspan;
  const uint32_t nk = kspan / PF_K, b0 = kbase / QK;
  const uint32_t nbg = K / QK;  // blocks per row

  if (tid == 0) {
    for (int s = 0; s < PF_S; ++s) {
      mbar_init(&a_full[s], PF_DQ_WARPS);
      mbar_init(&b_full[s], 1);
      mbar_init(&ab_empty[s], 1);
    }
    for (int s = 0; s < PF_WS; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], PF_DQ_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == PF_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(PF_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == PF_TMA_WARP) {
    if (lane == 0) {
      const uint32_t wbytes = QT == T_Q4K ? PF_M * Q4K_BYTES : PF_M * (128 + 64 + 16 + 16);
      for (uint32_t ks = 0; ks < nk && !*abort_flag; ++ks) {
        if ((ks & 3) == 0) {  // next raw weight block
          const uint32_t bl = ks >> 2, ws = bl % PF_WS;
          if (bl >= PF_WS && !pf_wait(&w_empty[ws], ((bl - PF_WS) / PF_WS) & 1, err, abort_flag)) break;
          uint8_t* wd = sm + OFF_W + ws * PF_WBLK;
          const uint32_t b = b0 + bl;
          mbar_expect_tx(&w_full[ws], wbytes);
          if (QT == T_Q4K) {
            tma_load_2d(wd, &maps.w0, (int)(b * Q4K_BYTES), (int)m0, &w_full[ws]);
          } else {
            tma_load_2d(wd, &maps.w0, (int)(128 * b), (int)m0, &w_full[ws]);
            tma_load_2d(wd + W6_QH, &maps.w1, (int)(128 * nbg + 64 * b), (int)m0, &w_full[ws]);
            tma_load_2d(wd + W6_SC, &maps.w2, (int)(192 * nbg + 16 * b), (int)m0, &w_full[ws]);
            tma_load_2d(wd + W6_D, &maps.w2, (int)(208 * nbg + 16 * (b >> 3)), (int)m0, &w_full[ws]);
          }
        }
        const uint32_t s = ks % PF_S;
        if (ks >= PF_S && !pf_wait(&ab_empty[s], ((ks - PF_S) / PF_S) & 1, err, abort_flag)) break;
        mbar_expect_tx(&b_full[s], PF_TILE_B);
        tma_load_2d(sm + OFF_B + s * PF_TILE_B, &maps.x, (int)(kbase + ks * PF_K), (int)t0, &b_full[s]);
      }
    }
  } else if (warp == PF_MMA_WARP) {
    if (lane == 0) {
      for (uint32_t ks = 0; ks < nk; ++ks) {
        const uint32_t s = ks % PF_S, par = (ks / PF_S) & 1;
        if (!pf_wait(&a_full[s], par, err, abort_flag) || !pf_wait(&b_full[s], par, err, abort_flag)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sm + OFF_A + s * PF_TILE_A), bb0 = smem_u32(sm + OFF_B + s * PF_TILE_B);
#pragma unroll
        for (uint32_t k4 = 0; k4 < PF_K / 16; ++k4)
          mma_f16(tmem, desc_sw128(a0 + 32 * k4), desc_sw128(bb0 + 32 * k4), (ks | k4) ? 1u : 0u);
        mma_commit(&ab_empty[s]);
      }
      mma_commit(done);  // arrives once every MMA issued above has completed
    }
  } else {  // warps 0-7: dequantise
    const uint32_t r = tid >> 1, h = tid & 1;
    for (uint32_t ks = 0; ks < nk; ++ks) {
      const uint32_t s = ks % PF_S, bl = ks >> 2, ws = bl % PF_WS;
      if ((ks & 3) == 0 && !pf_wait(&w_full[ws], (bl / PF_WS) & 1, err, abort_flag)) break;
      if (ks >= PF_S && !pf_wait(&ab_empty[s], ((ks - PF_S) / PF_S) & 1, err, abort_flag)) break;
      uint32_t v[16];
      dequant32<QT>(sm + OFF_W + ws * PF_WBLK, r, b0 + bl, ks & 3, h, v);
      uint8_t* A = sm + OFF_A + s * PF_TILE_A;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(A + sw128(r, 4 * h + c)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      proxy_fence();  // generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[s]);
        if ((ks & 3) == 3 || ks + 1 == nk) mbar_arrive(&w_empty[ws]);
      }
    }
  }

  // epilogue: warps 0-3 read the accumulator once every MMA has completed
  if (warp < 4) {
    const bool ok = pf_wait(done, 0, err, abort_flag) && !*abort_flag;
    tc_fence_after();
    if (__all_sync(0xffffffffu, ok)) {
      const uint32_t row = 32 * warp + lane, m = m0 + row;
#pragma unroll 1
      for (uint32_t cc = 0; cc < PF_N / 32; ++cc) {
        if (t0 + 32 * cc >= T) break;
        uint32_t v[32];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(tmem + ((32u * warp) << 16) + 32u * cc));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (m < M) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const uint32_t t = t0 + 32 * cc + jj;
            if (t < T) {
              const float r = __uint_as_float(v[jj]) * __ldg(xs + t);  // a power of two: exact
              if (k_split > 1)
                atomicAdd(&y[(size_t)t * M + m], r);
              else
                y[(size_t)t * M + m] = r;
            }
          }
        }
      }
    }
  } else if (warp == PF_MMA_WARP) {
    // on an abort the epilogue may not have waited: the TMEM is only freed
    // once the issued MMAs are done
    pf_wait(done, 0, err, abort_flag);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == PF_MMA_WARP)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS) : "memory");
}

// Token row blockIdx.x of x [T][k] -> f16 row of xb scaled by 2^s, s such that
// the row's largest magnitude lands in [2^14, 2^15) (|s| <= 100: the scaling
// stays exact in fp32); xs[t] = 2^-s undoes it in the epilogue.  A zero or
// non-finite row keeps s = 0.
__global__ void __launch_bounds__(256) to_f16_rows_kernel(const float* __restrict__ x, __half* __restrict__ xb,
                                                          float* __restrict__ xs, uint32_t k) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * k;
  __half* br = xb + (size_t)blockIdx.x * k;
  float mx = 0.f;
  for (uint32_t i = 2 * threadIdx.x; i < k; i += 2 * blockDim.x) {
    const float2 v = *reinterpret_cast<const float2*>(xr + i);
    mx = fmaxf(mx, fmaxf(fabsf(v.x), fabsf(v.y)));  // fmaxf drops NaN: checked below
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  int e = 0;
  if (mx > 0.f && isfinite(mx)) {
    frexpf(mx, &e);  // mx < 2^e <= 2 mx
    e = 15 - e;
    e = e > 100 ? 100 : (e < -100 ? -100 : e);
  }
  const float f = ldexpf(1.0f, e);
  if (threadIdx.x == 0) xs[blockIdx.x] = ldexpf(1.0f, -e);
  for (uint32_t i = 2 * threadIdx.x; i < k; i += 2 * blockDim.x) {
    const float2 v = *reinterpret_cast<const float2*>(xr + i);
    *reinterpret_cast<__half2*>(br + i) = __floats2half2_rn(v.x * f, v.y * f);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t es[2] = {1, 1};
  return encode_fn()(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// f16 rows, then one fp32 scale per token (k % 256 == 0: the scales start
// 512-byte aligned)
size_t prefill_x_bytes(uint32_t k, uint32_t n_tokens) { return (size_t)k * n_tokens * 2 + (size_t)n_tokens * 4; }

cudaError_t prefill_launch(uint32_t qt, const void* w, uint32_t row_stride, const float* x, void* xb_scratch,
                           float* y, uint32_t m, uint32_t k, uint32_t n_tokens, int* err, int num_sms,
                           cudaStream_t st) {
  if (!encode_fn()) return cudaErrorNotSupported;
  if (!n_tokens || k % QK) return cudaErrorInvalidValue;
  float* xs = reinterpret_cast<float*>(static_cast<uint8_t*>(xb_scratch) + (size_t)k * n_tokens * 2);
  to_f16_rows_kernel<<<n_tokens, 256, 0, st>>>(x, static_cast<__half*>(xb_scratch), xs, k);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PfMaps maps;
  bool ok = make_map(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xb_scratch, k, n_tokens, (uint64_t)k * 2, PF_K, PF_N,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (qt == T_Q4K) {
    ok = ok && make_map(&maps.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row_stride, m, row_stride, Q4K_BYTES, PF_M,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    maps.w1 = maps.w0;
    maps.w2 = maps.w0;
  } else {
    ok = ok && make_map(&maps.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row_stride, m, row_stride, 128, PF_M,
                        CU_TENSOR_MAP_SWIZZLE_NONE) &&
         make_map(&maps.w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row_stride, m, row_stride, 64, PF_M,
                  CU_TENSOR_MAP_SWIZZLE_NONE) &&
         make_map(&maps.w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row_stride, m, row_stride, 16, PF_M,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!ok) return cudaErrorInvalidValue;
  // split K in two when the row x token tiles alone would leave SMs idle
  const uint32_t gx = (m + PF_M - 1) / PF_M, gy = (n_tokens + PF_N - 1) / PF_N;
  const uint32_t ksplit = ((uint64_t)gx * gy < (uint64_t)num_sms && k % (2 * QK) == 0) ? 2 : 1;
  if (ksplit > 1) {
    e = cudaMemsetAsync(y, 0, (size_t)m * n_tokens * sizeof(float), st);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid(gx, gy, ksplit);
  if (qt == T_Q4K) {
    e = cudaFuncSetAttribute(prefill_kernel<T_Q4K>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
    if (e == cudaSuccess) prefill_kernel<T_Q4K><<<grid, PF_THREADS, PF_SMEM, st>>>(maps, y, xs, m, k, n_tokens, ksplit, err);
  } else {
    e = cudaFuncSetAttribute(prefill_kernel<T_Q6K_PLANAR>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
    if (e == cudaSuccess)
      prefill_kernel<T_Q6K_PLANAR><<<grid, PF_THREADS, PF_SMEM, st>>>(maps, y, xs, m, k, n_tokens, ksplit, err);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace shk
